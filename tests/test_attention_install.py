"""The attention routing keeps the reference speculator's SDPA contract.

``ShallowTreeSpeculator.__init__`` (src/specfit/runtime/eagle3_tree.py:
922-923) refuses a target whose ``config._attn_implementation`` is not
``"sdpa"``.  ``tree_attention.install`` routes the decoder layers to the tree
kernel through the attention modules' own config view, so the model config
still reads ``"sdpa"``.  These checks run on the CPU (no kernel is called):
the model is a tiny Qwen3-MoE on the meta device.
"""
import sys
from pathlib import Path

import pytest
import torch

REFERENCE_SRC = Path("/root/reference/src")


def _tiny_model():
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    cfg = Qwen3MoeConfig(vocab_size=64, hidden_size=32, intermediate_size=48, moe_intermediate_size=16,
                         num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                         num_experts=4, num_experts_per_tok=2, max_position_embeddings=64)
    cfg._attn_implementation = "sdpa"
    with torch.device("meta"):
        return Qwen3MoeForCausalLM(cfg)


def test_install_keeps_sdpa_on_the_model_config():
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    from specfit_b200.runtime.tree_attention import ATTN_IMPL, install, installed, tree_attention_forward

    model = _tiny_model()
    assert not installed(model)
    install(model)
    assert installed(model)
    assert model.config._attn_implementation == "sdpa"
    for layer in model.model.layers:
        view = layer.self_attn.config
        assert view is not model.config
        assert view._attn_implementation == ATTN_IMPL
        assert ALL_ATTENTION_FUNCTIONS.get_interface(view._attn_implementation, None) is tree_attention_forward
        for name in ("num_attention_heads", "num_key_value_heads", "hidden_size", "head_dim",
                     "attention_dropout", "rms_norm_eps"):
            assert getattr(view, name, None) == getattr(model.config, name, None)


@pytest.mark.skipif(not REFERENCE_SRC.is_dir(), reason="reference source tree not present")
def test_reference_speculator_accepts_an_installed_model():
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    try:
        import reference_shim
    finally:
        sys.path.pop(0)
    reference_shim.install(str(REFERENCE_SRC))
    from specfit.runtime.eagle3_tree import ShallowTreeSpeculator

    from specfit_b200.runtime.tree_attention import ATTN_IMPL, install

    class Drafter:
        layer_indices = (0, 1)

    model = _tiny_model()
    install(model)
    spec = ShallowTreeSpeculator(model, Drafter())
    assert spec.target is model
    # The previous wiring (the model config itself naming the kernel) is what
    # the reference refuses.
    model.config._attn_implementation = ATTN_IMPL
    with pytest.raises(ValueError, match="requires SDPA"):
        ShallowTreeSpeculator(model, Drafter())
