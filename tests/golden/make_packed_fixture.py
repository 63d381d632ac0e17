"""Generate ``tests/golden/packed_v1_tiny/``: a tiny Qwen3-MoE checkpoint in
the released per-expert safetensors layout (``source/``) and its packed-v1
form (``packed/``) written by the SpecFit reference's own packer
(``pack_qwen3_checkpoint``, src/specfit/adapters/qwen3_packed_checkpoint.py:
650-790).

Run in a container where the reference source tree is available:

    python tests/golden/make_packed_fixture.py --reference /path/to/SpecFit

The source weights are drawn from a seeded CPU generator (2 layers, 4
experts, hidden 64, moe_intermediate 32, vocab 100, bf16); the whole fixture
is a few hundred KB.  The loader's packed-v1 reader is tested against it
(``tests/test_qwen3_loader.py``).
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

OUT = HERE / "packed_v1_tiny"
LAYERS, EXPERTS, HIDDEN, INTER, VOCAB = 2, 4, 64, 32, 100


def tiny_config():
    from specfit_b200.runtime.qwen3_verifier import qwen3_moe_config

    return qwen3_moe_config(LAYERS, hidden=HIDDEN, experts=EXPERTS, top_k=2, moe_inter=INTER, heads=4,
                            kv_heads=2, head_dim=16, vocab=VOCAB)


def write_source(root: Path) -> None:
    """Per-expert tensors (``...mlp.experts.{e}.{gate,up,down}_proj.weight``)
    and every non-expert tensor of the Hugging Face model, one shard plus the
    index, ``config.json`` from the model config."""
    from safetensors.torch import save_file
    from transformers import Qwen3MoeForCausalLM

    cfg = tiny_config()
    torch.manual_seed(20)
    model = Qwen3MoeForCausalLM(cfg).to(torch.bfloat16)
    tensors = {}
    with torch.no_grad():
        for name, p in model.state_dict().items():
            p.normal_(0.0, 0.02)
            if ".mlp.experts." not in name:
                tensors[name] = p.detach().clone().contiguous()
        for layer in range(LAYERS):
            ex = model.model.layers[layer].mlp.experts
            for e in range(EXPERTS):
                gate, up = ex.gate_up_proj[e].detach().chunk(2, dim=0)
                base = f"model.layers.{layer}.mlp.experts.{e}"
                tensors[f"{base}.gate_proj.weight"] = gate.contiguous().clone()
                tensors[f"{base}.up_proj.weight"] = up.contiguous().clone()
                tensors[f"{base}.down_proj.weight"] = ex.down_proj[e].detach().contiguous().clone()
    root.mkdir(parents=True)
    shard = "model-00001-of-00001.safetensors"
    save_file(tensors, str(root / shard), metadata={"format": "pt"})
    (root / "model.safetensors.index.json").write_text(json.dumps(
        {"metadata": {"total_size": sum(t.numel() * t.element_size() for t in tensors.values())},
         "weight_map": {name: shard for name in sorted(tensors)}}, indent=2, sort_keys=True) + "\n")
    cfg_dict = cfg.to_dict()
    cfg_dict["torch_dtype"] = "bfloat16"
    cfg_dict["architectures"] = ["Qwen3MoeForCausalLM"]
    (root / "config.json").write_text(json.dumps(cfg_dict, indent=2, sort_keys=True) + "\n")


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("SPECFIT_REFERENCE", ""),
                        help="root of the SpecFit reference source tree")
    args = parser.parse_args()
    if not args.reference:
        parser.error("--reference is required")
    import reference_shim

    reference_shim.install(str(Path(args.reference) / "src"))
    from specfit.adapters.qwen3_packed_checkpoint import pack_qwen3_checkpoint

    if OUT.exists():
        shutil.rmtree(OUT)
    write_source(OUT / "source")
    pack_qwen3_checkpoint(OUT / "source", OUT / "packed")
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
