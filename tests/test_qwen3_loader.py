"""Checkpoint reading of ``load_offloaded_qwen3`` on the CPU: the expert
pool packed from a saved Hugging Face checkpoint equals the model's own
expert weights (gate | up | down per expert), in both the fused layout that
transformers writes and the per-expert layout of released checkpoints, and
every other tensor is found as a non-expert parameter."""
import torch

from specfit_b200.runtime.qwen3_loader import (_Shards, checkpoint_files, is_expert_tensor,
                                               nonexpert_names, read_expert_layer)
from specfit_b200.runtime.qwen3_verifier import qwen3_moe_config

H, I, E, L = 64, 32, 4, 2


def tiny_model():
    from transformers import Qwen3MoeForCausalLM

    cfg = qwen3_moe_config(L, hidden=H, experts=E, top_k=2, moe_inter=I, heads=4, kv_heads=2,
                           head_dim=16, vocab=100)
    torch.manual_seed(0)
    m = Qwen3MoeForCausalLM(cfg).to(torch.bfloat16)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0, 0.02)
    return m


def packed_reference(m, layer):
    ex = m.model.layers[layer].mlp.experts
    gu = ex.gate_up_proj.detach().reshape(E, 2 * H * I)
    dn = ex.down_proj.detach().reshape(E, H * I)
    return torch.cat((gu, dn), dim=1)


def test_saved_checkpoint_packs_the_model_experts(tmp_path):
    m = tiny_model()
    m.save_pretrained(tmp_path, safe_serialization=True)
    files = checkpoint_files(tmp_path)
    shards = _Shards(files)
    for layer in range(L):
        out = torch.empty(E, 3 * H * I, dtype=torch.bfloat16)
        read_expert_layer(shards, layer, E, H, I, out)
        assert torch.equal(out, packed_reference(m, layer))
    names = nonexpert_names(files)
    expected = {n for n in m.state_dict() if ".mlp.experts." not in n}
    assert set(names) == expected


def test_per_expert_layout(tmp_path):
    from safetensors.torch import save_file

    m = tiny_model()
    tensors = {}
    for layer in range(L):
        ex = m.model.layers[layer].mlp.experts
        for e in range(E):
            gate, up = ex.gate_up_proj[e].detach().chunk(2, dim=0)
            base = f"model.layers.{layer}.mlp.experts.{e}"
            tensors[f"{base}.gate_proj.weight"] = gate.contiguous()
            tensors[f"{base}.up_proj.weight"] = up.contiguous()
            tensors[f"{base}.down_proj.weight"] = ex.down_proj[e].detach().contiguous()
    tensors["model.norm.weight"] = m.model.norm.weight.detach()
    save_file(tensors, str(tmp_path / "model.safetensors"))
    files = checkpoint_files(tmp_path)
    assert all(is_expert_tensor(n) for n in files if n != "model.norm.weight")
    shards = _Shards(files)
    for layer in range(L):
        out = torch.empty(E, 3 * H * I, dtype=torch.bfloat16)
        read_expert_layer(shards, layer, E, H, I, out)
        assert torch.equal(out, packed_reference(m, layer))
    assert nonexpert_names(files) == ["model.norm.weight"]
