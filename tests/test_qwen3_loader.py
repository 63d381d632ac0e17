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


# ---- packed-v1 checkpoints (fixture written by the reference's own packer) ----
import json
import shutil
from pathlib import Path

import pytest

from specfit_b200.runtime.qwen3_loader import (PackedCheckpointError, map_packed_layer,
                                               open_packed_checkpoint)

FIXTURE = Path(__file__).resolve().parent / "golden" / "packed_v1_tiny"


def test_packed_fixture_experts_equal_the_source_checkpoint():
    ck = open_packed_checkpoint(FIXTURE / "packed", verify_hashes=True,
                                source_metadata_root=FIXTURE / "source")
    assert (ck.num_layers, ck.num_experts, ck.hidden_size, ck.moe_intermediate_size) == (L, E, H, I)
    shards = _Shards(checkpoint_files(FIXTURE / "source"))
    for layer in range(L):
        want = torch.empty(E, 3 * H * I, dtype=torch.bfloat16)
        read_expert_layer(shards, layer, E, H, I, want)
        got = map_packed_layer(ck.layer_files[layer], E, 3 * H * I)
        assert torch.equal(got, want)


def test_packed_fixture_nonexperts_equal_the_source_checkpoint():
    from safetensors import safe_open

    ck = open_packed_checkpoint(FIXTURE / "packed")
    src = _Shards(checkpoint_files(FIXTURE / "source"))
    with safe_open(str(ck.nonexpert_file), framework="pt", device="cpu") as f:
        names = sorted(f.keys())
        assert names == nonexpert_names(src.files)
        for n in names:
            assert torch.equal(f.get_tensor(n), src.get(n))


def _copy_fixture(tmp_path):
    dst = tmp_path / "packed"
    shutil.copytree(FIXTURE / "packed", dst)
    return dst


def _edit_manifest(root, fn):
    m = json.loads((root / "manifest.json").read_text())
    fn(m)
    (root / "manifest.json").write_text(json.dumps(m))


@pytest.mark.parametrize("edit,match", [
    (lambda m: m.__setitem__("complete", False), "complete"),
    (lambda m: m.__setitem__("schema", "other"), "schema"),
    (lambda m: m.__setitem__("schema_version", 2), "version"),
    (lambda m: m["model"].__setitem__("expert_layout", ["up_proj", "gate_proj", "down_proj"]), "expert layout does not match"),
    (lambda m: m["model"].__setitem__("expert_dtype", "F16"), "unsupported packed expert dtype"),
    (lambda m: m["files"]["layers"].pop(), "layer file count does not match"),
    (lambda m: m["files"]["layers"][1].__setitem__("shape", [E, 3 * H * I + 8]), "layer tensor shape does not match"),
    (lambda m: m["files"]["layers"][1].__setitem__("layer_id", 0), "layer IDs must be contiguous"),
    (lambda m: m["files"]["layers"][0].__setitem__("filename", "nonexperts.safetensors"), "file names must be unique"),
    (lambda m: m["files"]["nonexperts"].__setitem__("size_bytes", 1), "file size does not match"),
    (lambda m: m["files"]["layers"][0].__setitem__("filename", "/etc/passwd"), "layer 0 file name must stay under root"),
    (lambda m: m["files"]["layers"][1].__setitem__("filename", "../x.safetensors"), "layer 1 file name must stay under root"),
    (lambda m: m["files"]["nonexperts"].__setitem__("filename", "."), "nonexperts file name must stay under root"),
    (lambda m: m["files"]["layers"][0].pop("filename"), "'filename' must be a nonempty string"),
    (lambda m: m["files"]["layers"][0].__setitem__("filename", 7), "'filename' must be a nonempty string"),
    (lambda m: m["files"]["nonexperts"].pop("size_bytes"), "'size_bytes' must be a positive integer"),
    (lambda m: m["files"]["nonexperts"].__setitem__("size_bytes", "12"), "'size_bytes' must be a positive integer"),
    (lambda m: m["files"]["layers"][1].__setitem__("size_bytes", True), "'size_bytes' must be a positive integer"),
    (lambda m: m["files"]["layers"][1].pop("sha256"), "'sha256' must be a nonempty string"),
    (lambda m: m["files"]["layers"][1].__setitem__("sha256", "AB" * 32), "'sha256' must be a lowercase SHA256"),
    (lambda m: m["files"]["layers"][1].__setitem__("sha256", "ab" * 31), "'sha256' must be a lowercase SHA256"),
    (lambda m: m["files"].__setitem__("nonexperts", []), "nonexperts file record must be an object"),
])
def test_packed_manifest_mismatches_are_refused(tmp_path, edit, match):
    root = _copy_fixture(tmp_path)
    _edit_manifest(root, edit)
    with pytest.raises(PackedCheckpointError, match=match):
        open_packed_checkpoint(root)


def test_packed_corruption_found_only_with_hash_verification(tmp_path):
    root = _copy_fixture(tmp_path)
    path = root / "experts" / "layer-001.safetensors"
    raw = bytearray(path.read_bytes())
    raw[-3] ^= 0x40  # a bit of the last expert's down rows; the size is unchanged
    path.write_bytes(bytes(raw))
    open_packed_checkpoint(root)  # sizes still match
    with pytest.raises(PackedCheckpointError, match="SHA256 does not match"):
        open_packed_checkpoint(root, verify_hashes=True)


def test_packed_source_config_must_match(tmp_path):
    src = tmp_path / "source"
    shutil.copytree(FIXTURE / "source", src)
    cfg = json.loads((src / "config.json").read_text())
    cfg["rms_norm_eps"] = 1e-5
    (src / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(PackedCheckpointError, match="source config SHA256 does not match"):
        open_packed_checkpoint(FIXTURE / "packed", source_metadata_root=src)


def test_packed_source_index_is_required(tmp_path):
    src = tmp_path / "source"
    shutil.copytree(FIXTURE / "source", src)
    (src / "model.safetensors.index.json").unlink()
    with pytest.raises(PackedCheckpointError, match="source config or index metadata is missing"):
        open_packed_checkpoint(FIXTURE / "packed", source_metadata_root=src)


def test_packed_source_index_must_match(tmp_path):
    src = tmp_path / "source"
    shutil.copytree(FIXTURE / "source", src)
    index = src / "model.safetensors.index.json"
    index.write_text(index.read_text() + "\n")
    with pytest.raises(PackedCheckpointError, match="source index SHA256 does not match"):
        open_packed_checkpoint(FIXTURE / "packed", source_metadata_root=src)


def test_packed_missing_manifest(tmp_path):
    with pytest.raises(PackedCheckpointError, match="missing"):
        open_packed_checkpoint(tmp_path)


@pytest.mark.gpu
def test_gpu_source_and_packed_loads_give_equal_logits():
    """The same checkpoint loaded from its Hugging Face files, from the packed
    copy in a pinned pool, and from the packed files mapped and registered in
    place gives bit-identical logits, with experts filled through the cache."""
    from transformers import DynamicCache

    from specfit_b200.runtime.qwen3_loader import load_offloaded_qwen3

    dev = torch.device("cuda:0")
    ctx = torch.randint(0, 100, (1, 12), generator=torch.Generator().manual_seed(3)).to(dev)
    variants = ({}, {"packed_checkpoint_root": FIXTURE / "packed", "packed_expert_backing": "pinned_copy"},
                {"packed_checkpoint_root": FIXTURE / "packed", "verify_packed_hashes": True})
    logits = []
    for kw in variants:
        loaded = load_offloaded_qwen3(FIXTURE / "source", device=dev, slots_per_layer=2, **kw)
        try:
            with torch.no_grad():
                cache = DynamicCache(config=loaded.model.config)
                out = loaded.model(input_ids=ctx, past_key_values=cache, use_cache=True)
            torch.cuda.synchronize()
            logits.append(out.logits[0].float().cpu())
            assert loaded.cache_stats()["h2d_submissions"] > 0
        finally:
            loaded.close()
    assert torch.isfinite(logits[0]).all()
    assert torch.equal(logits[0], logits[1])
    assert torch.equal(logits[0], logits[2])
    # Stock Hugging Face (SDPA attention, stock experts) on the same files.
    from transformers import Qwen3MoeForCausalLM

    ref = Qwen3MoeForCausalLM.from_pretrained(FIXTURE / "source", dtype=torch.bfloat16,
                                              attn_implementation="sdpa").to(dev).eval()
    with torch.no_grad():
        theirs = ref(input_ids=ctx, past_key_values=DynamicCache(config=ref.config),
                     use_cache=True).logits[0].float().cpu()
    assert (logits[0] - theirs).abs().max().item() <= 2e-2
    cos = torch.nn.functional.cosine_similarity(logits[0], theirs, dim=-1)
    assert cos.min().item() >= 0.999


@pytest.mark.gpu
def test_gpu_loaded_model_reads_sdpa_and_runs_the_tree_kernel():
    """The loaded model's config reports "sdpa" (the reference speculator's
    requirement, eagle3_tree.py:922-923) while every layer's attention calls
    the tree kernel; a 4-D tree mask gives the same logits as stock SDPA."""
    from transformers import DynamicCache, Qwen3MoeForCausalLM

    from specfit_b200.runtime.qwen3_loader import load_offloaded_qwen3
    from specfit_b200.runtime.tree_attention import installed

    dev = torch.device("cuda:0")
    loaded = load_offloaded_qwen3(FIXTURE / "source", device=dev, slots_per_layer=4)
    ref = Qwen3MoeForCausalLM.from_pretrained(FIXTURE / "source", dtype=torch.bfloat16,
                                              attn_implementation="sdpa").to(dev).eval()
    try:
        assert loaded.model.config._attn_implementation == "sdpa"
        assert installed(loaded.model)
        ctx = torch.randint(0, 100, (1, 9), generator=torch.Generator().manual_seed(5)).to(dev)
        ids = torch.tensor([[3, 17, 40, 41, 8]], device=dev)
        parents = (0, 1, 1, 2)  # seed row 0, nodes 1..4
        visible = torch.zeros(5, 9 + 5, dtype=torch.bool)
        visible[:, :9] = True
        for i in range(5):
            n = i
            while True:
                visible[i, 9 + n] = True
                if n == 0:
                    break
                n = parents[n - 1]
        mask = visible[None, None].to(dev)
        pos = torch.tensor([[9, 10, 11, 11, 12]], device=dev)
        outs = []
        for model in (loaded.model, ref):
            cache = DynamicCache(config=model.config)
            with torch.no_grad():
                model(input_ids=ctx, past_key_values=cache, use_cache=True)
                outs.append(model(input_ids=ids, attention_mask=mask, position_ids=pos,
                                  past_key_values=cache, use_cache=True).logits[0].float().cpu())
        assert (outs[0] - outs[1]).abs().max().item() <= 2e-2
        cos = torch.nn.functional.cosine_similarity(outs[0], outs[1], dim=-1)
        assert cos.min().item() >= 0.999
    finally:
        loaded.close()
