"""``load_offloaded_qwen3``: a real Qwen3-MoE checkpoint on the B200 path.

The reference loader (``src/specfit/runtime/qwen3_offloaded_model.py:667-840``)
reads a Hugging Face model directory (``config.json`` plus safetensors
shards), keeps every routed expert in page-locked host memory behind one
``GpuExpertCache`` per layer, and materialises the rest of the model on the
GPU.  This loader does the same for the B200 path: the expert weights of all
layers are packed into one ``ExpertHostPool`` (``[layers, experts, 3*H*I]``
bf16, ``gate | up | down`` rows -- the slot layout the kernels read), every
``layer.mlp`` becomes ``Qwen3B200SparseMoeBlock`` (router + offloaded
experts), and the non-expert parameters are copied to the device from the
shards.

Both expert layouts found in safetensors files are read: one tensor per
expert and projection (``...mlp.experts.{e}.{gate,up,down}_proj.weight``,
the released Qwen3-MoE checkpoints) and the fused per-layer tensors of
transformers 5 (``...mlp.experts.gate_up_proj [E, 2I, H]``, gate rows first,
and ``...mlp.experts.down_proj [E, H, I]``).

Not supported here: the reference's packed-v1 checkpoints and their
registered-mmap backing (``packed_checkpoint_root``); passing one raises
``ValueError``.
"""
from __future__ import annotations

import json
import re
from pathlib import Path

import torch

from .qwen3_offloaded_experts import ExpertExecutionPolicy, ReductionMode

_EXPERT_RE = re.compile(r"^model\.layers\.(\d+)\.mlp\.experts\.(?:(\d+)\.(gate_proj|up_proj|down_proj)\.weight"
                        r"|(gate_up_proj|down_proj))$")


def checkpoint_files(root) -> dict:
    """Tensor name -> safetensors file of a Hugging Face model directory
    (``model.safetensors.index.json`` when sharded, else the single
    ``model.safetensors``)."""
    root = Path(root)
    index = root / "model.safetensors.index.json"
    if index.exists():
        weight_map = json.loads(index.read_text())["weight_map"]
        return {name: root / fname for name, fname in weight_map.items()}
    single = root / "model.safetensors"
    if not single.exists():
        raise FileNotFoundError(f"no safetensors checkpoint under {root}")
    from safetensors import safe_open

    with safe_open(str(single), framework="pt", device="cpu") as f:
        return {name: single for name in f.keys()}


def is_expert_tensor(name: str) -> bool:
    return _EXPERT_RE.match(name) is not None


class _Shards:
    """Open safetensors files by path, reading tensors on the CPU."""

    def __init__(self, files: dict) -> None:
        self.files = files
        self._open: dict = {}

    def get(self, name: str) -> torch.Tensor:
        from safetensors import safe_open

        path = self.files[name]
        f = self._open.get(path)
        if f is None:
            f = self._open[path] = safe_open(str(path), framework="pt", device="cpu")
        return f.get_tensor(name)

    def __contains__(self, name: str) -> bool:
        return name in self.files


def read_expert_layer(shards: _Shards, layer: int, experts: int, hidden: int, inter: int,
                      out: torch.Tensor) -> None:
    """Pack layer ``layer``'s experts into ``out [experts, 3*H*I]``: per expert
    ``gate [I, H] | up [I, H] | down [H, I]`` flattened, cast to ``out``'s dtype."""
    hi = hidden * inter
    fused = f"model.layers.{layer}.mlp.experts.gate_up_proj"
    if fused in shards:
        gu = shards.get(fused)
        dn = shards.get(f"model.layers.{layer}.mlp.experts.down_proj")
        if gu.shape != (experts, 2 * inter, hidden) or dn.shape != (experts, hidden, inter):
            raise ValueError(f"layer {layer}: fused expert tensors have unexpected shapes")
        out[:, : 2 * hi].copy_(gu.reshape(experts, 2 * hi))
        out[:, 2 * hi:].copy_(dn.reshape(experts, hi))
        return
    for e in range(experts):
        base = f"model.layers.{layer}.mlp.experts.{e}"
        parts = []
        for proj, shape in (("gate_proj", (inter, hidden)), ("up_proj", (inter, hidden)),
                            ("down_proj", (hidden, inter))):
            name = f"{base}.{proj}.weight"
            if name not in shards:
                raise KeyError(f"checkpoint has no {name}")
            t = shards.get(name)
            if tuple(t.shape) != shape:
                raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {shape}")
            parts.append(t.reshape(-1))
        out[e].copy_(torch.cat(parts))


def nonexpert_names(files: dict) -> list:
    """Every checkpoint tensor that is not a routed expert weight."""
    return sorted(n for n in files if not is_expert_tensor(n))


def load_offloaded_qwen3(model_root, *, device, slots_per_layer: int, packed_checkpoint_root=None,
                         packed_expert_backing=None, verify_packed_hashes: bool = False,
                         reduction_mode=ReductionMode.CANONICAL,
                         expert_execution_policy=ExpertExecutionPolicy.EXPERT_ID_ASCENDING,
                         attn_implementation: str = "sdpa", cache_observer=None,
                         h2d_prefetch: bool = True):
    """Load a Hugging Face Qwen3-MoE directory as a ``LoadedOffloadedQwen3``
    (same arguments and validation as the reference's loader).  With
    ``attn_implementation="sdpa"`` (the reference's default and requirement
    for tree verification) attention runs on the tree-attention kernel; any
    other registered implementation name is passed to transformers."""
    from transformers import GenerationConfig, Qwen3MoeConfig, Qwen3MoeForCausalLM

    from .gpu_expert_cache import GpuExpertCache
    from .moe_block import Qwen3B200SparseMoeBlock, Qwen3B200TopKRouter
    from .qwen3_offloaded_experts import Qwen3OffloadedExperts
    from .qwen3_verifier import ExpertHostPool, LoadedB200Qwen3
    from .tree_attention import ATTN_IMPL, register as register_attention

    if type(h2d_prefetch) is not bool:
        raise ValueError("h2d_prefetch must be a boolean")
    policy = ExpertExecutionPolicy(expert_execution_policy)
    reduction = ReductionMode(reduction_mode)
    if packed_checkpoint_root is not None or packed_expert_backing not in (None, "pinned_copy"):
        raise ValueError("packed-v1 checkpoints (registered_mmap backing) are not supported by this loader")
    del verify_packed_hashes  # meaningful only for packed-v1 checkpoints
    root = Path(model_root).resolve()
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("offloaded Qwen3 requires a CUDA device")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    cfg = Qwen3MoeConfig.from_pretrained(root, local_files_only=True)
    if cfg.hidden_act != "silu":
        raise ValueError("P0 loader requires hidden_act='silu'")
    if not 1 <= slots_per_layer <= cfg.num_experts:
        raise ValueError(f"slots_per_layer must be in [1, {cfg.num_experts}]")
    if cfg.mlp_only_layers or getattr(cfg, "decoder_sparse_step", 1) != 1:
        raise ValueError("P0 loader requires an MoE block in every layer")
    if attn_implementation == "sdpa":
        register_attention()
        cfg._attn_implementation = ATTN_IMPL
    else:
        cfg._attn_implementation = attn_implementation

    files = checkpoint_files(root)
    shards = _Shards(files)
    L, E = cfg.num_hidden_layers, cfg.num_experts
    H, I = cfg.hidden_size, cfg.moe_intermediate_size
    pool = ExpertHostPool(L, E, 3 * H * I, torch.bfloat16)
    for layer in range(L):
        read_expert_layer(shards, layer, E, H, I, pool.data[layer])

    with torch.device("meta"):
        model = Qwen3MoeForCausalLM(cfg)
    caches = []
    for l, layer in enumerate(model.model.layers):
        cache = GpuExpertCache(pool.sources(l), slot_count=slots_per_layer, device=dev,
                               adopt_pinned_sources=True, observer=cache_observer)
        experts = Qwen3OffloadedExperts(layer_id=l, cache=cache, hidden_size=H, intermediate_size=I,
                                        reduction_mode=reduction, execution_policy=policy,
                                        h2d_prefetch=h2d_prefetch)
        gate = Qwen3B200TopKRouter(E, H, cfg.num_experts_per_tok, cfg.norm_topk_prob, device="meta")
        layer.mlp = Qwen3B200SparseMoeBlock(gate, experts)
        caches.append(cache)
    model.to_empty(device=dev)
    params = dict(model.named_parameters())
    names = nonexpert_names(files)
    missing = sorted(set(params) - set(names))
    if cfg.tie_word_embeddings and missing == ["lm_head.weight"]:
        missing = []
    if missing:
        raise KeyError(f"checkpoint lacks parameters: {missing[:5]}")
    with torch.no_grad():
        for name in names:
            if name not in params:
                continue  # e.g. buffers saved by other versions
            t = shards.get(name)
            p = params[name]
            if tuple(t.shape) != tuple(p.shape):
                raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(p.shape)}")
            p.data = t.to(device=dev, dtype=torch.bfloat16)
        if cfg.tie_word_embeddings:
            model.lm_head.weight = model.model.embed_tokens.weight
    # RoPE frequencies in fp32, built on the device (as a model loaded in bf16 keeps them).
    model.model.rotary_emb = type(model.model.rotary_emb)(config=cfg, device=dev)
    if (root / "generation_config.json").exists():
        model.generation_config = GenerationConfig.from_pretrained(root, local_files_only=True)
    model.requires_grad_(False)
    model.eval()
    torch.cuda.synchronize(dev)
    return LoadedB200Qwen3(model, tuple(caches), pool)
