"""Tree-masked attention registered as a Hugging Face attention function.

The reference runs the verify pass through SDPA with a 4-D boolean mask
(``src/specfit/runtime/eagle3_tree.py:1243-1250``) and its speculator refuses
any model whose ``config._attn_implementation`` is not ``"sdpa"``
(``eagle3_tree.py:922-923``).  ``install`` keeps that contract: the model's
config still reads ``"sdpa"`` (so Hugging Face prepares SDPA-style masks and
the reference speculator accepts the model), while every decoder layer's
attention module holds a config view whose implementation is ``ATTN_IMPL``,
under which ``tree_attention_forward`` is registered.  ``Qwen3MoeAttention``
(transformers/models/qwen3_moe/modeling_qwen3_moe.py:172-186) looks its
attention function up from its own ``self.config``, so it calls
``sf_tree_attention`` with the same inputs SDPA would get: query
``[B, Hq, T, D]``, key/value ``[B, Hkv, Tk, D]`` after the cache update, and
the mask as prepared by the caller (a 4-D mask is passed through unchanged).

The mask is packed once per mask tensor into one bit per (query, key) — the
layout the kernel consumes — and reused by every layer of the forward pass.
A missing mask means causal attention over the new tokens after the whole
cached prefix (prefill and plain decode).
"""
from __future__ import annotations

import copy
import weakref

import torch

from .. import ops

ATTN_IMPL = "specfit_b200_tree"

_pack_cache: dict = {}


def _packed_bits(mask: torch.Tensor, q_len: int, kv_len: int, batch: int):
    entry = _pack_cache.get("entry")
    if entry is not None:
        ref, version, shape, bits = entry
        if ref() is mask and version == mask._version and shape == (batch, q_len, kv_len):
            return bits
    m = mask
    if m.dtype != torch.bool:
        m = m > torch.finfo(m.dtype).min / 2
    m = m.expand(batch, 1, q_len, kv_len)
    bits = [ops.tree_bits_from_mask(m[b, 0], 0) for b in range(batch)]
    # One live mask at a time: every layer of a forward sees the same tensor.
    _pack_cache["entry"] = (weakref.ref(mask), mask._version, (batch, q_len, kv_len), bits)
    return bits


def clear_mask_cache() -> None:
    """Forget the packed mask, so the next forward packs its mask again (a
    CUDA-graph capture must record the packing, not reuse eager results)."""
    _pack_cache.clear()


_causal_cache: dict = {}


def _causal_bits(q_len: int, device) -> torch.Tensor:
    key = (q_len, str(device))
    hit = _causal_cache.get(key)
    if hit is None:
        hit = ops.tree_bits_from_parents(tuple(range(q_len - 1)), device)  # a chain
        _causal_cache[key] = hit
    return hit


def tree_attention_forward(module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                           attention_mask, scaling: float | None = None, dropout: float = 0.0,
                           **kwargs):
    if dropout:
        raise ValueError("tree attention is inference-only (dropout must be 0)")
    batch, hq, q_len, dim = query.shape
    kv_len = key.shape[2]
    out = torch.empty(batch, q_len, hq, dim, dtype=query.dtype, device=query.device)
    if attention_mask is None:
        bits = [_causal_bits(q_len, query.device)] * batch
        prefix = kv_len - q_len
    else:
        bits = _packed_bits(attention_mask, q_len, kv_len, batch)
        prefix = 0
    for b in range(batch):
        ops.tree_attention(query[b], key[b], value[b], bits[b], prefix, scale=scaling, out=out[b])
    return out, None


def register() -> str:
    from transformers import AttentionInterface

    AttentionInterface.register(ATTN_IMPL, tree_attention_forward)
    return ATTN_IMPL


def install(model) -> None:
    """Route the attention of every decoder layer of a Hugging Face Qwen3-MoE
    model (``model.model.layers[i].self_attn``) through ``sf_tree_attention``
    while ``model.config._attn_implementation`` stays ``"sdpa"``.

    The attention modules share one shallow copy of the model config that
    differs only in ``_attn_implementation``; everything else the modules
    read from it (head counts, dims, dropout) is the model's own value."""
    register()
    cfg = model.config
    if cfg._attn_implementation != "sdpa":
        cfg._attn_implementation = "sdpa"
    view = copy.copy(cfg)
    view._attn_implementation = ATTN_IMPL
    for layer in model.model.layers:
        layer.self_attn.config = view


def installed(model) -> bool:
    """Whether ``install`` routed ``model``'s attention to the tree kernel."""
    layers = model.model.layers
    return bool(layers) and all(
        getattr(l.self_attn.config, "_attn_implementation", None) == ATTN_IMPL for l in layers)
