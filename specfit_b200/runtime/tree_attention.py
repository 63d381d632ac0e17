"""Tree-masked attention registered as a Hugging Face attention function.

The reference runs the verify pass through SDPA with a 4-D boolean mask
(``src/specfit/runtime/eagle3_tree.py:1243-1250``; SDPA is required,
:922-923).  Registering ``tree_attention_forward`` under ``ATTN_IMPL`` makes
``Qwen3MoeAttention`` (transformers/models/qwen3_moe/modeling_qwen3_moe.py:
172-186) call ``sf_tree_attention`` instead, with the same inputs: query
``[B, Hq, T, D]``, key/value ``[B, Hkv, Tk, D]`` after the cache update, and
the mask as prepared by the caller (a 4-D mask is passed through unchanged).

The mask is packed once per mask tensor into one bit per (query, key) — the
layout the kernel consumes — and reused by every layer of the forward pass.
A missing mask means causal attention over the new tokens after the whole
cached prefix (prefill and plain decode).
"""
from __future__ import annotations

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
