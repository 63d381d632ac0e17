"""Numpy restatement of the verification-tree helpers and the tree-masked GQA
attention of the verify pass (TEST INFRASTRUCTURE ONLY).

* ``verification_position_ids`` / ``verification_attention_mask`` /
  ``accepted_path`` restate ``Eagle3DraftTree`` in
  ``src/specfit/runtime/eagle3_types.py:435-502``.
* ``tree_attention`` restates the attention of ``Qwen3MoeAttention.forward``
  (transformers/models/qwen3_moe/modeling_qwen3_moe.py:156-195) from the KV
  cache update onward: SDPA with the 4-D boolean tree mask, GQA by repeating
  each KV head over ``num_heads // num_kv_heads`` query heads, scale
  ``head_dim ** -0.5``.
"""
from __future__ import annotations

import numpy as np


def verification_position_ids(depths, base_kv_length: int) -> np.ndarray:
    """eagle3_types.py:435-448: seed at ``base``, node i at ``base + depth_i``."""
    if base_kv_length < 0:
        raise ValueError("base_kv_length must be non-negative")
    return np.array([base_kv_length] + [base_kv_length + d for d in depths], dtype=np.int64)


def verification_attention_mask(parent_ids, base_kv_length: int) -> np.ndarray:
    """eagle3_types.py:450-473: prefix fully visible; each query sees itself
    and its ancestors (node 0 is the pending seed)."""
    q = 1 + len(parent_ids)
    mask = np.zeros((q, base_kv_length + q), dtype=bool)
    mask[:, :base_kv_length] = True
    for node in range(q):
        a = node
        while True:
            mask[node, base_kv_length + a] = True
            if a == 0:
                break
            a = parent_ids[a - 1]
    return mask


def ancestor_bits(parent_ids) -> np.ndarray:
    """Per query row, the tree-part visibility as little-endian uint32 words
    (bit j of row i set when tree column j is visible); the layout the CUDA
    tree attention consumes."""
    q = 1 + len(parent_ids)
    words = (q + 31) // 32
    bits = np.zeros((q, words), dtype=np.uint32)
    tree = verification_attention_mask(parent_ids, 0)
    for i in range(q):
        for j in np.nonzero(tree[i])[0]:
            bits[i, j // 32] |= np.uint32(1) << np.uint32(j % 32)
    return bits


def accepted_path(parent_ids, token_ids, verifier_tokens) -> tuple:
    """eagle3_types.py:475-502: greedy walk from the seed through the child
    whose token equals the target's prediction at the parent."""
    verifier = [int(v) for v in verifier_tokens]
    if len(verifier) != 1 + len(token_ids):
        raise ValueError("verifier tokens do not match the draft tree")
    children: dict = {}
    for node, parent in enumerate(parent_ids, start=1):
        children.setdefault(parent, []).append(node)
    accepted = []
    parent = 0
    while True:
        predicted = verifier[parent]
        matching = [n for n in children.get(parent, ()) if token_ids[n - 1] == predicted]
        if not matching:
            break
        if len(matching) != 1:
            raise RuntimeError("target token matches multiple sibling nodes")
        parent = matching[0]
        accepted.append(parent)
    return tuple(accepted)


def tree_attention(q, k, v, mask, scale=None) -> np.ndarray:
    """Masked GQA attention in float64.

    ``q[Hq, Tq, D]``, ``k/v[Hkv, Tk, D]``, ``mask[Tq, Tk]`` (True = visible).
    Returns ``[Hq, Tq, D]`` float32."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    hq, tq, d = q.shape
    hkv = k.shape[0]
    group = hq // hkv
    scale = d ** -0.5 if scale is None else scale
    out = np.empty((hq, tq, d), dtype=np.float64)
    for h in range(hq):
        kh = k[h // group]
        vh = v[h // group]
        s = (q[h] @ kh.T) * scale
        s = np.where(mask, s, -np.inf)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[h] = p @ vh
    return out.astype(np.float32)
