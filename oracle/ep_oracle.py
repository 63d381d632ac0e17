"""CPU restatement of the expert-parallel exchange (TEST INFRASTRUCTURE ONLY).

The reference has no expert parallelism (it is single-GPU by construction:
scripts/run_specfit_main_comparison.py:465 refuses more than one device), so
this restates the exchange as a permutation over the single-GPU expert
groups of ``moe_oracle.dispatch`` / ``moe_oracle.moe_experts``
(src/specfit/runtime/qwen3_offloaded_experts.py:98-164):

* ``send_pack``: rank r owns experts [r*E/W, (r+1)*E/W).  One row per
  (token, destination) pair with at least one route there, grouped by
  destination then token: [hidden bytes | int32 ids[K] | float32 w[K] | pad]
  with the local ids ascending (-1 padded, weights 0 padded).
* ``recv_group``: stable grouping of the received (pair, slot) positions by
  local expert, padding skipped; ``return_src`` lists the sorted row of each
  valid slot in (pair, slot) order.
* ``route_row``: where each (token, k) route's output lands in the rows
  returned to the source (grouped by rank, then token, then local id).

Used by the CPU (gloo) tests of the multi-rank flow and as the byte-exact
checker of the CUDA send/receive kernels.  Never imported by the product.
"""
from __future__ import annotations

import numpy as np


def row_bytes(elem_size: int, hidden: int, top_k: int) -> int:
    raw = hidden * elem_size + 8 * top_k
    return (raw + 15) // 16 * 16


def send_pack(hidden_bytes: np.ndarray, top_k_index: np.ndarray, top_k_weights: np.ndarray,
              num_experts: int, world: int):
    """Returns ``(rows uint8 [P, row_bytes], counts int64 [world, 2],
    route_row int32 [T*K])``.  ``hidden_bytes``: uint8 [T, H*elem_size]."""
    hb = np.ascontiguousarray(hidden_bytes, dtype=np.uint8)
    idx = np.asarray(top_k_index, dtype=np.int64)
    w = np.asarray(top_k_weights, dtype=np.float32)
    T, K = idx.shape
    if num_experts % world:
        raise ValueError("num_experts must be divisible by world")
    per = num_experts // world
    hbytes = hb.shape[1]
    rb = (hbytes + 8 * K + 15) // 16 * 16
    if idx.size and (idx.min() < 0 or idx.max() >= num_experts):
        raise ValueError("expert index out of range")
    owner = idx // per
    pairs = [[t for t in range(T) if (owner[t] == r).any()] for r in range(world)]
    routes = [int((owner == r).sum()) for r in range(world)]
    counts = np.array([[len(pairs[r]), routes[r]] for r in range(world)], dtype=np.int64)
    rows = np.zeros((sum(len(p) for p in pairs), rb), dtype=np.uint8)
    route_row = np.full(T * K, -1, dtype=np.int32)
    i, ret = 0, 0
    for r in range(world):
        for t in pairs[r]:
            ks = [k for k in range(K) if owner[t, k] == r]
            ks.sort(key=lambda k: int(idx[t, k]))
            ids = np.full(K, -1, dtype=np.int32)
            ws = np.zeros(K, dtype=np.float32)
            for j, k in enumerate(ks):
                ids[j] = idx[t, k] - r * per
                ws[j] = w[t, k]
                route_row[t * K + k] = ret + j
            ret += len(ks)
            rows[i, :hbytes] = hb[t]
            rows[i, hbytes: hbytes + 4 * K] = ids.view(np.uint8)
            rows[i, hbytes + 4 * K: hbytes + 8 * K] = ws.view(np.uint8)
            i += 1
    return rows, counts, route_row


def unpack_meta(rows: np.ndarray, hbytes: int, top_k: int):
    """(ids int32 [P, K], weights f32 [P, K]) of received rows."""
    r = np.ascontiguousarray(rows, dtype=np.uint8)
    ids = r[:, hbytes: hbytes + 4 * top_k].copy().view(np.int32).reshape(-1, top_k)
    ws = r[:, hbytes + 4 * top_k: hbytes + 8 * top_k].copy().view(np.float32).reshape(-1, top_k)
    return ids, ws


def recv_group(rows: np.ndarray, hbytes: int, top_k: int, local_experts: int):
    """Stable grouping of the received slots.  Returns ``counts, offsets,
    sorted_pos`` (valid positions p = pair*K + slot, ascending by (expert, p))
    and ``return_src``."""
    ids, _ = unpack_meta(rows, hbytes, top_k)
    flat = ids.reshape(-1).astype(np.int64)
    valid = np.nonzero(flat >= 0)[0]
    if valid.size and flat[valid].max() >= local_experts:
        raise ValueError("local expert id out of range")
    order = valid[np.argsort(flat[valid], kind="stable")]
    counts = np.bincount(flat[valid], minlength=local_experts).astype(np.int32)
    offsets = np.zeros(local_experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    inv = np.full(flat.size, -1, dtype=np.int32)
    inv[order] = np.arange(order.size, dtype=np.int32)
    return_src = inv[valid].astype(np.int32)  # valid positions ascend = (pair, slot) order
    return counts, offsets, order.astype(np.int32), return_src


def exchange(blocks_by_source):
    """Concatenate what each source sent to one destination, in rank order."""
    return np.concatenate(blocks_by_source, axis=0) if blocks_by_source else None
