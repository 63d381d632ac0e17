"""Numpy restatement of SpecFit's MoE verify block (TEST INFRASTRUCTURE ONLY).

This module is the CPU oracle: tests compare the CUDA path against it, and
``bench.py --impl reference`` times it (or the reference's PyTorch CPU
path).  The product package never imports it.

Each function cites the reference code it restates.  ``transformers/...``
means ``transformers/models/qwen3_moe/modeling_qwen3_moe.py`` (5.5.0 installed,
5.6.0 pinned by the reference); other paths are inside the SpecFit tree.

Numeric contract (shared with the CUDA kernels, so kernel == oracle is exact
for every integer output):

* Router logits: fp32 models use the exact dot product rounded once; bf16
  models sum the (exact) bf16*bf16 products in fp32 in the fixed order of the
  CUDA router (see ``router_logits``) and round once to bf16.  The reference's
  cuBLAS / MKL GEMM also accumulates in fp32 but in its own order, so its
  rounded logits can differ from these by one ulp; tests count such cases.
* Top-k is taken over the logits, ordered by (logit descending, expert id
  ascending).  Softmax is monotone, so this is the reference's
  ``topk(softmax(logits))`` (transformers/...:267-268) with the tie rule made
  explicit: among equal values the lower expert id wins.  The reference's own
  ``torch.topk`` leaves tie order implementation-defined.
"""
from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even), used to emulate the reference's bf16
# tensors on the CPU.


def bf16_round(values: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); returns float32."""
    a = np.ascontiguousarray(values, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def f64_to_bf16(values: np.ndarray) -> np.ndarray:
    """Round float64 values directly to bf16 (one rounding, ties to even);
    going through float32 first could round twice."""
    a = np.asarray(values, dtype=np.float64)
    mant, exp = np.frexp(a)  # a = mant * 2**exp, 0.5 <= |mant| < 1
    # bf16 keeps 8 significant bits: scale the mantissa to [128, 256).
    scaled = mant * 256.0
    rounded = np.rint(scaled)  # numpy rint is round-half-to-even
    out = np.ldexp(rounded / 256.0, exp)
    return out.astype(np.float32)


# ---------------------------------------------------------------------------
# K1: router (transformers/...:263-272, Qwen3MoeTopKRouter.forward)


def router_logits(x: np.ndarray, weight: np.ndarray, dtype: str) -> np.ndarray:
    """``F.linear(x, W)`` (transformers/...:265) in the model dtype.

    fp32: the exact dot product (fp64 sum of exact products) rounded once.
    bf16: exact bf16*bf16 products summed in fp32 in the order the CUDA router
    uses -- "lane" l = 0..31 adds positions h = 256 j + 8 l + v in (j, v)
    order, then the 32 lane sums are combined by an xor butterfly with offsets
    16, 8, 4, 2, 1 -- and rounded once to bf16 (RNE), i.e. an fp32-accumulated
    GEMM like the reference's, with a reproducible order."""
    if dtype == "f32":
        exact = np.asarray(x, dtype=np.float64) @ np.asarray(weight, dtype=np.float64).T
        return exact.astype(np.float32)
    if dtype != "bf16":
        raise ValueError(f"unsupported dtype {dtype!r}")
    xs = np.asarray(x, dtype=np.float32)
    ws = np.asarray(weight, dtype=np.float32)
    tokens, hidden = xs.shape
    experts = ws.shape[0]
    blocks = -(-hidden // 256)
    pad = blocks * 256 - hidden
    xr = np.pad(xs, ((0, 0), (0, pad))).reshape(tokens, blocks, 32, 8)
    wr = np.pad(ws, ((0, 0), (0, pad))).reshape(experts, blocks, 32, 8)
    out = np.empty((tokens, experts), dtype=np.float32)
    lanes = np.arange(32)
    for t0 in range(0, tokens, 64):  # bound the temporary size
        xt = xr[t0:t0 + 64]
        acc = np.zeros((xt.shape[0], experts, 32), dtype=np.float32)
        for j in range(blocks):
            for v in range(8):
                acc = acc + xt[:, None, j, :, v] * wr[None, :, j, :, v]  # exact products
        for off in (16, 8, 4, 2, 1):
            acc = acc + acc[..., lanes ^ off]
        out[t0:t0 + 64] = acc[..., 0]
    return bf16_round(out)


def softmax_f32(logits: np.ndarray) -> np.ndarray:
    """``softmax(logits, dtype=float32)`` over the expert axis (transformers/...:266)."""
    z = np.asarray(logits, dtype=np.float32)
    m = z.max(axis=-1, keepdims=True)
    e = np.exp(z - m, dtype=np.float32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def topk_lowest_id(values: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest values per row, ties broken by lower index."""
    v = np.asarray(values)
    e = v.shape[-1]
    order = np.lexsort((np.broadcast_to(np.arange(e), v.shape), -v.astype(np.float64)), axis=-1)
    return order[..., :k].astype(np.int64)


def router_topk(
    x: np.ndarray,
    weight: np.ndarray,
    top_k: int,
    norm_topk_prob: bool = True,
    dtype: str = "bf16",
):
    """Restates ``Qwen3MoeTopKRouter.forward`` (transformers/...:263-272).

    Returns ``(probs[T,E] f32, weights[T,K] f32, indices[T,K] int64, logits)``.
    ``probs`` is what the reference returns as ``router_logits`` (the softmax
    output); weights are the top-k probabilities, renormalised by their sum
    when ``norm_topk_prob`` (transformers/...:269-270) and kept in float32
    (transformers/...:271).
    """
    logits = router_logits(x, weight, dtype)
    probs = softmax_f32(logits)
    idx = topk_lowest_id(logits, top_k)
    top = np.take_along_axis(probs, idx, axis=-1).astype(np.float32)
    if norm_topk_prob:
        denom = np.zeros(top.shape[:-1] + (1,), dtype=np.float32)
        for j in range(top.shape[-1]):  # sequential fp32 sum in k order
            denom[..., 0] = (denom[..., 0] + top[..., j]).astype(np.float32)
        top = (top / denom).astype(np.float32)
    return probs, top, idx, logits


def boundary_ties(logits: np.ndarray, k: int) -> np.ndarray:
    """Rows whose k-th and (k+1)-th largest logits are equal (tie at the cut)."""
    s = -np.sort(-np.asarray(logits, dtype=np.float64), axis=-1)
    if s.shape[-1] <= k:
        return np.zeros(s.shape[:-1], dtype=bool)
    return s[..., k - 1] == s[..., k]


# ---------------------------------------------------------------------------
# K2: dispatch (qwen3_offloaded_experts.py:173-178 stable sort + grouping;
# the per-expert ``torch.where`` of :120-122 yields the same ascending order).


def dispatch(top_k_index: np.ndarray, num_experts: int):
    """Group the flattened routes by expert, stably.

    Returns ``counts[E]``, ``offsets[E+1]``, ``sorted_pos[T*K]`` (flattened
    route positions ``t*K+k`` in ascending (expert, position) order, i.e.
    ``torch.sort(top_k_index.reshape(-1), stable=True)``'s second output,
    qwen3_offloaded_experts.py:173), ``inv_pos`` (its inverse permutation)
    and ``active`` (experts with a non-empty group, ascending, padded with -1).
    """
    flat = np.asarray(top_k_index, dtype=np.int64).reshape(-1)
    if flat.size and (flat.min() < 0 or flat.max() >= num_experts):
        raise ValueError("expert index out of range")
    sorted_pos = np.argsort(flat, kind="stable").astype(np.int32)
    counts = np.bincount(flat, minlength=num_experts).astype(np.int32)
    offsets = np.zeros(num_experts + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    inv_pos = np.empty_like(sorted_pos)
    inv_pos[sorted_pos] = np.arange(sorted_pos.size, dtype=np.int32)
    active_ids = np.nonzero(counts)[0].astype(np.int32)
    active = np.full(num_experts, -1, dtype=np.int32)
    active[: active_ids.size] = active_ids
    return counts, offsets, sorted_pos, inv_pos, active, int(active_ids.size)


# ---------------------------------------------------------------------------
# K3: expert forward (qwen3_offloaded_experts.py:38-62) on a packed slot
# ``[gate(I*H) | up(I*H) | down(H*I)]`` (qwen3_packed_checkpoint.py:20-23).


def unpack_expert(packed: np.ndarray, hidden: int, inter: int):
    n = hidden * inter
    flat = np.asarray(packed).reshape(-1)
    if flat.size != 3 * n:
        raise ValueError(f"packed expert has {flat.size} elements, expected {3 * n}")
    gate = flat[:n].reshape(inter, hidden)
    up = flat[n : 2 * n].reshape(inter, hidden)
    down = flat[2 * n :].reshape(hidden, inter)
    return gate, up, down


def silu_f32(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, dtype=np.float32)
    return (v / (np.float32(1.0) + np.exp(-v, dtype=np.float32))).astype(np.float32)


def expert_forward(x_rows: np.ndarray, packed: np.ndarray, hidden: int, inter: int, dtype: str):
    """``_expert_forward`` (qwen3_offloaded_experts.py:38-62).

    In bf16 every torch op output is a bf16 tensor: the gate/up GEMM output
    (:60), ``silu(gate)`` and ``* up`` (:61), and the down GEMM (:62).  GEMMs
    accumulate in fp32 (fp64 here for the fp32 model).
    """
    gate, up, down = unpack_expert(packed, hidden, inter)
    x = np.asarray(x_rows, dtype=np.float32)
    if dtype == "bf16":
        g = bf16_round(x @ gate.astype(np.float32).T)
        u = bf16_round(x @ up.astype(np.float32).T)
        act = bf16_round(bf16_round(silu_f32(g)) * u)
        return bf16_round(act @ down.astype(np.float32).T)
    x64 = x.astype(np.float64)
    g = (x64 @ gate.astype(np.float64).T).astype(np.float32)
    u = (x64 @ up.astype(np.float64).T).astype(np.float32)
    act = (silu_f32(g) * u).astype(np.float32)
    return (act.astype(np.float64) @ down.astype(np.float64).T).astype(np.float32)


def weight_rows(values: np.ndarray, weights: np.ndarray, dtype: str) -> np.ndarray:
    """``values.mul_(w)`` (qwen3_offloaded_experts.py:132-138, :198): the
    product is formed in fp32 and stored back in the values' dtype."""
    prod = (np.asarray(values, np.float32) * np.asarray(weights, np.float32)[:, None]).astype(np.float32)
    return bf16_round(prod) if dtype == "bf16" else prod


def combine(
    contributions,
    tokens: int,
    hidden: int,
    dtype: str,
    order,
) -> np.ndarray:
    """Sequential ``index_add_`` of every expert's weighted rows in ``order``
    (canonical = ascending expert id, qwen3_offloaded_experts.py:155-163 and
    :200-202; arrival order = execution order, :144-149).  In bf16 every add
    rounds back to bf16."""
    out = np.zeros((tokens, hidden), dtype=np.float32)
    for expert_id in order:
        token_idx, values = contributions[expert_id]
        summed = (out[token_idx] + values).astype(np.float32)
        out[token_idx] = bf16_round(summed) if dtype == "bf16" else summed
    return out


def moe_experts(
    hidden_states: np.ndarray,
    top_k_index: np.ndarray,
    top_k_weights: np.ndarray,
    packed_experts,
    hidden: int,
    inter: int,
    dtype: str,
    order=None,
) -> np.ndarray:
    """``Qwen3OffloadedExperts.forward`` (qwen3_offloaded_experts.py:98-164).

    ``packed_experts`` maps expert id -> packed slot array.  ``order`` is the
    reduction order (``None`` = canonical ascending ids)."""
    idx = np.asarray(top_k_index, dtype=np.int64)
    w = np.asarray(top_k_weights, dtype=np.float32)
    x = np.asarray(hidden_states, dtype=np.float32)
    active = sorted(int(e) for e in np.unique(idx))
    contributions = {}
    for expert_id in active:
        token_idx, k_pos = np.nonzero(idx == expert_id)  # torch.where, :120-122
        y = expert_forward(x[token_idx], packed_experts[expert_id], hidden, inter, dtype)
        contributions[expert_id] = (token_idx, weight_rows(y, w[token_idx, k_pos], dtype))
    reduce_order = active if order is None else list(order)
    return combine(contributions, x.shape[0], hidden, dtype, reduce_order)


def moe_block(x, router_weight, packed_experts, hidden, inter, top_k, norm_topk_prob, dtype):
    """``Qwen3MoeSparseMoeBlock.forward`` (transformers/...:281-287) with the
    offloaded experts installed (qwen3_offloaded_model.py:597-606)."""
    probs, weights, idx, logits = router_topk(x, router_weight, top_k, norm_topk_prob, dtype)
    out = moe_experts(x, idx, weights, packed_experts, hidden, inter, dtype)
    return out, probs, weights, idx, logits
