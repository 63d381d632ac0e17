"""Torch-tensor front end of the native kernels.

Each function validates its tensors, allocates outputs and workspace with
torch's caching allocator (the C ABI itself never allocates), and enqueues the
kernel on the current CUDA stream.  Everything is asynchronous unless noted.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _native as N

_DTYPES = {torch.float32: N.SF_DTYPE_F32, torch.bfloat16: N.SF_DTYPE_BF16}

# Kernels of this library launched through this module (host-side count).
LAUNCHES = [0]


def _launched(n: int) -> None:
    LAUNCHES[0] += n


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if t.device.type != "cuda":
            raise ValueError("specfit_b200 ops need CUDA tensors")
        if t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


# ---------------------------------------------------------------------------
# K1 router


def router_topk(hidden: torch.Tensor, weight: torch.Tensor, top_k: int, norm_topk_prob: bool = True,
                return_logits: bool = False):
    """``Qwen3MoeTopKRouter.forward`` on the GPU.

    Returns ``(probs[T,E] f32, weights[T,K] f32, indices[T,K] int64)`` and,
    with ``return_logits``, the rounded logits in the model dtype."""
    dev = _require_cuda(hidden, weight)
    h = hidden.reshape(-1, hidden.shape[-1]).contiguous()
    w = weight.contiguous()
    if w.dtype != h.dtype:
        raise ValueError("router weight and hidden states must share a dtype")
    tokens, hid = h.shape
    experts = w.shape[0]
    if w.shape[1] != hid:
        raise ValueError("router weight width must equal the hidden size")
    probs = torch.empty(tokens, experts, dtype=torch.float32, device=dev)
    topw = torch.empty(tokens, top_k, dtype=torch.float32, device=dev)
    topi = torch.empty(tokens, top_k, dtype=torch.int64, device=dev)
    logits = torch.empty(tokens, experts, dtype=h.dtype, device=dev) if return_logits else None
    ws_bytes = N.lib.sf_router_topk_workspace_bytes(tokens, experts)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    N.check(
        N.lib.sf_router_topk(h.data_ptr(), w.data_ptr(), dtype_code(h.dtype), tokens, hid, experts,
                             top_k, int(bool(norm_topk_prob)), probs.data_ptr(), topw.data_ptr(),
                             topi.data_ptr(), _ptr(logits), ws.data_ptr(), ws_bytes, _stream(dev)),
        "sf_router_topk",
    )
    _launched(2)
    if return_logits:
        return probs, topw, topi, logits
    return probs, topw, topi


# ---------------------------------------------------------------------------
# K2 dispatch + gather


@dataclass
class Dispatch:
    counts: torch.Tensor  # [E] int32
    offsets: torch.Tensor  # [E+1] int32
    sorted_pos: torch.Tensor  # [T*K] int32
    inv_pos: torch.Tensor  # [T*K] int32
    active: torch.Tensor  # [E] int32, -1 padded
    num_active: torch.Tensor  # [1] int32
    error: torch.Tensor  # [1] int32
    tokens: int
    top_k: int
    num_experts: int


def moe_dispatch(top_k_index: torch.Tensor, num_experts: int,
                 active_total: torch.Tensor | None = None) -> Dispatch:
    """Stable grouping of the routes by expert; with ``active_total`` (a
    device int64 scalar) the launch also adds the number of active experts
    to it."""
    dev = _require_cuda(top_k_index)
    if top_k_index.dtype != torch.int64 or top_k_index.ndim != 2:
        raise ValueError("top_k_index must be int64 [tokens, top_k]")
    idx = top_k_index.contiguous()
    tokens, top_k = idx.shape
    n = tokens * top_k
    i32 = dict(dtype=torch.int32, device=dev)
    # One allocation for every int32 output keeps the host overhead low.
    buf = torch.empty(num_experts + (num_experts + 1) + 2 * n + num_experts + 2, **i32)
    counts = buf[:num_experts]
    offsets = buf[num_experts: 2 * num_experts + 1]
    sorted_pos = buf[2 * num_experts + 1: 2 * num_experts + 1 + n]
    inv_pos = buf[2 * num_experts + 1 + n: 2 * num_experts + 1 + 2 * n]
    active = buf[2 * num_experts + 1 + 2 * n: 3 * num_experts + 1 + 2 * n]
    num_active = buf[3 * num_experts + 1 + 2 * n: 3 * num_experts + 2 + 2 * n]
    error = buf[3 * num_experts + 2 + 2 * n:]  # set to 0 / 1 by the kernel
    N.check(
        N.lib.sf_moe_dispatch_ex(idx.data_ptr(), tokens, top_k, num_experts, counts.data_ptr(),
                                 offsets.data_ptr(), sorted_pos.data_ptr(), inv_pos.data_ptr(),
                                 active.data_ptr(), num_active.data_ptr(), error.data_ptr(),
                                 _ptr(active_total), _stream(dev)),
        "sf_moe_dispatch",
    )
    _launched(1)
    return Dispatch(counts, offsets, sorted_pos, inv_pos, active, num_active, error, tokens, top_k,
                    num_experts)


def moe_gather(hidden: torch.Tensor, top_k_weights: torch.Tensor, d: Dispatch,
               out_hidden: torch.Tensor | None = None, out_weights: torch.Tensor | None = None):
    dev = _require_cuda(hidden, top_k_weights)
    h = hidden.contiguous()
    w = top_k_weights.contiguous()
    rows = d.tokens * d.top_k
    xs = out_hidden if out_hidden is not None else torch.empty(rows, h.shape[1], dtype=h.dtype,
                                                                device=dev)
    ws = out_weights if out_weights is not None else torch.empty(rows, dtype=torch.float32,
                                                                  device=dev)
    N.check(
        N.lib.sf_moe_gather(h.data_ptr(), dtype_code(h.dtype), d.tokens, h.shape[1], w.data_ptr(),
                            dtype_code(w.dtype), d.top_k, d.sorted_pos.data_ptr(), xs.data_ptr(),
                            ws.data_ptr(), _stream(dev)),
        "sf_moe_gather",
    )
    _launched(1)
    return xs, ws


# ---------------------------------------------------------------------------
# K3 grouped SwiGLU


def grouped_swiglu(hidden_sorted: torch.Tensor, weights_sorted: torch.Tensor, d: Dispatch,
                   expert_slot: torch.Tensor, storage: torch.Tensor, hidden_size: int,
                   intermediate_size: int, impl: int = N.SF_SWIGLU_AUTO,
                   active: torch.Tensor | None = None, num_active: torch.Tensor | None = None,
                   act_workspace: torch.Tensor | None = None, out: torch.Tensor | None = None):
    """Weighted SwiGLU rows for every active expert, in dispatch order.

    ``storage`` is ``[slots, >= 3*H*I]`` packed expert slots; ``expert_slot``
    (int32 [E]) names the slot of each expert.  ``active``/``num_active``
    default to the dispatch's (a subset may be passed to compute one wave)."""
    dev = _require_cuda(hidden_sorted, weights_sorted, expert_slot, storage)
    if storage.dtype != hidden_sorted.dtype:
        raise ValueError("expert storage and hidden states must share a dtype")
    rows = hidden_sorted.shape[0]
    act = act_workspace if act_workspace is not None else torch.empty(
        max(rows, 1), intermediate_size, dtype=hidden_sorted.dtype, device=dev)
    y = out if out is not None else torch.empty(rows, hidden_size, dtype=hidden_sorted.dtype,
                                                device=dev)
    act_list = d.active if active is None else active
    n_act = d.num_active if num_active is None else num_active
    N.check(
        N.lib.sf_grouped_swiglu_ex(
            hidden_sorted.data_ptr(), weights_sorted.data_ptr(), dtype_code(hidden_sorted.dtype),
            d.offsets.data_ptr(), act_list.data_ptr(), n_act.data_ptr(), expert_slot.data_ptr(),
            storage.data_ptr(), storage.shape[0], storage.stride(0), d.num_experts, hidden_size,
            intermediate_size, rows, act.data_ptr(), y.data_ptr(), impl, _stream(dev)),
        "sf_grouped_swiglu",
    )
    _launched(2)
    return y


def grouped_swiglu_gathered(hidden: torch.Tensor, top_k_weights: torch.Tensor, d: Dispatch,
                            expert_slot: torch.Tensor, storage: torch.Tensor, hidden_size: int,
                            intermediate_size: int, act_workspace: torch.Tensor | None = None,
                            out: torch.Tensor | None = None):
    """``moe_gather`` then ``grouped_swiglu`` in one tcgen05 call that reads
    each expert's token rows straight from ``hidden`` (``[T, H]`` bf16) by TMA
    gather4 and the routing weights from ``top_k_weights`` (fp32 ``[T, K]``);
    bit-identical to the two calls.  Where the tcgen05 kernel does not apply
    it runs the two calls."""
    dev = _require_cuda(hidden, top_k_weights, expert_slot, storage)
    h = hidden.contiguous()
    w = top_k_weights.contiguous()
    rows = d.tokens * d.top_k
    if (h.dtype == torch.bfloat16 and w.dtype == torch.float32 and storage.dtype == torch.bfloat16
            and rows > 0):
        act = act_workspace if act_workspace is not None else torch.empty(
            rows, intermediate_size, dtype=h.dtype, device=dev)
        y = out if out is not None else torch.empty(rows, hidden_size, dtype=h.dtype, device=dev)
        rc = N.lib.sf_grouped_swiglu_gathered(
            h.data_ptr(), d.tokens, w.data_ptr(), d.top_k, d.sorted_pos.data_ptr(), d.offsets.data_ptr(),
            d.active.data_ptr(), d.num_active.data_ptr(), expert_slot.data_ptr(), storage.data_ptr(),
            storage.shape[0], storage.stride(0), d.num_experts, hidden_size, intermediate_size,
            act.data_ptr(), y.data_ptr(), _stream(dev))
        if rc == N.SF_OK:
            _launched(2)
            return y
        if rc != N.SF_ERR_UNSUPPORTED:
            N.check(rc, "sf_grouped_swiglu_gathered")
    xs, ws = moe_gather(h, w, d)
    return grouped_swiglu(xs, ws, d, expert_slot, storage, hidden_size, intermediate_size,
                          act_workspace=act_workspace, out=out)


# ---------------------------------------------------------------------------
# K4 combine


def moe_combine(out_sorted: torch.Tensor, d: Dispatch, top_k_index: torch.Tensor,
                expert_rank: torch.Tensor | None = None, reduce: int = N.SF_REDUCE_MODEL_DTYPE,
                out: torch.Tensor | None = None) -> torch.Tensor:
    dev = _require_cuda(out_sorted, top_k_index)
    res = out if out is not None else torch.empty(d.tokens, out_sorted.shape[1],
                                                  dtype=out_sorted.dtype, device=dev)
    if d.tokens == 0:
        return res
    N.check(
        N.lib.sf_moe_combine(out_sorted.data_ptr(), dtype_code(out_sorted.dtype),
                             d.inv_pos.data_ptr(), top_k_index.contiguous().data_ptr(),
                             _ptr(expert_rank), d.num_experts, d.tokens, d.top_k,
                             out_sorted.shape[1], reduce, res.data_ptr(), _stream(dev)),
        "sf_moe_combine",
    )
    _launched(1)
    return res



def moe_combine_add_rmsnorm(out_sorted: torch.Tensor, d: Dispatch, top_k_index: torch.Tensor,
                            residual: torch.Tensor, norm_weight: torch.Tensor, eps: float,
                            out: torch.Tensor, reduce: int = N.SF_REDUCE_MODEL_DTYPE) -> torch.Tensor:
    """``moe_combine`` then the residual add (``residual`` updated in place)
    and RMSNorm into ``out`` in one launch, bit-identical to the two steps."""
    dev = _require_cuda(out_sorted, top_k_index, residual, out)
    if d.tokens == 0:
        return out
    N.check(N.lib.sf_moe_combine_add_rmsnorm(out_sorted.data_ptr(), d.inv_pos.data_ptr(),
                                             top_k_index.contiguous().data_ptr(), None, d.num_experts,
                                             d.tokens, d.top_k, out_sorted.shape[1], reduce,
                                             residual.data_ptr(), residual.data_ptr(),
                                             norm_weight.data_ptr(), float(eps), out.data_ptr(),
                                             _stream(dev)), "sf_moe_combine_add_rmsnorm")
    _launched(1)
    return out

# ---------------------------------------------------------------------------
# K5 slot fill


def slot_fill_batch(dsts, srcs, stream: torch.cuda.Stream) -> None:
    """Host->device copies ``dst[i].copy_(src[i])`` on ``stream``."""
    n = len(dsts)
    if n == 0:
        return
    d_arr = (ctypes.c_void_p * n)(*[t.data_ptr() for t in dsts])
    s_arr = (ctypes.c_void_p * n)(*[t.data_ptr() for t in srcs])
    b_arr = (ctypes.c_size_t * n)(*[t.numel() * t.element_size() for t in dsts])
    for dst, src in zip(dsts, srcs):
        if dst.numel() * dst.element_size() != src.numel() * src.element_size():
            raise ValueError("slot fill source and destination sizes differ")
    N.check(N.lib.sf_slot_fill_batch(d_arr, s_arr, b_arr, n, stream.cuda_stream),
            "sf_slot_fill_batch")


# ---------------------------------------------------------------------------
# K6 tree attention


def tree_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, tree_bits: torch.Tensor | None,
                   prefix_len: int, scale: float | None = None,
                   out: torch.Tensor | None = None, impl: int = N.SF_ATTN_AUTO) -> torch.Tensor:
    """Masked GQA attention.  ``q[Hq, Tq, D]``, ``k/v[Hkv, Tk, D]`` (bf16, any
    strides with unit stride on D); keys ``< prefix_len`` are visible to every
    query, tree key j is visible to row i when bit j of ``tree_bits[i]`` is
    set.  Returns ``[Tq, Hq, D]`` bf16."""
    dev = _require_cuda(q, k, v)
    hq, tq, dim = q.shape
    hkv, tk, _ = k.shape
    if q.stride(2) != 1 or k.stride(2) != 1 or v.stride(2) != 1:
        raise ValueError("head_dim must be contiguous")
    if k.stride() != v.stride():
        raise ValueError("k and v must share strides")
    res = out if out is not None else torch.empty(tq, hq, dim, dtype=q.dtype, device=dev)
    if tree_bits is not None:
        bits = tree_bits.contiguous()
        words = bits.shape[1]
    else:
        bits, words = None, 0
    ws_bytes = N.lib.sf_tree_attention_workspace_bytes(hq, tq, tk)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    sc = float(dim ** -0.5 if scale is None else scale)
    N.check(
        N.lib.sf_tree_attention_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(bits), words, tq,
                                   tk, prefix_len, hq, hkv, dim, q.stride(0), q.stride(1),
                                   k.stride(0), k.stride(1), sc, res.data_ptr(), ws.data_ptr(),
                                   ws_bytes, impl, _stream(dev)),
        "sf_tree_attention",
    )
    _launched(2)
    return res



def tree_attention_batched(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, tree_bits: torch.Tensor | None,
                           prefix_len: int, scale: float | None = None,
                           out: torch.Tensor | None = None) -> torch.Tensor | None:
    """``tree_attention`` of B requests in one launch of the tcgen05 kernel:
    ``q[B, Hq, Tq, D]``, ``k/v[B, Hkv, Tk, D]`` (any batch and head strides,
    unit stride on D), ``tree_bits[B, Tq, words]`` or None; returns
    ``[B, Tq, Hq, D]`` bf16, or None where that kernel does not take the
    layout (the caller then runs ``tree_attention`` per request)."""
    dev = _require_cuda(q, k, v)
    b, hq, tq, dim = q.shape
    _, hkv, tk, _ = k.shape
    if q.stride(3) != 1 or k.stride(3) != 1 or v.stride(3) != 1 or k.stride() != v.stride():
        return None
    res = out if out is not None else torch.empty(b, tq, hq, dim, dtype=q.dtype, device=dev)
    if res.stride(3) != 1 or res.stride(2) != dim or res.stride(1) != hq * dim:
        return None
    if tree_bits is not None:
        bits = tree_bits if tree_bits.is_contiguous() else tree_bits.contiguous()
        words, bits_bs = bits.shape[2], bits.stride(0)
    else:
        bits, words, bits_bs = None, 0, 0
    ws_bytes = N.lib.sf_tree_attention_batched_workspace_bytes(b, hq, tq, tk)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    sc = float(dim ** -0.5 if scale is None else scale)
    rc = N.lib.sf_tree_attention_batched(q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(bits), words, b,
                                         q.stride(0), k.stride(0), bits_bs, res.stride(0), tq, tk, prefix_len,
                                         hq, hkv, dim, q.stride(1), q.stride(2), k.stride(1), k.stride(2), sc,
                                         res.data_ptr(), ws.data_ptr(), ws_bytes, _stream(dev))
    if rc == N.SF_ERR_UNSUPPORTED:
        return None
    N.check(rc, "sf_tree_attention_batched")
    _launched(2)
    return res

def tree_mask_words(ancestor_sets: torch.Tensor, start: torch.Tensor, words: int,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Visibility words over a whole KV buffer for ``tree_attention`` with
    prefix 0: row r sees column c when c < start (a device int64 scalar: the
    committed rows) or when bit c - start of ``ancestor_sets[r]`` (int64) is
    set.  Returns int32 ``[rows, words]`` (``sf_tree_mask_words``)."""
    dev = _require_cuda(ancestor_sets, start)
    rows = ancestor_sets.shape[0]
    res = out if out is not None else torch.empty(rows, words, dtype=torch.int32, device=dev)
    N.check(N.lib.sf_tree_mask_words(ancestor_sets.contiguous().data_ptr(), rows, start.data_ptr(),
                                     words, res.data_ptr(), _stream(dev)), "sf_tree_mask_words")
    _launched(1 if rows else 0)
    return res


def tree_bits_from_parents(parent_ids, device) -> torch.Tensor:
    """Ancestor bitmask of a verification tree: row i (0 = the pending seed,
    i >= 1 = node i) has bit j set when column j is i itself or an ancestor
    (``Eagle3DraftTree.verification_attention_mask``,
    ``runtime/eagle3_types.py:450-473``).  int32 words, little-endian bits."""
    q = 1 + len(parent_ids)
    words = (q + 31) // 32
    rows = [0] * q  # python ints as bitsets
    rows[0] = 1
    for node, parent in enumerate(parent_ids, start=1):
        rows[node] = rows[parent] | (1 << node)
    data = []
    for r in rows:
        for w in range(words):
            word = (r >> (32 * w)) & 0xFFFFFFFF
            data.append(word - (1 << 32) if word >= (1 << 31) else word)
    return torch.tensor(data, dtype=torch.int32).view(q, words).to(device)


def tree_bits_from_mask(mask: torch.Tensor, prefix_len: int) -> torch.Tensor:
    """Pack a boolean ``[Tq, Tk]`` mask's tree block (columns >= prefix_len)
    into int32 words on the mask's device."""
    tree = mask[:, prefix_len:].to(torch.int64)
    tq, cols = tree.shape
    words = max(1, (cols + 31) // 32)
    pad = words * 32 - cols
    if pad:
        tree = torch.nn.functional.pad(tree, (0, pad))
    tree = tree.view(tq, words, 32)
    shifts = torch.arange(32, device=mask.device, dtype=torch.int64)
    packed = (tree << shifts).sum(-1)
    packed = torch.where(packed >= (1 << 31), packed - (1 << 32), packed)
    return packed.to(torch.int32)


# ---------------------------------------------------------------------------
# K7 expert parallelism (dispatch / return rows of the all-to-all exchange)


def ep_row_bytes(dtype: torch.dtype, hidden_size: int, top_k: int) -> int:
    """Bytes of one exchanged row: hidden, K local expert ids, K weights."""
    n = N.lib.sf_ep_row_bytes(dtype_code(dtype), hidden_size, top_k)
    if n < 0:
        raise ValueError("unsupported expert-parallel row shape")
    return int(n)


@dataclass
class EpSend:
    rows: torch.Tensor  # uint8 [tokens*world, row_bytes] (the first sum(pairs) rows are used)
    counts: torch.Tensor  # int64 [world, 2]: (pairs, routes) per destination rank
    route_row: torch.Tensor  # int32 [tokens*top_k]: row of each route's output on return
    error: torch.Tensor  # int32 [1]
    tokens: int
    top_k: int
    num_experts: int
    world: int


def ep_send_pack(hidden: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor,
                 num_experts: int, world: int) -> EpSend:
    """Rows to send to each rank (grouped by rank, then token) and the plan."""
    dev = _require_cuda(hidden, top_k_index, top_k_weights)
    if top_k_index.dtype != torch.int64 or top_k_index.ndim != 2:
        raise ValueError("top_k_index must be int64 [tokens, top_k]")
    h = hidden.contiguous()
    idx = top_k_index.contiguous()
    w = top_k_weights.contiguous()
    tokens, top_k = idx.shape
    rb = ep_row_bytes(h.dtype, h.shape[1], top_k)
    rows = torch.empty(max(tokens * world, 1), rb, dtype=torch.uint8, device=dev)
    i32 = torch.empty(tokens * top_k + tokens * world + 1, dtype=torch.int32, device=dev)
    route_row = i32[: tokens * top_k]
    pair_token = i32[tokens * top_k: tokens * top_k + tokens * world]
    error = i32[tokens * top_k + tokens * world:]
    error.zero_()
    counts = torch.empty(world, 2, dtype=torch.int64, device=dev)
    N.check(N.lib.sf_ep_send_pack(h.data_ptr(), dtype_code(h.dtype), tokens, h.shape[1],
                                  idx.data_ptr(), w.data_ptr(), dtype_code(w.dtype), top_k,
                                  num_experts, world, rows.data_ptr(), rb, counts.data_ptr(),
                                  route_row.data_ptr(), pair_token.data_ptr(), error.data_ptr(),
                                  _stream(dev)), "sf_ep_send_pack")
    _launched(1 if tokens == 0 else 2)
    return EpSend(rows, counts, route_row, error, tokens, top_k, num_experts, world)


def ep_recv_group(recv_rows: torch.Tensor, pairs: int, hidden_size: int, top_k: int,
                  local_experts: int, dtype: torch.dtype):
    """Groups the received route slots by local expert.  Returns the
    ``Dispatch`` over the local experts (``tokens`` = pairs) and
    ``return_src`` (int32 [pairs*top_k]; its first ``routes`` entries name
    the sorted row of each valid slot in (pair, slot) order)."""
    dev = _require_cuda(recv_rows)
    rb = ep_row_bytes(dtype, hidden_size, top_k)
    if recv_rows.dtype != torch.uint8 or recv_rows.shape[0] < pairs or recv_rows.shape[-1] != rb:
        raise ValueError("recv_rows must be uint8 [>= pairs, row_bytes]")
    n = pairs * top_k
    E = local_experts
    i32 = dict(dtype=torch.int32, device=dev)
    buf = torch.empty(E + (E + 1) + 3 * n + E + 2, **i32)
    counts = buf[:E]
    offsets = buf[E: 2 * E + 1]
    sorted_pos = buf[2 * E + 1: 2 * E + 1 + n]
    inv_pos = buf[2 * E + 1 + n: 2 * E + 1 + 2 * n]
    return_src = buf[2 * E + 1 + 2 * n: 2 * E + 1 + 3 * n]
    active = buf[2 * E + 1 + 3 * n: 3 * E + 1 + 3 * n]
    num_active = buf[3 * E + 1 + 3 * n: 3 * E + 2 + 3 * n]
    error = buf[3 * E + 2 + 3 * n:]
    error.zero_()
    N.check(N.lib.sf_ep_recv_group(recv_rows.data_ptr(), rb, dtype_code(dtype), pairs, hidden_size,
                                   top_k, E, counts.data_ptr(), offsets.data_ptr(),
                                   sorted_pos.data_ptr(), inv_pos.data_ptr(), active.data_ptr(),
                                   num_active.data_ptr(), return_src.data_ptr(), error.data_ptr(),
                                   _stream(dev)), "sf_ep_recv_group")
    _launched(1)
    d = Dispatch(counts, offsets, sorted_pos, inv_pos, active, num_active, error, pairs, top_k, E)
    return d, return_src


def ep_recv_gather(recv_rows: torch.Tensor, d: Dispatch, hidden_size: int, dtype: torch.dtype,
                   routes: int):
    """Sorted hidden rows ``[routes, H]`` and their routing weights (fp32)."""
    dev = _require_cuda(recv_rows)
    rb = ep_row_bytes(dtype, hidden_size, d.top_k)
    xs = torch.empty(max(routes, 1), hidden_size, dtype=dtype, device=dev)[:routes]
    ws = torch.empty(max(routes, 1), dtype=torch.float32, device=dev)[:routes]
    N.check(N.lib.sf_ep_recv_gather(recv_rows.data_ptr(), rb, dtype_code(dtype), hidden_size,
                                    d.top_k, d.sorted_pos.data_ptr(), routes, xs.data_ptr(),
                                    ws.data_ptr(), _stream(dev)), "sf_ep_recv_gather")
    _launched(1 if routes else 0)
    return xs, ws


def ep_return_pack(out_sorted: torch.Tensor, return_src: torch.Tensor, routes: int) -> torch.Tensor:
    """One output row per received route, in (pair, slot) order."""
    dev = _require_cuda(out_sorted, return_src)
    H = out_sorted.shape[1]
    rows = torch.empty(max(routes, 1), H, dtype=out_sorted.dtype, device=dev)[:routes]
    N.check(N.lib.sf_ep_return_pack(out_sorted.data_ptr(), dtype_code(out_sorted.dtype), H,
                                    return_src.data_ptr(), routes, rows.data_ptr(), _stream(dev)),
            "sf_ep_return_pack")
    _launched(1 if routes else 0)
    return rows


def ep_combine(returned: torch.Tensor, send: EpSend, top_k_index: torch.Tensor,
               reduce: int = N.SF_REDUCE_MODEL_DTYPE, out: torch.Tensor | None = None) -> torch.Tensor:
    """The single-GPU combine over the returned rows (ascending expert id)."""
    dev = _require_cuda(top_k_index)
    H = returned.shape[1]
    res = out if out is not None else torch.empty(send.tokens, H, dtype=returned.dtype, device=dev)
    if send.tokens == 0:
        return res
    _require_cuda(returned)
    N.check(N.lib.sf_moe_combine(returned.data_ptr(), dtype_code(returned.dtype),
                                 send.route_row.data_ptr(), top_k_index.contiguous().data_ptr(),
                                 None, send.num_experts, send.tokens, send.top_k, H, reduce,
                                 res.data_ptr(), _stream(dev)), "sf_moe_combine")
    _launched(1)
    return res


def logsoftmax_topk(logits: torch.Tensor, k: int, scale: float = 1.0,
                    out: tuple[torch.Tensor, torch.Tensor] | None = None):
    """``torch.topk(torch.log_softmax(logits.float() * scale, -1), k)`` over the
    last dim of bf16 logits in one launch: (values fp32, indices int64), each
    ``[..., k]``.  Among equal values the lower index comes first."""
    dev = _require_cuda(logits)
    if logits.dtype != torch.bfloat16:
        raise TypeError("logsoftmax_topk takes bf16 logits")
    x = logits.contiguous()
    V = x.shape[-1]
    rows = x.numel() // V if V else 0
    shape = tuple(x.shape[:-1]) + (k,)
    if out is None:
        vals = torch.empty(shape, dtype=torch.float32, device=dev)
        idx = torch.empty(shape, dtype=torch.int64, device=dev)
    else:
        vals, idx = out
    N.check(N.lib.sf_logsoftmax_topk(x.data_ptr(), rows, V, float(scale), int(k), vals.data_ptr(),
                                     idx.data_ptr(), _stream(dev)), "sf_logsoftmax_topk")
    _launched(1 if rows else 0)
    return vals, idx



LINEAR_MAX_OUT = 4096  # measured on B200: wider weights stream as fast through cuBLAS
LINEAR_MIN_IN = 4096
_SMS: dict = {}


def _wide_output(n_out: int, device: torch.device) -> bool:
    """At least one 128-row weight tile per SM: ``sf_linear_bf16`` then runs
    its persistent streaming kernel (the 151,936-row lm_head), measured on a
    B200 a little faster than the library GEMM at 7 and 65 rows."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return n_out >= 128 * _SMS[idx]


def linear_argmax(x: torch.Tensor, weight: torch.Tensor, logits: bool = True):
    """The lm_head and the greedy pick in one pass over the weight:
    ``(F.linear(x, weight) or None, argmax)`` for bf16 ``x [rows, K]`` (rows
    <= 128), ``weight [V, K]``.  The argmax is over the bf16-rounded logits,
    the lowest index among equal maxima (``torch.argmax`` on the logits this
    call returns); int64 ``[rows]``."""
    dev = _require_cuda(x, weight)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("linear_argmax takes bf16 inputs")
    xx = x.reshape(-1, x.shape[-1]).contiguous()
    w = weight.contiguous()
    rows, k = xx.shape
    v = w.shape[0]
    y = torch.empty(rows, v, dtype=x.dtype, device=dev) if logits else None
    am = torch.empty(rows, dtype=torch.int64, device=dev)
    nbytes = N.lib.sf_linear_argmax_workspace_bytes(rows, k, v)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    N.check(N.lib.sf_linear_bf16_argmax(xx.data_ptr(), rows, k, w.data_ptr(), v, _ptr(y), am.data_ptr(),
                                        ws.data_ptr(), nbytes, _stream(dev)), "sf_linear_bf16_argmax")
    _launched(2 if rows else 0)
    if y is not None:
        y = y.reshape(*x.shape[:-1], v)
    return y, am.reshape(x.shape[:-1])


def linear(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear(x, weight)`` (no bias) for bf16 ``x [..., K]`` on the
    tcgen05 kernel (``sf_linear_bf16``) where it measured faster than the
    library GEMM on a B200: few rows (<= 32) against a tall, narrow weight
    whose K split is what fills the GPU (out_features <= LINEAR_MAX_OUT,
    in_features >= LINEAR_MIN_IN: the o projection and the drafter's
    2048-wide outputs), and up to 128 rows against a wide weight (at least
    one 128-row tile per SM: the lm_head).  Other shapes (the q|k|v
    projection among them) take the library GEMM."""
    k = x.shape[-1]
    rows = x.numel() // k if k else 0
    n_out = weight.shape[0]
    if (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and rows > 0
            and x.is_contiguous() and weight.is_contiguous()
            and ((rows <= 32 and n_out <= LINEAR_MAX_OUT and k >= LINEAR_MIN_IN)
                 or (rows <= 128 and _wide_output(n_out, x.device)))):
        res = out if out is not None else torch.empty(*x.shape[:-1], n_out, dtype=x.dtype, device=x.device)
        rc = N.lib.sf_linear_bf16(x.data_ptr(), rows, k, weight.data_ptr(), n_out, res.data_ptr(),
                                  _stream(x.device))
        if rc == N.SF_OK:
            _launched(1)
            return res
        if rc != N.SF_ERR_UNSUPPORTED:
            N.check(rc, "sf_linear_bf16")
    y = torch.nn.functional.linear(x, weight)
    if out is not None:
        out.copy_(y)
        return out
    return y
