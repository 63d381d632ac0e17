"""ctypes binding of the C ABI in ``include/specfit_b200.h``.

The library is loaded from the package directory (built in-tree by
``python -m specfit_b200.build``).  There is no fallback: if the library is
missing or a symbol is absent, importing an op raises immediately.
"""
from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libspecfit_b200.so"
HEADER = PKG.parent / "include" / "specfit_b200.h"

SF_OK = 0
SF_ERR_INVALID_ARGUMENT = 1
SF_ERR_CUDA = 2
SF_ERR_UNSUPPORTED = 3
SF_ERR_WORKSPACE = 4
SF_ERR_STATE = 5
SF_ERR_NO_SLOT = 6

SF_CACHE_ACQUIRE = 0
SF_CACHE_NONBLOCKING = 1
SF_CACHE_RESIDENT_ONLY = 2
SF_CACHE_PROBABILITY = 3
SF_GRANT_NONE = 0
SF_GRANT_HIT = 1
SF_GRANT_JOIN = 2
SF_GRANT_MISS = 3
SF_CACHE_RESET_COLD = 0
SF_CACHE_RESET_DISCARD = 1
SF_SLOT_EXPERT = 0
SF_SLOT_GENERATION = 1
SF_SLOT_STAMP = 2
SF_SLOT_READY = 3
SF_SLOT_GUARDS = 4

SF_DTYPE_F32 = 0
SF_DTYPE_BF16 = 1

SF_REDUCE_MODEL_DTYPE = 0
SF_REDUCE_F32 = 1

SF_SWIGLU_AUTO = 0
SF_SWIGLU_SIMT = 1
SF_SWIGLU_TCGEN05 = 2

SF_ATTN_AUTO = 0
SF_ATTN_SIMT = 1
SF_ATTN_MMA = 2
SF_ATTN_TCGEN05 = 3

_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

class EpPeer(ctypes.Structure):
    """``sf_ep_peer`` (include/specfit_b200.h)."""

    _fields_ = [("world", _i32), ("rank", _i32), ("top_k", _i32), ("hidden_size", _i32),
                ("dtype", _i32), ("local_experts", _i32), ("grid", _i32), ("wait_limit_ms", _i32),
                ("cap_pairs", _i64), ("cap_routes", _i64), ("row_bytes", _i64),
                ("out_row_bytes", _i64), ("peers", _vp), ("local", _vp), ("epochs", _vp),
                ("status", _vp), ("off_recv_rows", _i64), ("off_ret_rows", _i64),
                ("off_recv_counts", _i64), ("off_recv_arrive", _i64), ("off_ret_arrive", _i64)]


_peer_p = ctypes.POINTER(EpPeer)
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64


class SfCacheGrant(ctypes.Structure):
    _fields_ = [("kind", _i32), ("slot", _i32), ("generation", _u32), ("victim", _i32),
                ("submission", _i64), ("ready_event", _u64)]


class SfCacheCounters(ctypes.Structure):
    _fields_ = [(name, _i64) for name in (
        "h2d_submissions", "resident_hits", "inflight_joins", "evictions", "pending_use_guards",
        "sequence", "submission_sequence", "state_version", "outstanding_fills")]


class SfCacheSlot(ctypes.Structure):
    _fields_ = [("expert", _i32), ("generation", _u32), ("leases", _i32), ("guards", _i32),
                ("stamp", _i64), ("ready_event", _u64), ("guards_pending", _i32), ("pad", _i32)]


class SfCacheFill(ctypes.Structure):
    _fields_ = [("expert", _i32), ("slot", _i32), ("generation", _u32), ("done", _i32),
                ("submission", _i64), ("ready_event", _u64)]

# name -> (restype, argtypes)
SIGNATURES = {
    "sf_last_error": (ctypes.c_char_p, []),
    "sf_abi_version": (_i32, []),
    "sf_device_status": (_i32, [ctypes.POINTER(_i32), _i32]),
    "sf_router_topk_workspace_bytes": (_sz, [_i64, _i32]),
    "sf_router_topk": (_i32, [_vp, _vp, _i32, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp,
                              _vp, _sz, _vp]),
    "sf_router_topk_noalloc_max_elems": (_i64, []),
    "sf_router_topk_noalloc": (_i32, [_vp, _vp, _i32, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _vp,
                                      _vp, _vp]),
    "sf_moe_dispatch": (_i32, [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "sf_moe_dispatch_ex": (_i32, [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "sf_moe_gather": (_i32, [_vp, _i32, _i64, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp]),
    "sf_grouped_swiglu": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32,
                                 _i32, _i64, _vp, _vp, _vp]),
    "sf_grouped_swiglu_ex": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32,
                                    _i32, _i32, _i64, _vp, _vp, _i32, _vp]),
    "sf_grouped_swiglu_gathered": (_i32, [_vp, _i64, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                          _i32, _i32, _i32, _vp, _vp, _vp]),
    "sf_moe_combine": (_i32, [_vp, _i32, _vp, _vp, _vp, _i32, _i64, _i32, _i32, _i32, _vp, _vp]),
    "sf_cache_create": (_i32, [_i32, _i32, _vp, _sz, _vp, _vp, ctypes.POINTER(_vp)]),
    "sf_cache_destroy": (None, [_vp]),
    "sf_cache_set_copy_stream": (_i32, [_vp, _vp]),
    "sf_cache_acquire": (_i32, [_vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp, ctypes.POINTER(_i32)]),
    "sf_cache_touch": (_i32, [_vp, _i32, _i32, _u32]),
    "sf_cache_check": (_i32, [_vp, _i32, _i32, _u32]),
    "sf_cache_wait": (_i32, [_vp, _i32, _i32, _u32, _vp, _i32]),
    "sf_cache_release": (_i32, [_vp, _i32, _i32, _u32, _vp, _i32]),
    "sf_cache_state": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp]),
    "sf_cache_fills": (_i32, [_vp, _vp, _i32, ctypes.POINTER(_i32)]),
    "sf_cache_quiescent": (_i32, [_vp, ctypes.POINTER(_i32)]),
    "sf_cache_resident_table": (_i32, [_vp, _vp, ctypes.POINTER(_i32)]),
    "sf_cache_add_hits": (_i32, [_vp, _i64]),
    "sf_cache_reset": (_i32, [_vp, _i32]),
    "sf_cache_slot_edit": (_i32, [_vp, _i32, _i32, _i64]),
    "sf_cache_forget": (_i32, [_vp, _i32]),
    "sf_cache_set_version": (_i32, [_vp, _i64]),
    "sf_cache_export": (_i32, [_vp, _vp, _sz, ctypes.POINTER(_sz)]),
    "sf_cache_import": (_i32, [_vp, _vp, _sz]),
    "sf_cache_export_slots": (_i32, [_vp, _vp, _vp, _vp, _vp, ctypes.POINTER(_i64), _vp]),
    "sf_cache_adopt_slots": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp]),
    "sf_dir_plan": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp,
                           _vp, _vp, _vp, _vp, _vp]),
    "sf_dir_plan_ex": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp,
                              _vp, _vp, _vp, _vp, _u64, _vp]),
    "sf_dir_fill": (_i32, [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp]),
    "sf_capture_body_stream": (_i32, [ctypes.POINTER(_vp)]),
    "sf_capture_cond_handle": (_i32, [_vp, ctypes.POINTER(_u64)]),
    "sf_capture_if_begin": (_i32, [_vp, _vp, _u64]),
    "sf_capture_if_end": (_i32, [_vp, _vp]),
    "sf_host_device_address": (_i32, [_vp, ctypes.POINTER(_u64)]),
    "sf_slot_fill_batch": (_i32, [ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_sz),
                                  _i32, _vp]),
    "sf_specfit_select": (_i32, [_i32, _vp, _vp, _vp, _i32, _vp, _vp, _i32, ctypes.c_double,
                                 ctypes.c_double, _vp, _vp, _vp]),
    "sf_compensated_sum": (ctypes.c_double, [_vp, _i32]),
    "sf_specfit_pack_routes": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp, _i32]),
    "sf_tree_attention_workspace_bytes": (_sz, [_i32, _i64, _i64]),
    "sf_tree_attention": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _i32, _i32, _i32,
                                 _i64, _i64, _i64, _i64, _f32, _vp, _vp, _sz, _vp]),
    "sf_tree_attention_ex": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _i32, _i32, _i32,
                                    _i64, _i64, _i64, _i64, _f32, _vp, _vp, _sz, _i32, _vp]),
    "sf_tree_attention_batched_workspace_bytes": (_sz, [_i32, _i32, _i64, _i64]),
    "sf_tree_attention_batched": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i64, _i64, _i64, _i64, _i64, _i64,
                                         _i64, _i32, _i32, _i32, _i64, _i64, _i64, _i64, _f32, _vp, _vp,
                                         _sz, _vp]),
    "sf_ep_row_bytes": (_i64, [_i32, _i32, _i32]),
    "sf_ep_send_pack": (_i32, [_vp, _i32, _i64, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _i64,
                               _vp, _vp, _vp, _vp, _vp]),
    "sf_ep_recv_group": (_i32, [_vp, _i64, _i32, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp,
                                _vp, _vp, _vp, _vp]),
    "sf_ep_recv_gather": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _i64, _vp, _vp, _vp]),
    "sf_ep_return_pack": (_i32, [_vp, _i32, _i32, _vp, _i64, _vp, _vp]),
    "sf_ep_peer_layout": (_i64, [_peer_p]),
    "sf_ipc_alloc": (_i32, [_sz, ctypes.POINTER(_vp), _vp]),
    "sf_ipc_free": (_i32, [_vp]),
    "sf_ipc_open": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "sf_ipc_close": (_i32, [_vp]),
    "sf_ep_peer_send": (_i32, [_peer_p, _vp, _i64, _vp, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp,
                               _vp]),
    "sf_ep_peer_recv": (_i32, [_peer_p, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "sf_ep_peer_return": (_i32, [_peer_p, _vp, _vp, _vp, _vp]),
    "sf_ep_peer_return_plan": (_i32, [_peer_p, _vp, _vp, _vp, _vp]),
    "sf_grouped_swiglu_peer": (_i32, [_peer_p, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _vp, _vp,
                                      _vp, _vp]),
    "sf_ep_peer_finish": (_i32, [_peer_p, _vp, _vp, _i64, _i32, _i32, _vp, _vp]),
    "sf_tree_mask_words": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp]),
    "sf_kv_compact": (_i32, [_vp, _i32, _i32, _i32, _i64, _i64, _vp, _i32, _vp, _vp]),
    "sf_logsoftmax_topk": (_i32, [_vp, _i64, _i64, _f32, _i32, _vp, _vp, _vp]),
    "sf_linear_bf16": (_i32, [_vp, _i64, _i64, _vp, _i64, _vp, _vp]),
    "sf_linear_argmax_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "sf_linear_bf16_argmax": (_i32, [_vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _sz, _vp]),
    "sf_draft_level": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp, _vp, _i32, _i32, _i64, _i32, _i32, _vp,
                              _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "sf_rope_rows": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp, _vp]),
    "sf_moe_combine_add_rmsnorm": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _i32, _i32, _i32, _vp, _vp, _vp,
                                          _f32, _vp, _vp]),
    "sf_add_rmsnorm": (_i32, [_vp, _vp, _vp, _vp, _f32, _i64, _i32, _vp, _vp]),
    "sf_qk_norm_rope": (_i32, [_vp, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _f32, _vp, _vp,
                               _vp, _i64, _i64, _i64, _vp, _vp]),
}


class NativeError(RuntimeError):
    """A CUDA or unsupported-configuration failure reported by the library."""


def declared_symbols() -> list:
    """Every entry point declared in include/specfit_b200.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^SF_API [^(]*?\b(sf_\w+)\(", text, flags=re.M)))


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m specfit_b200.build` "
            "(there is no CPU fallback for the specfit_b200 path)"
        )
    lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_LAZY | os.RTLD_GLOBAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError -> loud failure
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    msg = lib.sf_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    if status == SF_OK:
        return
    msg = last_error()
    if status == SF_ERR_INVALID_ARGUMENT:
        raise ValueError(f"{what}: {msg}")
    if status == SF_ERR_STATE:
        raise RuntimeError(msg)
    raise NativeError(f"{what} failed (status {status}): {msg}")


def device_status(reset: bool = False) -> int:
    out = _i32(0)
    check(lib.sf_device_status(ctypes.byref(out), int(reset)), "sf_device_status")
    return out.value
