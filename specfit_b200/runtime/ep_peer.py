"""Peer-memory regions of an expert-parallel group (the sync-free exchange).

Each rank allocates one region (``sf_ipc_alloc``), the ranks trade CUDA IPC
handles through the process group, and every rank maps the others' regions
into its own device context (``sf_ipc_open``: peer access over NVLink).  The
``sf_ep_peer`` descriptor then lets the K7 peer kernels push rows into, and
read arrivals from, any rank's region with no host involvement.

With one rank the region is only this process's own, and the same kernels
run the exchange with itself (each wait is satisfied by the push launched
before it on the same stream).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from .. import _native as N
from .. import ops


class PeerExchange:
    def __init__(self, *, rank: int, world: int, max_tokens: int, hidden_size: int, top_k: int,
                 local_experts: int, device, dtype=torch.bfloat16, group=None, grid: int | None = None,
                 wait_limit_ms: int = 2000, fused_return: bool = True) -> None:
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device(device)
        self.dtype = dtype
        # The return all-to-all stored by the expert GEMM's epilogue (bf16,
        # tcgen05 shapes); otherwise a separate push kernel after it.  Every
        # rank of an exchange must make the same choice.
        self.fused_return = fused_return
        self._ticket = torch.zeros(1, dtype=torch.int32, device=self.device)
        d = N.EpPeer()
        d.world, d.rank, d.top_k, d.hidden_size = world, rank, top_k, hidden_size
        d.dtype = ops.dtype_code(dtype)
        d.local_experts = local_experts
        if grid is None:  # the push and gather kernels: one CTA per SM (equal on every rank of a box)
            grid = torch.cuda.get_device_properties(self.device).multi_processor_count
        d.grid, d.wait_limit_ms = grid, wait_limit_ms
        d.cap_pairs = max_tokens
        d.cap_routes = max_tokens * top_k
        d.row_bytes = ops.ep_row_bytes(dtype, hidden_size, top_k)
        d.out_row_bytes = hidden_size * torch.empty((), dtype=dtype).element_size()
        self.bytes = int(N.lib.sf_ep_peer_layout(ctypes.byref(d)))
        self.desc = d
        # When a list, every layer appends its phase events (send, receive,
        # grouped SwiGLU, return, finish boundaries) for a timing pass.
        self.phase_events = None
        self._opened: list = []
        self._base = None
        with torch.cuda.device(self.device):
            base = ctypes.c_void_p()
            handle = (ctypes.c_char * 64)()
            N.check(N.lib.sf_ipc_alloc(self.bytes, ctypes.byref(base), handle), "sf_ipc_alloc")
            self._base = base.value
            bases = [0] * world
            bases[rank] = base.value
            if world > 1:
                handles = [None] * world
                dist.all_gather_object(handles, bytes(handle), group=group)
                for r, h in enumerate(handles):
                    if r == rank:
                        continue
                    p = ctypes.c_void_p()
                    hb = ctypes.create_string_buffer(h, 64)
                    N.check(N.lib.sf_ipc_open(hb, ctypes.byref(p)), "sf_ipc_open")
                    self._opened.append(p.value)
                    bases[r] = p.value
            self.peers = torch.tensor(bases, dtype=torch.int64, device=self.device)
            self.state = torch.zeros(4, dtype=torch.int64, device=self.device)  # epochs[2], status
            d.peers = self.peers.data_ptr()
            d.local = base.value
            d.epochs = self.state.data_ptr()
            d.status = self.state[2:].data_ptr()
            torch.cuda.synchronize(self.device)
        if world > 1:
            dist.barrier(group=group)  # every region zeroed and mapped before any push

    @property
    def cap_pairs(self) -> int:
        return self.desc.cap_pairs

    def status(self) -> tuple:
        """(site, missing ranks bitmask) of the first wait that gave up, or (0, 0)."""
        st = self.state[2:].view(torch.int32).cpu()
        return int(st[0]), int(st[1])

    def check(self) -> None:
        site, missing = self.status()
        if site:
            where = {1: "receive", 2: "return"}.get(site, str(site))
            ranks = [r for r in range(self.world) if missing >> r & 1]
            raise RuntimeError(f"expert-parallel peer exchange: {where} wait gave up; "
                               f"ranks {ranks} did not arrive")

    PHASES = ("send_pack_push", "receive_wait_group_gather", "grouped_swiglu", "return_push",
              "return_wait_combine")

    def phase_times_us(self) -> dict:
        """Median microseconds of each phase over the layers recorded in
        ``phase_events`` (synchronises the device)."""
        import statistics

        torch.cuda.synchronize(self.device)
        rows = [[a.elapsed_time(b) * 1e3 for a, b in zip(m, m[1:])] for m in self.phase_events or []]
        if not rows:
            return {}
        return {name: round(statistics.median(r[i] for r in rows), 2) for i, name in enumerate(self.PHASES)}

    def close(self) -> None:
        if self._base is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                N.lib.sf_ipc_close(p)
            self._opened = []
            if self.world > 1:
                dist.barrier(group=self.group)  # nobody maps this region any more
            N.lib.sf_ipc_free(self._base)
        self._base = None

    # -- one layer -----------------------------------------------------------------

    def layer(self, moe, hidden: torch.Tensor, top_k_index: torch.Tensor,
              top_k_weights: torch.Tensor) -> torch.Tensor:
        """The MoE experts of one layer through the peer exchange (``moe``:
        an ``ExpertParallelMoE`` of this rank).  No host synchronisation."""
        d = self.desc
        dev = hidden.device
        T, K = top_k_index.shape
        if T > d.cap_pairs:
            raise ValueError(f"{T} tokens exceed the peer exchange capacity {d.cap_pairs}")
        stream = torch.cuda.current_stream(dev).cuda_stream
        marks = [] if self.phase_events is not None else None

        def mark():
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append(ev)

        mark()
        h = hidden.contiguous()
        idx = top_k_index.contiguous()
        w = top_k_weights.contiguous()
        E = moe.num_experts
        El = moe.local_experts
        staging = torch.empty(max(T * self.world, 1), d.row_bytes, dtype=torch.uint8, device=dev)
        send_i32 = torch.empty(T * K + T * self.world + 1, dtype=torch.int32, device=dev)
        route_row = send_i32[: T * K]
        pair_token = send_i32[T * K: T * K + T * self.world]
        send_err = send_i32[T * K + T * self.world:]
        send_err.zero_()
        send_counts = torch.empty(self.world, 2, dtype=torch.int64, device=dev)
        N.check(N.lib.sf_ep_peer_send(ctypes.byref(d), h.data_ptr(), T, idx.data_ptr(), w.data_ptr(),
                                      ops.dtype_code(w.dtype), E, staging.data_ptr(),
                                      send_counts.data_ptr(), route_row.data_ptr(),
                                      pair_token.data_ptr(), send_err.data_ptr(), stream),
                "sf_ep_peer_send")
        mark()
        n = self.world * d.cap_pairs * K
        rows = self.world * d.cap_routes
        buf = torch.empty(El + (El + 1) + 3 * n + El + 2, dtype=torch.int32, device=dev)
        counts = buf[:El]
        offsets = buf[El: 2 * El + 1]
        sorted_pos = buf[2 * El + 1: 2 * El + 1 + n]
        inv_pos = buf[2 * El + 1 + n: 2 * El + 1 + 2 * n]
        return_src = buf[2 * El + 1 + 2 * n: 2 * El + 1 + 3 * n]
        active = buf[2 * El + 1 + 3 * n: 3 * El + 1 + 3 * n]
        num_active = buf[3 * El + 1 + 3 * n: 3 * El + 2 + 3 * n]
        err = buf[3 * El + 2 + 3 * n:]
        err.zero_()
        xs = torch.empty(rows, d.hidden_size, dtype=self.dtype, device=dev)
        ws = torch.empty(rows, dtype=torch.float32, device=dev)
        N.check(N.lib.sf_ep_peer_recv(ctypes.byref(d), counts.data_ptr(), offsets.data_ptr(),
                                      sorted_pos.data_ptr(), inv_pos.data_ptr(), active.data_ptr(),
                                      num_active.data_ptr(), return_src.data_ptr(), err.data_ptr(),
                                      xs.data_ptr(), ws.data_ptr(), stream), "sf_ep_peer_recv")
        mark()
        if (self.fused_return and self.dtype == torch.bfloat16 and moe.storage.dtype == torch.bfloat16
                and moe.hidden % 128 == 0 and moe.inter % 64 == 0):
            # The return rides on the expert GEMM: phase 2 stores each output
            # row straight into its source's region and the last CTA signals.
            dst_row = torch.empty(rows, dtype=torch.int64, device=dev)
            N.check(N.lib.sf_ep_peer_return_plan(ctypes.byref(d), return_src.data_ptr(), offsets.data_ptr(),
                                                 dst_row.data_ptr(), stream), "sf_ep_peer_return_plan")
            act = torch.empty(max(rows, 1), moe.inter, dtype=self.dtype, device=dev)
            N.check(N.lib.sf_grouped_swiglu_peer(ctypes.byref(d), xs.data_ptr(), ws.data_ptr(), offsets.data_ptr(),
                                                 active.data_ptr(), num_active.data_ptr(), moe.slot.data_ptr(),
                                                 moe.storage.data_ptr(), moe.storage.shape[0],
                                                 moe.storage.stride(0), moe.inter, act.data_ptr(),
                                                 dst_row.data_ptr(), self._ticket.data_ptr(), stream),
                    "sf_grouped_swiglu_peer")
            ops._launched(3)  # the plan and the two SwiGLU phases
            mark()
            mark()  # (the return has no phase of its own)
        else:
            disp = ops.Dispatch(counts, offsets, sorted_pos, inv_pos, active, num_active, err,
                                self.world * d.cap_pairs, K, El)
            ys = ops.grouped_swiglu(xs, ws, disp, moe.slot, moe.storage, moe.hidden, moe.inter)
            mark()
            N.check(N.lib.sf_ep_peer_return(ctypes.byref(d), ys.data_ptr(), return_src.data_ptr(),
                                            offsets.data_ptr(), stream), "sf_ep_peer_return")
            ops._launched(1)
            mark()
        out = torch.empty(T, d.hidden_size, dtype=self.dtype, device=dev)
        N.check(N.lib.sf_ep_peer_finish(ctypes.byref(d), idx.data_ptr(), route_row.data_ptr(), T, E,
                                        N.SF_REDUCE_MODEL_DTYPE, out.data_ptr(), stream),
                "sf_ep_peer_finish")
        mark()
        if marks is not None:
            self.phase_events.append(marks)
        ops._launched(6 if T else 5)  # send (plan, push), receive (wait, group, gather), finish
        return out
