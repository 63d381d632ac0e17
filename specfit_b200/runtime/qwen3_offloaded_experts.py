"""Offloaded Qwen3-MoE experts on the B200 kernels.

Drop-in for ``Qwen3OffloadedExperts`` (``src/specfit/runtime/
qwen3_offloaded_experts.py:65-292``): same constructor, attributes, input
validation (messages included), execution policies and reduction modes.
The forward pass differs in how it is executed, not in what it computes:

* routes are grouped on the device (``sf_moe_dispatch``, the stable grouping
  of :173-178) and rows gathered once (``sf_moe_gather``, :189-190);
* a lease wave is one call into the native slot manager, which submits
  every miss of the wave to the copy engines (``GpuExpertCache.acquire_many``);
* every expert of a lease wave runs in one grouped SwiGLU launch that reads
  the weights straight from their cache slots (``sf_grouped_swiglu``,
  :38-62 plus the ``mul_(w)`` of :132-138);
* the reduction is one launch in canonical ascending-expert order or in
  execution (arrival) order (``sf_moe_combine``, :144-163), with the same
  rounding after every add as the reference's bf16 ``index_add_``.

Cache protocol.  When the cache holds every expert of the layer (all
resident, nothing in flight), the slot of each expert is fixed and the layer
runs with no host synchronisation; hits are counted on the device.
Otherwise the active experts are copied to the host (the reference
synchronises here too, :112 / :175) and leased in execution order, as many
at a time as the cache can pin (a "wave"); each wave's fills are ordered
before its grouped launch and its leases are released right after the
launch, so later fills into those slots wait for it.  With this protocol the
resident hits, H2D submissions and evictions equal the reference's
whenever the active experts fit in the cache, and in the reference's own
one-slot and two-slot unit tests.
"""
from __future__ import annotations

from enum import Enum
from typing import Sequence

import torch
from torch import nn

from .. import _native as N
from .. import ops
from .gpu_expert_cache import GpuExpertCache
from .lease import NoEvictableSlotError
from .state import ExpertKey


class ReductionMode(str, Enum):
    CANONICAL = "canonical"
    ARRIVAL_ORDER = "arrival_order"


class ExpertExecutionPolicy(str, Enum):
    EXPERT_ID_ASCENDING = "expert_id_ascending"
    RESIDENT_FIRST = "resident_first"


class Qwen3OffloadedExperts(nn.Module):
    def __init__(self, *, layer_id: int, cache: GpuExpertCache, hidden_size: int,
                 intermediate_size: int, reduction_mode=ReductionMode.CANONICAL,
                 execution_policy=ExpertExecutionPolicy.EXPERT_ID_ASCENDING,
                 h2d_prefetch: bool = True, swiglu_impl: int = N.SF_SWIGLU_AUTO) -> None:
        super().__init__()
        if layer_id < 0:
            raise ValueError("layer_id must be non-negative")
        if hidden_size <= 0:
            raise ValueError("hidden_size must be positive")
        if intermediate_size <= 0:
            raise ValueError("intermediate_size must be positive")
        if type(h2d_prefetch) is not bool:
            raise ValueError("h2d_prefetch must be a boolean")
        self.layer_id = layer_id
        self.cache = cache
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.reduction_mode = ReductionMode(reduction_mode)
        self.execution_policy = ExpertExecutionPolicy(execution_policy)
        self.h2d_prefetch = h2d_prefetch
        self.swiglu_impl = swiglu_impl
        # Resident fast path: read the token rows inside the grouped SwiGLU
        # (TMA gather4) instead of gathering a sorted copy first.
        self.fused_gather = False
        self._prediction_scheduler = None
        ids = [k.expert_id for k in cache.source_keys()
               if isinstance(k, ExpertKey) and k.layer_id == layer_id]
        self.num_experts = (max(ids) + 1) if ids else 0
        self._keys = tuple(ExpertKey(layer_id, e) for e in range(self.num_experts))

    # ------------------------------------------------------------ forward
    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                top_k_weights: torch.Tensor, *, execution_order: Sequence[int] | None = None):
        self._validate_inputs(hidden_states, top_k_index, top_k_weights)
        if self._prediction_scheduler is not None:
            if execution_order is not None:
                raise ValueError("explicit execution_order conflicts with dynamic predicted prefetch")
            return self._forward_scheduled(hidden_states, top_k_index, top_k_weights)
        tokens = hidden_states.shape[0]
        if tokens == 0:
            return torch.zeros_like(hidden_states)
        if self.num_experts == 0:
            raise KeyError(f"unknown expert {ExpertKey(self.layer_id, int(top_k_index.reshape(-1)[0]))!r}")
        h = hidden_states.contiguous()
        if self.cache.device_managed:
            if execution_order is not None:
                raise ValueError("an explicit execution_order needs a host-managed expert cache")
            ys, d = self._forward_device(h, top_k_index, top_k_weights)
            return ops.moe_combine(ys, d, top_k_index)
        d = ops.moe_dispatch(top_k_index, self.num_experts)
        xs, ws = ops.moe_gather(h, top_k_weights, d)
        storage = self.cache.storage.view(self.cache.slot_count, -1)
        # With every expert resident, both policies order the experts by id,
        # so arrival order equals the canonical order as well.
        fixed = self.cache.device_slot_table(self._keys) if execution_order is None else None
        if fixed is not None:
            # Every expert resident: one launch, no host round trip.
            ys = ops.grouped_swiglu(xs, ws, d, fixed, storage, self.hidden_size,
                                    self.intermediate_size, impl=self.swiglu_impl)
            out = ops.moe_combine(ys, d, top_k_index)
            self.cache.note_device_hits(d.num_active)  # after the combine: the MoE kernels run back to back
            return out
        return self._forward_waves(h, top_k_index, d, xs, ws, storage, execution_order)

    def forward_sorted(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                       top_k_weights: torch.Tensor):
        """The resident fast path of ``forward`` up to, not including, the
        combine: returns ``(ys, d)`` (weighted expert rows in sorted order and
        the dispatch) for a caller that fuses the combine with what follows,
        or ``None`` when that path does not apply (a prediction scheduler, an
        empty input, experts not all resident)."""
        self._validate_inputs(hidden_states, top_k_index, top_k_weights)
        if self._prediction_scheduler is not None or hidden_states.shape[0] == 0 or self.num_experts == 0:
            return None
        if self.cache.device_managed:
            return self._forward_device(hidden_states.contiguous(), top_k_index, top_k_weights)
        fixed = self.cache.device_slot_table(self._keys)
        if fixed is None:
            return None
        h = hidden_states.contiguous()
        # Every active expert is a resident hit: the dispatch launch counts them.
        d = ops.moe_dispatch(top_k_index, self.num_experts, active_total=self.cache.device_hit_counter())
        storage = self.cache.storage.view(self.cache.slot_count, -1)
        if self.fused_gather and self.swiglu_impl != N.SF_SWIGLU_SIMT:
            ys = ops.grouped_swiglu_gathered(h, top_k_weights, d, fixed, storage, self.hidden_size,
                                             self.intermediate_size)
            return ys, d
        xs, ws = ops.moe_gather(h, top_k_weights, d)
        ys = ops.grouped_swiglu(xs, ws, d, fixed, storage, self.hidden_size, self.intermediate_size,
                                impl=self.swiglu_impl)
        return ys, d

    def _forward_device(self, h, top_k_index, top_k_weights):
        """The layer with a device-managed cache: the directory plans the
        waves the host path would run (same leases, evictions and fills, in
        the same order) and each wave's misses are copied from host memory
        by a kernel, so nothing here waits for the device.  Returns the
        weighted expert rows in dispatch order and the dispatch."""
        cache = self.cache
        directory = cache.directory
        if cache.source_keys() != self._keys:
            raise RuntimeError("device-managed mode needs the cache's sources to be this layer's experts "
                               "in id order")
        if self.reduction_mode is not ReductionMode.CANONICAL:
            raise ValueError("device-managed mode reduces canonically only")
        stream = torch.cuda.current_stream(h.device).cuda_stream
        d = ops.moe_dispatch(top_k_index, self.num_experts)
        xs, ws = ops.moe_gather(h, top_k_weights, d)
        storage = cache.storage.view(cache.slot_count, -1)
        # Under graph capture the waves after the first go into the body of a
        # conditional node that the plan kernel opens only when the layer
        # needs more experts than its slots; eagerly, every wave is launched
        # (an empty one returns at once).
        later = (directory.capture_handle(stream)
                 if directory.waves > 1 and torch.cuda.is_current_stream_capturing() else 0)
        directory.plan(d, self.execution_policy is ExpertExecutionPolicy.RESIDENT_FIRST, stream, later)
        ys = torch.empty(xs.shape[0], self.hidden_size, dtype=h.dtype, device=h.device)
        act = torch.empty(max(xs.shape[0], 1), self.intermediate_size, dtype=h.dtype, device=h.device)

        def wave(w, st):
            directory.fill(w, storage, st)
            ops.grouped_swiglu(xs, ws, d, directory.wave_table[w], storage, self.hidden_size,
                               self.intermediate_size, impl=self.swiglu_impl, active=directory.wave_active[w],
                               num_active=directory.wave_count[w:w + 1], act_workspace=act, out=ys)

        wave(0, stream)
        if later:
            body = directory.later_waves_stream(h.device)
            N.check(N.lib.sf_capture_if_begin(stream, body.cuda_stream, later), "sf_capture_if_begin")
            try:
                with torch.cuda.stream(body):
                    for w in range(1, directory.waves):
                        wave(w, body.cuda_stream)
            finally:
                N.check(N.lib.sf_capture_if_end(stream, body.cuda_stream), "sf_capture_if_end")
        else:
            for w in range(1, directory.waves):
                wave(w, stream)
        ops._launched(1 + directory.waves)  # the plan and one fill per wave (SwiGLU counts itself)
        return ys, d

    def _forward_waves(self, h, top_k_index, d, xs, ws, storage, execution_order):
        dev = h.device
        host = torch.cat((d.num_active, d.error, d.active)).cpu()  # the one host sync
        n_active, err = int(host[0]), int(host[1])
        if err:
            bad = top_k_index[(top_k_index < 0) | (top_k_index >= self.num_experts)]
            raise KeyError(f"unknown expert {ExpertKey(self.layer_id, max(int(bad[0]), 0))!r}")
        active = tuple(int(e) for e in host[2:2 + n_active].tolist())
        order = self._resolve_execution_order(active, execution_order)
        ys = torch.empty(xs.shape[0], self.hidden_size, dtype=h.dtype, device=dev)
        act = torch.empty(max(xs.shape[0], 1), self.intermediate_size, dtype=h.dtype, device=dev)
        stream = torch.cuda.current_stream(dev)
        pos = 0
        while pos < len(order):
            # One native call leases the wave and submits all of its misses;
            # it stops at the first expert with no unleased slot left.
            leases = self.cache.acquire_many([self._keys[e] for e in order[pos:]])
            wave = list(zip(order[pos:pos + len(leases)], leases))
            try:
                table = torch.full((self.num_experts + 1 + len(wave),), -1, dtype=torch.int32)
                for j, (e, lease) in enumerate(wave):
                    lease.wait(stream)
                    table[e] = lease.slot_id
                    table[self.num_experts + 1 + j] = e
                table[self.num_experts] = len(wave)
                table = table.pin_memory().to(dev, non_blocking=True)
                ops.grouped_swiglu(xs, ws, d, table[: self.num_experts], storage, self.hidden_size,
                                   self.intermediate_size, impl=self.swiglu_impl,
                                   active=table[self.num_experts + 1:],
                                   num_active=table[self.num_experts: self.num_experts + 1],
                                   act_workspace=act, out=ys)
            finally:
                for _, lease in wave:
                    lease.release()
            pos += len(wave)
        rank = None
        if self.reduction_mode is ReductionMode.ARRIVAL_ORDER:
            r = torch.zeros(self.num_experts, dtype=torch.int32)
            for i, e in enumerate(order):
                r[e] = i
            rank = r.to(dev)
        return ops.moe_combine(ys, d, top_k_index, expert_rank=rank)

    def _forward_scheduled(self, hidden_states, top_k_index, top_k_weights):
        """Under ``Qwen3ExpertPrefetch`` (``_forward_prefetched``,
        qwen3_offloaded_experts.py:166-203): the layer's real experts are
        handed over one at a time, completed fills first; each runs as a
        one-expert grouped launch on its rows of the dispatch order, and the
        contributions are reduced once, canonically."""
        scheduler = self._prediction_scheduler
        dev = hidden_states.device
        if hidden_states.shape[0] == 0:
            for _ in scheduler.experts(self.layer_id, ()):
                pass
            return torch.zeros_like(hidden_states)
        if self.num_experts == 0:
            raise KeyError(f"unknown expert {ExpertKey(self.layer_id, int(top_k_index.reshape(-1)[0]))!r}")
        h = hidden_states.contiguous()
        d = ops.moe_dispatch(top_k_index, self.num_experts)
        host = torch.cat((d.num_active, d.error, d.active)).cpu()  # the router's experts
        n_active, err = int(host[0]), int(host[1])
        if err:
            bad = top_k_index[(top_k_index < 0) | (top_k_index >= self.num_experts)]
            raise KeyError(f"unknown expert {ExpertKey(self.layer_id, max(int(bad[0]), 0))!r}")
        active = tuple(int(e) for e in host[2:2 + n_active].tolist())
        E = self.num_experts
        # One pinned row per expert: slot table (E entries) | count 1 | the id.
        rows = torch.full((max(n_active, 1), E + 2), -1, dtype=torch.int32, pin_memory=True)
        storage = self.cache.storage.view(self.cache.slot_count, -1)
        stream = torch.cuda.current_stream(dev)
        xs = ws = ys = act = None
        with_tables = torch.empty(max(n_active, 1), E + 2, dtype=torch.int32, device=dev)
        for j, (expert_id, lease) in enumerate(scheduler.experts(self.layer_id, active)):
            with lease:
                if xs is None:
                    # The scheduler has submitted the real misses; gather now.
                    xs, ws = ops.moe_gather(h, top_k_weights, d)
                    ys = torch.empty(xs.shape[0], self.hidden_size, dtype=h.dtype, device=dev)
                    act = torch.empty(max(xs.shape[0], 1), self.intermediate_size, dtype=h.dtype,
                                      device=dev)
                lease.wait(stream)
                rows[j, expert_id] = lease.slot_id
                rows[j, E] = 1
                rows[j, E + 1] = expert_id
                table = with_tables[j]
                table.copy_(rows[j], non_blocking=True)
                ops.grouped_swiglu(xs, ws, d, table[:E], storage, self.hidden_size,
                                   self.intermediate_size, impl=self.swiglu_impl,
                                   active=table[E + 1:], num_active=table[E:E + 1],
                                   act_workspace=act, out=ys)
        return ops.moe_combine(ys, d, top_k_index)

    # --------------------------------------------------------- validation
    def _validate_inputs(self, hidden_states, top_k_index, top_k_weights) -> None:
        if hidden_states.ndim != 2:
            raise ValueError("hidden_states must have shape [tokens, hidden]")
        if hidden_states.shape[1] != self.hidden_size:
            raise ValueError(f"hidden_states width is {hidden_states.shape[1]}, expected {self.hidden_size}")
        if top_k_index.ndim != 2:
            raise ValueError("top_k_index must have shape [tokens, top_k]")
        if top_k_weights.shape != top_k_index.shape:
            raise ValueError("top_k_weights must match top_k_index shape")
        if top_k_index.shape[0] != hidden_states.shape[0]:
            raise ValueError("routing tensors must match the token count")
        if top_k_index.dtype is not torch.long:
            raise ValueError("top_k_index must use torch.long")
        if hidden_states.device != self.cache.device:
            raise ValueError("hidden_states must be on the cache device")
        if top_k_index.device != hidden_states.device:
            raise ValueError("top_k_index must be on the hidden-state device")
        if top_k_weights.device != hidden_states.device:
            raise ValueError("top_k_weights must be on the hidden-state device")

    def _resolve_execution_order(self, active_experts: tuple, execution_order) -> tuple:
        """Same policy as the reference (qwen3_offloaded_experts.py:262-292)."""
        if execution_order is not None:
            order = tuple(int(e) for e in execution_order)
            if len(order) != len(set(order)):
                raise ValueError("execution_order must not contain duplicates")
            if set(order) != set(active_experts):
                raise ValueError("execution_order must contain every active expert exactly once")
            return order
        if self.execution_policy is ExpertExecutionPolicy.EXPERT_ID_ASCENDING:
            return active_experts
        resident = frozenset(self.cache.resident_expert_ids())
        first = tuple(e for e in active_experts if ExpertKey(self.layer_id, e) in resident)
        return first + tuple(e for e in active_experts if ExpertKey(self.layer_id, e) not in resident)
