"""GPU expert cache: fixed device slots filled from pinned host copies.

Drop-in for ``GpuExpertCache`` (``src/specfit/runtime/gpu_expert_cache.py``):
same constructor, public methods, error types and messages, statistics and
observer events, and the private members other modules of the reference
touch.  Semantics kept:

* victim = the unleased slot minimising (occupied, last_used_sequence,
  slot_id) (:495-518); ``ready_only`` probing additionally needs the slot's
  fill and its readers' use events complete (:497-508);
* a miss bumps the slot generation, makes the copy stream wait for the
  previous readers' use events, copies the pinned source on the copy stream
  and records the slot's ready event (:543-589);
* finished copies become resident when polled in submission order (:591-609);
* leases pin a slot generation; release records a use event on every
  consumer stream (:684-718).

What is new here:

* the copy is issued through ``sf_slot_fill_batch`` (one ``cudaMemcpyAsync``
  per slot on the copy stream);
* ``storage`` / ``slot_stride`` expose the slot array to the grouped SwiGLU
  kernel, which reads expert weights straight from their slots;
* ``device_slot_table()``: when every source is resident and nothing is in
  flight (capacity >= sources), the slot of each expert is fixed, so the MoE
  block can run with no host synchronisation at all.  Hits in that mode are
  counted on the device (``note_device_hits``) and folded into ``stats()``.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass
from threading import RLock
from time import perf_counter_ns
from typing import Hashable, Mapping

import torch

from .. import ops
from .cache_snapshot import CacheSlotSnapshot, GpuExpertCacheSnapshot, PendingTransferSnapshot
from .lease import ExpertCacheStats, ExpertLease, NoEvictableSlotError
from .state import RuntimeEventKind


@dataclass(slots=True)
class _Counters:
    h2d_submissions: int = 0
    resident_hits: int = 0
    inflight_joins: int = 0
    evictions: int = 0


class _Slot:
    __slots__ = ("slot_id", "tensor", "expert_id", "generation", "active_leases",
                 "last_used_sequence", "ready_event", "use_events")

    def __init__(self, slot_id: int, tensor: torch.Tensor) -> None:
        self.slot_id = slot_id
        self.tensor = tensor
        self.expert_id = None
        self.generation = 0
        self.active_leases = 0
        self.last_used_sequence = 0
        self.ready_event = None
        self.use_events: dict = {}

    def copy_meta(self, tensor: torch.Tensor) -> "_Slot":
        other = _Slot(self.slot_id, tensor)
        other.expert_id = self.expert_id
        other.generation = self.generation
        other.active_leases = self.active_leases
        other.last_used_sequence = self.last_used_sequence
        other.ready_event = self.ready_event
        other.use_events = dict(self.use_events)
        return other


@dataclass(frozen=True, slots=True)
class _Transfer:
    expert_id: Hashable
    slot_id: int
    generation: int
    submission_sequence: int
    ready_event: object


@dataclass(frozen=True)
class _Checkpoint:
    owner: object
    weights: torch.Tensor
    slots: tuple
    resident: dict
    inflight: dict
    transfers: tuple
    counters: _Counters
    sequence: int
    submission_sequence: int
    state_version: int


class GpuExpertCache:
    def __init__(self, cpu_sources: Mapping[Hashable, torch.Tensor], *, slot_count: int,
                 device, adopt_pinned_sources: bool = False, cache_id: str | None = None,
                 queue_id: str | None = None, observer=None, source_owner=None) -> None:
        if not cpu_sources:
            raise ValueError("cpu_sources must contain at least one expert")
        if slot_count <= 0:
            raise ValueError("slot_count must be positive")
        if source_owner is not None and not adopt_pinned_sources:
            raise ValueError("source_owner requires adopt_pinned_sources=True")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("GpuExpertCache requires a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())

        items = list(cpu_sources.items())
        shape, dtype = items[0][1].shape, items[0][1].dtype
        self._sources: dict = {}
        self._source_order: dict = {}
        for order, (key, src) in enumerate(items):
            if src.device.type != "cpu":
                raise ValueError(f"expert {key!r} source must be on CPU")
            if src.shape != shape:
                raise ValueError("all expert sources must have the same shape")
            if src.dtype != dtype:
                raise ValueError("all expert sources must have the same dtype")
            if adopt_pinned_sources and src.is_pinned() and src.is_contiguous():
                pinned = src.detach()
            else:
                if source_owner is not None:
                    raise ValueError("owned expert sources must be contiguous pinned CPU tensors")
                pinned = torch.empty(src.shape, dtype=src.dtype, device="cpu", pin_memory=True)
                pinned.copy_(src.detach())
            self._sources[key] = pinned
            self._source_order[key] = order

        with torch.cuda.device(self.device):
            self.copy_stream = torch.cuda.Stream(device=self.device)
            self._storage = torch.empty((slot_count, *shape), dtype=dtype, device=self.device)
            # A recycled allocation may still have readers on the allocating
            # stream: order the first side-stream write after them.
            self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))
        for name, value in (("cache_id", cache_id), ("queue_id", queue_id)):
            if value is not None and (not isinstance(value, str) or not value):
                raise ValueError(f"{name} must be a non-empty string")
        self.cache_id = cache_id or f"cuda-{self.device.index}-stream-{int(self.copy_stream.cuda_stream)}"
        self.queue_id = queue_id or f"{self.cache_id}-copy"
        self._slots = [_Slot(i, self._storage[i]) for i in range(slot_count)]
        self._resident: dict = {}
        self._inflight: dict = {}
        self._outstanding_transfers: deque = deque()
        self._stats = _Counters()
        self._sequence = 0
        self._submission_sequence = 0
        self._state_version = 0
        self._observer = observer
        self._source_owner = source_owner
        self._closed = False
        self._closing = False
        self._lock = RLock()
        self._device_hits = None  # lazily created int64 device counter
        self._slot_table_cache = None  # (state_version, keys, tensor)

    # ------------------------------------------------------------ properties
    @property
    def storage(self) -> torch.Tensor:
        """``[slot_count, *source_shape]`` device tensor holding every slot."""
        return self._storage

    @property
    def slot_count(self) -> int:
        return len(self._slots)

    @property
    def sources_are_pinned(self) -> bool:
        return not (self._closed or self._closing) and all(s.is_pinned() for s in self._sources.values())

    @property
    def closed(self) -> bool:
        with self._lock:
            return self._closed

    @property
    def active_lease_count(self) -> int:
        with self._lock:
            return sum(slot.active_leases for slot in self._slots)

    def source_keys(self) -> tuple:
        return tuple(self._sources)

    # -------------------------------------------------------------- acquire
    def acquire(self, expert_id: Hashable) -> ExpertLease:
        return self._acquire(expert_id, defer_touch=False)

    def _prefetch(self, expert_id: Hashable) -> ExpertLease:
        return self._acquire(expert_id, defer_touch=True)

    def _check_open_and_known(self, expert_id: Hashable) -> None:
        if self._closed or self._closing:
            raise RuntimeError("expert cache is closed")
        if expert_id not in self._sources:
            raise KeyError(f"unknown expert {expert_id!r}")

    def _prefetch_nonblocking(self, expert_id: Hashable, *, resident_only: bool = False,
                              eviction_probabilities: Mapping | None = None) -> ExpertLease | None:
        with self._lock:
            self._check_open_and_known(expert_id)
            self._reap_completed_transfers()
            if expert_id in self._resident or expert_id in self._inflight:
                return self._acquire(expert_id, defer_touch=True)
            if resident_only:
                return None
            if eviction_probabilities is None:
                slot = self._choose_lru_slot(ready_only=True)
            else:
                slot = self._choose_probability_slot(expert_id, eviction_probabilities)
            if slot is None:
                return None
            self._assign_and_submit(slot, expert_id)
            return self._new_lease(slot, defer_touch=True)

    def _acquire(self, expert_id: Hashable, *, defer_touch: bool) -> ExpertLease:
        with self._lock:
            self._check_open_and_known(expert_id)
            self._reap_completed_transfers()
            transfer = self._inflight.get(expert_id)
            if transfer is not None:
                slot = self._slots[transfer.slot_id]
                self._emit(RuntimeEventKind.INFLIGHT_JOIN, expert_id, slot,
                           submission_sequence=transfer.submission_sequence,
                           ready_event=transfer.ready_event)
                self._stats.inflight_joins += 1
                return self._new_lease(slot, defer_touch=defer_touch)
            slot_id = self._resident.get(expert_id)
            if slot_id is not None:
                slot = self._slots[slot_id]
                self._emit(RuntimeEventKind.RESIDENT_HIT, expert_id, slot)
                self._stats.resident_hits += 1
                lease = self._new_lease(slot, defer_touch=defer_touch)
                lease._ready_confirmed = True  # resident => its copy completed
                return lease
            slot = self._choose_lru_slot()
            if slot is None:
                raise NoEvictableSlotError("all GPU expert slots have active leases")
            self._assign_and_submit(slot, expert_id)
            return self._new_lease(slot, defer_touch=defer_touch)

    # ------------------------------------------------------------ victims
    @staticmethod
    def _lru_key(slot: _Slot):
        return (slot.expert_id is not None, slot.last_used_sequence, slot.slot_id)

    def _slot_writable(self, slot: _Slot) -> bool:
        copied = (slot.ready_event is None or self._resident.get(slot.expert_id) == slot.slot_id
                  or slot.ready_event.query())
        return copied and all(ev.query() for ev in slot.use_events.values())

    def _choose_lru_slot(self, *, ready_only: bool = False) -> _Slot | None:
        free = [s for s in self._slots if s.active_leases == 0]
        if not free:
            return None
        if not ready_only:
            return min(free, key=self._lru_key)
        for slot in sorted(free, key=self._lru_key):
            if self._slot_writable(slot):
                return slot
        return None

    def _choose_probability_slot(self, expert_id: Hashable, probabilities: Mapping) -> _Slot | None:
        """Replace an unleased, writable expert whose probability is lower
        than the incoming one's (gpu_expert_cache.py:520-541)."""
        incoming = probabilities.get(expert_id, 0.0)
        free = [s for s in self._slots if s.active_leases == 0]
        order = sorted(free, key=lambda s: (s.expert_id is not None,
                                            probabilities.get(s.expert_id, 0.0),
                                            s.last_used_sequence, s.slot_id))
        for slot in order:
            if slot.expert_id is not None and probabilities.get(slot.expert_id, 0.0) >= incoming:
                break
            if self._slot_writable(slot):
                return slot
        return None

    # --------------------------------------------------------------- fills
    def _assign_and_submit(self, slot: _Slot, expert_id: Hashable) -> None:
        victim = slot.expert_id
        if victim is not None:
            self._resident.pop(victim, None)
            self._inflight.pop(victim, None)
            self._stats.evictions += 1
        slot.generation += 1
        slot.expert_id = expert_id
        guards = tuple(slot.use_events.values())
        slot.use_events.clear()
        stream = self.copy_stream
        for guard in guards:
            stream.wait_event(guard)
        ops.slot_fill_batch([slot.tensor], [self._sources[expert_id]], stream)
        ready = torch.cuda.Event(blocking=False)
        ready.record(stream)
        slot.ready_event = ready
        transfer = _Transfer(expert_id, slot.slot_id, slot.generation, self._submission_sequence, ready)
        self._inflight[expert_id] = transfer
        self._outstanding_transfers.append(transfer)
        self._stats.h2d_submissions += 1
        self._submission_sequence += 1
        if victim is not None:
            self._emit(RuntimeEventKind.EVICT, expert_id, slot, victim_expert_id=victim)
        self._emit(RuntimeEventKind.H2D_SUBMIT, expert_id, slot,
                   submission_sequence=transfer.submission_sequence, ready_event=ready)

    def _reap_completed_transfers(self) -> None:
        changed = False
        pending = self._outstanding_transfers
        while pending and pending[0].ready_event.query():
            t = pending.popleft()
            slot = self._slots[t.slot_id]
            if slot.expert_id == t.expert_id and slot.generation == t.generation:
                self._resident[t.expert_id] = t.slot_id
            if self._inflight.get(t.expert_id) == t:
                del self._inflight[t.expert_id]
            changed = True
        if changed:
            self._state_version += 1

    def _reap_completed_use_guards(self) -> None:
        changed = False
        for slot in self._slots:
            for sid, ev in list(slot.use_events.items()):
                if ev.query():
                    del slot.use_events[sid]
                    changed = True
        if changed:
            self._state_version += 1

    # -------------------------------------------------------------- leases
    def _touch(self, slot: _Slot) -> None:
        self._sequence += 1
        self._state_version += 1
        slot.last_used_sequence = self._sequence

    def _new_lease(self, slot: _Slot, *, defer_touch: bool) -> ExpertLease:
        if slot.expert_id is None or slot.ready_event is None:
            raise RuntimeError("cannot lease an unassigned GPU slot")
        slot.active_leases += 1
        if defer_touch:
            self._state_version += 1
        else:
            self._touch(slot)
        return ExpertLease(self, slot.expert_id, slot.slot_id, slot.generation, slot.ready_event,
                           _defer_touch=defer_touch)

    def _checked_slot(self, expert_id, slot_id: int, generation: int) -> _Slot:
        slot = self._slots[slot_id]
        if slot.expert_id != expert_id or slot.generation != generation or slot.active_leases <= 0:
            raise RuntimeError("expert lease refers to a reused GPU slot")
        return slot

    def _lease_tensor(self, expert_id, slot_id: int, generation: int, *, touch: bool = False):
        with self._lock:
            slot = self._checked_slot(expert_id, slot_id, generation)
            if touch:
                self._touch(slot)
            return slot.tensor

    def _record_consume_wait(self, *, expert_id, slot_id, generation, ready_event, stream) -> None:
        if self._observer is None:
            return
        self._observer.record(kind=RuntimeEventKind.CONSUME_WAIT, cache_id=self.cache_id,
                              queue_id=self.queue_id, expert_id=expert_id, slot_id=slot_id,
                              generation=generation, ready_event=ready_event,
                              stream_ids=(int(stream.cuda_stream),))

    def _release(self, expert_id, slot_id: int, generation: int, used_streams: tuple) -> None:
        with self._lock:
            slot = self._checked_slot(expert_id, slot_id, generation)
            for stream in used_streams:
                ev = torch.cuda.Event(blocking=False)
                ev.record(stream)
                slot.use_events[stream.cuda_stream] = ev
            self._emit(RuntimeEventKind.RELEASE, expert_id, slot,
                       stream_ids=tuple(sorted(int(s.cuda_stream) for s in used_streams)))
            slot.active_leases -= 1
            self._touch(slot)

    def _emit(self, kind, expert_id, slot: _Slot, *, submission_sequence=None, victim_expert_id=None,
              ready_event=None, stream_ids=()) -> None:
        if self._observer is None:
            return
        self._observer.record(kind=kind, cache_id=self.cache_id, queue_id=self.queue_id,
                              expert_id=expert_id, slot_id=slot.slot_id, generation=slot.generation,
                              submission_sequence=submission_sequence,
                              victim_expert_id=victim_expert_id, ready_event=ready_event,
                              stream_ids=stream_ids)

    # ---------------------------------------------------------- fast path
    def device_slot_table(self, keys) -> torch.Tensor | None:
        """int32 device tensor with the slot of each key, or ``None`` unless
        every source is resident with nothing in flight or leased and the
        cache holds all sources (so no slot can change while it is used)."""
        with self._lock:
            if self._closed or self._closing:
                raise RuntimeError("expert cache is closed")
            if len(self._slots) < len(self._sources):
                return None
            self._reap_completed_transfers()
            if self._inflight or len(self._resident) != len(self._sources):
                return None
            keys = tuple(keys)
            cached = self._slot_table_cache
            if cached is not None and cached[0] == self._state_version and cached[1] == keys:
                return cached[2]
            table = torch.tensor([self._resident.get(k, -1) for k in keys], dtype=torch.int32)
            table = table.to(self.device, non_blocking=False)
            self._slot_table_cache = (self._state_version, keys, table)
            return table

    def device_hit_counter(self) -> torch.Tensor:
        """The device int64 scalar that kernels add resident hits to
        (``ops.moe_dispatch(..., active_total=)``); read on the host only
        when the statistics are read."""
        if self._device_hits is None:
            self._device_hits = torch.zeros((), dtype=torch.int64, device=self.device)
        return self._device_hits

    def note_device_hits(self, count: torch.Tensor) -> None:
        """Adds a device-side count of resident hits (no host sync)."""
        if self._device_hits is None:
            self._device_hits = torch.zeros((), dtype=torch.int64, device=self.device)
        self._device_hits.add_(count.reshape(()))  # int32 into the int64 total, one launch

    def _flush_device_hits(self) -> None:
        if self._device_hits is not None:
            self._stats.resident_hits += int(self._device_hits.item())
            self._device_hits.zero_()

    def prefill_all(self) -> None:
        """Submit a fill for every non-resident source (warm-up helper)."""
        for key in self._sources:
            with self._lock:
                self._reap_completed_transfers()
                if key in self._resident or key in self._inflight:
                    continue
            self.acquire(key).release()

    # ---------------------------------------------------------- inspection
    def stats(self) -> ExpertCacheStats:
        with self._lock:
            self._flush_device_hits()
            self._reap_completed_use_guards()
            return self._stats_snapshot()

    def _stats_snapshot(self, *, pending_use_guards: int | None = None) -> ExpertCacheStats:
        if pending_use_guards is None:
            pending_use_guards = sum(len(s.use_events) for s in self._slots)
        return ExpertCacheStats(self._stats.h2d_submissions, self._stats.resident_hits,
                                self._stats.inflight_joins, self._stats.evictions,
                                pending_use_guards)

    def resident_expert_ids(self) -> tuple:
        with self._lock:
            self._reap_completed_transfers()
            return tuple(sorted(self._resident, key=self._source_order.__getitem__))

    def snapshot(self) -> GpuExpertCacheSnapshot:
        with self._lock:
            self._flush_device_hits()
            done = {t.submission_sequence: t.ready_event.query() for t in self._outstanding_transfers}
            guards = {s.slot_id: sum(not ev.query() for ev in s.use_events.values()) for s in self._slots}
            current = {(t.slot_id, t.generation): t for t in self._inflight.values()}
            slots = []
            for s in self._slots:
                t = current.get((s.slot_id, s.generation))
                if s.expert_id is None:
                    ready = False
                elif t is not None:
                    ready = done[t.submission_sequence]
                else:
                    ready = s.expert_id in self._resident
                slots.append(CacheSlotSnapshot(s.slot_id, s.expert_id, s.generation, s.active_leases,
                                               s.last_used_sequence, ready, guards[s.slot_id]))
            pending = tuple(
                PendingTransferSnapshot(t.expert_id, t.slot_id, t.generation, t.submission_sequence,
                                        t.ready_event, False)
                for t in self._outstanding_transfers if not done[t.submission_sequence])
            return GpuExpertCacheSnapshot(self.cache_id, self.queue_id, len(self._slots),
                                          self._state_version, self._sequence,
                                          self._submission_sequence, tuple(slots), pending,
                                          self._stats_snapshot(pending_use_guards=sum(guards.values())))

    # ----------------------------------------------------- reset / restore
    def _quiescent(self) -> bool:
        return (all(t.ready_event.query() for t in self._outstanding_transfers)
                and all(ev.query() for s in self._slots for ev in s.use_events.values()))

    def cold_reset(self) -> None:
        with self._lock:
            if self._closed or self._closing:
                raise RuntimeError("expert cache is closed")
            if any(s.active_leases for s in self._slots):
                raise RuntimeError("cold reset cannot run while an active lease exists")
            if not self._quiescent():
                raise RuntimeError("cold reset requires explicit CUDA synchronization")
            if self._device_hits is not None:
                self._device_hits.zero_()
            self._resident.clear()
            self._inflight.clear()
            self._outstanding_transfers.clear()
            for s in self._slots:
                s.expert_id = None
                s.generation = 0
                s.active_leases = 0
                s.last_used_sequence = 0
                s.ready_event = None
                s.use_events.clear()
            self._stats = _Counters()
            self._sequence = 0
            self._submission_sequence = 0
            self._state_version = 0
            self._slot_table_cache = None

    def _require_checkpoint_boundary(self) -> None:
        if self._closed or self._closing:
            raise RuntimeError("expert cache is closed")
        if self._observer is not None:
            raise RuntimeError("checkpoint restoration requires no active cache observer")
        if any(s.active_leases for s in self._slots):
            raise RuntimeError("checkpoint boundary cannot contain active leases")
        if not self._quiescent():
            raise RuntimeError("checkpoint boundary requires explicit CUDA synchronization")

    def _capture_checkpoint(self) -> _Checkpoint:
        with self._lock:
            self._require_checkpoint_boundary()
            self._flush_device_hits()
            weights = torch.empty_like(self._storage, device="cpu", pin_memory=True)
            weights.copy_(self._storage.detach())
            counters = _Counters(**{f: getattr(self._stats, f) for f in _Counters.__slots__})
            return _Checkpoint(self, weights, tuple(s.copy_meta(weights[s.slot_id]) for s in self._slots),
                               dict(self._resident), dict(self._inflight),
                               tuple(self._outstanding_transfers), counters, self._sequence,
                               self._submission_sequence, self._state_version)

    def _restore_checkpoint(self, checkpoint: _Checkpoint) -> dict:
        started = perf_counter_ns()
        with self._lock:
            self._require_checkpoint_boundary()
            if checkpoint.owner is not self:
                raise ValueError("expert checkpoint belongs to a different cache instance")
            checked = perf_counter_ns()
            self._storage.copy_(checkpoint.weights)
            copied = perf_counter_ns()
            torch.cuda.current_stream(self.device).synchronize()
            synced = perf_counter_ns()
            self._slots = [s.copy_meta(self._storage[s.slot_id]) for s in checkpoint.slots]
            self._resident = dict(checkpoint.resident)
            self._inflight = dict(checkpoint.inflight)
            self._outstanding_transfers = deque(checkpoint.transfers)
            self._stats = _Counters(**{f: getattr(checkpoint.counters, f) for f in _Counters.__slots__})
            self._sequence = checkpoint.sequence
            self._submission_sequence = checkpoint.submission_sequence
            self._state_version = checkpoint.state_version
            self._slot_table_cache = None
            finished = perf_counter_ns()
            return dict(weight_bytes=checkpoint.weights.numel() * checkpoint.weights.element_size(),
                        weights_pinned=checkpoint.weights.is_pinned(),
                        total_wall_ns=finished - started,
                        timings_ns=dict(boundary_check=checked - started,
                                        weight_copy_call=copied - checked,
                                        stream_synchronize=synced - copied,
                                        metadata_restore=finished - synced))

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            if not self._closing and any(s.active_leases for s in self._slots):
                raise RuntimeError("expert cache cannot close while an active lease exists")
            self._closing = True
            torch.cuda.synchronize(self.device)
            self._resident.clear()
            self._inflight.clear()
            self._outstanding_transfers.clear()
            for s in self._slots:
                s.expert_id = None
                s.ready_event = None
                s.use_events.clear()
            self._sources.clear()
            owner, self._source_owner = self._source_owner, None
            if owner is not None:
                owner.close()
            self._slot_table_cache = None
            self._closed = True
            self._closing = False
