"""GPU expert cache: a Python face over the native slot manager.

Drop-in for ``GpuExpertCache`` (``src/specfit/runtime/gpu_expert_cache.py``):
same constructor, public methods, error types and messages, statistics,
observer records and snapshots, and the private members other modules of
the reference read or edit (``_slots``, ``_resident``, ``_inflight``,
``_outstanding_transfers``, ``_submission_sequence``, ``_state_version``,
``_sources``, ``_lock``, ``_prefetch``, ``_prefetch_nonblocking``, the
checkpoint hooks).

Where the work happens.  All slot bookkeeping — which slot an expert is in,
generations, the LRU order, fill submission and publication, use guards,
counters — lives in the native manager (``csrc/expert_cache.cu``, C ABI
``sf_cache_*``).  This class owns the tensors (device slots, page-locked
sources), the ``torch.cuda.Event`` objects that stand for fills, the
observer calls, and translation between expert keys and the manager's
expert indices.  The private members above are *views* that read the
manager's state and write edits through to it, so code that clears
``_resident`` or edits a slot's ``generation`` keeps working.

Additions over the reference:

* ``acquire_many(keys)``: a wave of leases in one native call; every miss of
  the wave is submitted to the copy engines by that call;
* ``storage`` for the grouped SwiGLU kernel, which reads expert weights
  straight from their slots, and ``device_slot_table()`` for the case where
  every expert is resident (the MoE block then runs with no host
  synchronisation; its hits are counted on the device and folded into
  ``stats()``);
* device-managed mode (``enter_device_mode`` / ``leave_device_mode``): the
  bookkeeping moves to HBM (``runtime/expert_directory.py``) and misses are
  planned and filled on the device, so a pass with misses needs no host
  round trip; reading ``stats()`` / ``snapshot()`` mirrors the device state
  back, and host leases are refused until the mode is left.
"""
from __future__ import annotations

import ctypes
import weakref
from dataclasses import dataclass
from threading import RLock
from time import perf_counter_ns
from typing import Hashable, Iterable, Mapping

import torch

from .. import _native as N
from .cache_snapshot import CacheSlotSnapshot, GpuExpertCacheSnapshot, PendingTransferSnapshot
from .expert_directory import DeviceExpertDirectory
from .lease import ExpertCacheStats, ExpertLease, NoEvictableSlotError
from .state import RuntimeEventKind

_ABSENT, _INFLIGHT, _RESIDENT = 0, 1, 2


@dataclass(frozen=True, slots=True)
class _Transfer:
    """One outstanding fill as the reference's transfer records expose it."""
    expert_id: Hashable
    slot_id: int
    generation: int
    submission_sequence: int
    ready_event: object


@dataclass(frozen=True)
class _Checkpoint:
    owner: object
    weights: torch.Tensor
    image: bytes
    events: dict
    device_hits: int


class _NativeState:
    """One read of the manager's state: counters, slots, expert locations."""

    __slots__ = ("counters", "slots", "where", "home", "fill_seq")

    def __init__(self, cache: "GpuExpertCache", refresh: int) -> None:
        n_slots, n_exp = cache._n_slots, len(cache._keys)
        self.counters = N.SfCacheCounters()
        self.slots = (N.SfCacheSlot * n_slots)()
        self.where = (ctypes.c_int32 * n_exp)()
        self.home = (ctypes.c_int32 * n_exp)()
        self.fill_seq = (ctypes.c_int64 * n_exp)()
        N.check(N.lib.sf_cache_state(cache._h, refresh, ctypes.byref(self.counters), self.slots,
                                     self.where, self.home, self.fill_seq), "sf_cache_state")


# ------------------------------------------------------------------ views


class _SlotView:
    """A slot as the reference's ``_Slot`` records it; edits write through."""

    __slots__ = ("_cache", "slot_id")

    def __init__(self, cache: "GpuExpertCache", slot_id: int) -> None:
        self._cache = weakref.proxy(cache)  # no reference cycle: a closed cache frees its slots at once
        self.slot_id = slot_id

    def _row(self):
        return _NativeState(self._cache, 0).slots[self.slot_id]

    def _edit(self, field: int, value: int) -> None:
        N.check(N.lib.sf_cache_slot_edit(self._cache._h, self.slot_id, field, value), "sf_cache_slot_edit")

    @property
    def tensor(self) -> torch.Tensor:
        return self._cache._storage[self.slot_id]

    @property
    def expert_id(self):
        e = self._row().expert
        return None if e < 0 else self._cache._keys[e]

    @expert_id.setter
    def expert_id(self, value) -> None:
        if value is not None:
            raise ValueError("a slot's expert can only be cleared")
        self._edit(N.SF_SLOT_EXPERT, -1)

    @property
    def generation(self) -> int:
        return int(self._row().generation)

    @generation.setter
    def generation(self, value: int) -> None:
        self._edit(N.SF_SLOT_GENERATION, int(value))

    @property
    def last_used_sequence(self) -> int:
        return int(self._row().stamp)

    @last_used_sequence.setter
    def last_used_sequence(self, value: int) -> None:
        self._edit(N.SF_SLOT_STAMP, int(value))

    @property
    def active_leases(self) -> int:
        return int(self._row().leases)

    @property
    def ready_event(self):
        return self._cache._events.get(int(self._row().ready_event))

    @ready_event.setter
    def ready_event(self, value) -> None:
        if value is not None:
            raise ValueError("a slot's ready event can only be cleared")
        self._edit(N.SF_SLOT_READY, 0)

    @property
    def use_events(self) -> "_GuardView":
        return _GuardView(self)


class _GuardView:
    """A slot's use guards: counted and cleared (the events stay native)."""

    __slots__ = ("_slot",)

    def __init__(self, slot: _SlotView) -> None:
        self._slot = slot

    def __len__(self) -> int:
        return int(self._slot._row().guards)

    def clear(self) -> None:
        self._slot._edit(N.SF_SLOT_GUARDS, 0)


class _LocationView:
    """Experts at one location (resident, or in flight) as a read-mostly
    mapping: resident experts map to their slot, in-flight ones to their
    transfer record.  ``clear()`` forgets that location for every expert."""

    __slots__ = ("_cache", "_code")

    def __init__(self, cache: "GpuExpertCache", code: int) -> None:
        self._cache = weakref.proxy(cache)
        self._code = code

    def _items(self):
        cache = self._cache
        st = _NativeState(cache, 1)
        out = {}
        for e, key in enumerate(cache._keys):
            if st.where[e] != self._code:
                continue
            slot = int(st.home[e])
            if self._code == _RESIDENT:
                out[key] = slot
            else:
                row = st.slots[slot]
                out[key] = _Transfer(key, slot, int(row.generation), int(st.fill_seq[e]),
                                     cache._events.get(int(row.ready_event)))
        return out

    def __contains__(self, key) -> bool:
        e = self._cache._index.get(key)
        return e is not None and _NativeState(self._cache, 1).where[e] == self._code

    def get(self, key, default=None):
        return self._items().get(key, default)

    def __getitem__(self, key):
        return self._items()[key]

    def __len__(self) -> int:
        st = _NativeState(self._cache, 1)
        return sum(1 for e in range(len(self._cache._keys)) if st.where[e] == self._code)

    def __bool__(self) -> bool:
        return len(self) > 0

    def __iter__(self):
        return iter(self._items())

    def keys(self):
        return self._items().keys()

    def values(self):
        return self._items().values()

    def items(self):
        return self._items().items()

    def clear(self) -> None:
        N.check(N.lib.sf_cache_forget(self._cache._h, 1 if self._code == _RESIDENT else 2), "sf_cache_forget")


class _FillQueueView:
    """Outstanding fills in submission order (``_Transfer`` records)."""

    __slots__ = ("_cache",)

    def __init__(self, cache: "GpuExpertCache") -> None:
        self._cache = weakref.proxy(cache)

    def _rows(self):
        return self._cache._native_fills()

    def __iter__(self):
        cache = self._cache
        return iter([_Transfer(cache._keys[f.expert], int(f.slot), int(f.generation), int(f.submission),
                               cache._events.get(int(f.ready_event))) for f in self._rows()])

    def __len__(self) -> int:
        return len(self._rows())

    def __bool__(self) -> bool:
        return len(self) > 0

    def clear(self) -> None:
        N.check(N.lib.sf_cache_forget(self._cache._h, 4), "sf_cache_forget")


# ------------------------------------------------------------------ cache


def _pinned_sources(cpu_sources: Mapping, adopt: bool, owned: bool) -> dict:
    """Validates the host sources and returns them page-locked and
    contiguous, in source order (adopting tensors that already are)."""
    items = list(cpu_sources.items())
    shape, dtype = items[0][1].shape, items[0][1].dtype
    out = {}
    for key, src in items:
        if src.device.type != "cpu":
            raise ValueError(f"expert {key!r} source must be on CPU")
        if src.shape != shape:
            raise ValueError("all expert sources must have the same shape")
        if src.dtype != dtype:
            raise ValueError("all expert sources must have the same dtype")
        if adopt and src.is_pinned() and src.is_contiguous():
            out[key] = src.detach()
            continue
        if owned:
            raise ValueError("owned expert sources must be contiguous pinned CPU tensors")
        pinned = torch.empty(src.shape, dtype=src.dtype, device="cpu", pin_memory=True)
        pinned.copy_(src.detach())
        out[key] = pinned
    return out


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
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("GpuExpertCache requires a CUDA device")
        self.device = dev if dev.index is not None else torch.device("cuda", torch.cuda.current_device())
        self._sources = _pinned_sources(cpu_sources, adopt_pinned_sources, source_owner is not None)
        self._keys = tuple(self._sources)
        self._index = {k: i for i, k in enumerate(self._keys)}
        first = self._sources[self._keys[0]]
        with torch.cuda.device(self.device):
            self._copy_stream = torch.cuda.Stream(device=self.device)
            self._storage = torch.empty((slot_count, *first.shape), dtype=first.dtype, device=self.device)
            # The slots may reuse memory still read on the allocating stream.
            self._copy_stream.wait_stream(torch.cuda.current_stream(self.device))
        for name, value in (("cache_id", cache_id), ("queue_id", queue_id)):
            if value is not None and (not isinstance(value, str) or not value):
                raise ValueError(f"{name} must be a non-empty string")
        self.cache_id = cache_id or f"cuda-{self.device.index}-stream-{int(self._copy_stream.cuda_stream)}"
        self.queue_id = queue_id or f"{self.cache_id}-copy"

        self._n_slots = slot_count
        srcs = (ctypes.c_void_p * len(self._keys))(*[self._sources[k].data_ptr() for k in self._keys])
        h = ctypes.c_void_p()
        N.check(N.lib.sf_cache_create(slot_count, len(self._keys), self._storage.data_ptr(),
                                      first.numel() * first.element_size(), srcs,
                                      self._copy_stream.cuda_stream, ctypes.byref(h)), "sf_cache_create")
        self._h = h.value
        self._slots = [_SlotView(self, i) for i in range(slot_count)]
        self._resident = _LocationView(self, _RESIDENT)
        self._inflight = _LocationView(self, _INFLIGHT)
        self._outstanding_transfers = _FillQueueView(self)
        self._events: dict = {}          # ready-event handle -> torch.cuda.Event
        self._spare_events: list = []    # created, never used for a fill yet
        self._observer = observer
        self._source_owner = source_owner
        self._closed = False
        self._closing = False
        self._lock = RLock()
        self._device_hits = None         # int64 device counter of fast-path hits
        self._table = None               # (state version, keys, device slot table)
        self._directory = None           # DeviceExpertDirectory, built on first use
        self._device_mode = False

    # ------------------------------------------------------------ properties
    @property
    def copy_stream(self) -> torch.cuda.Stream:
        return self._copy_stream

    @copy_stream.setter
    def copy_stream(self, stream: torch.cuda.Stream) -> None:
        N.check(N.lib.sf_cache_set_copy_stream(self._h, stream.cuda_stream), "sf_cache_set_copy_stream")
        self._copy_stream = stream

    @property
    def storage(self) -> torch.Tensor:
        """``[slot_count, *source_shape]`` device tensor holding every slot."""
        return self._storage

    @property
    def slot_count(self) -> int:
        return self._n_slots

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
            if self._closed:
                return 0
            st = _NativeState(self, 0)
            return sum(int(st.slots[s].leases) for s in range(self._n_slots))

    @property
    def _submission_sequence(self) -> int:
        return int(_NativeState(self, 0).counters.submission_sequence)

    @property
    def _sequence(self) -> int:
        return int(_NativeState(self, 0).counters.sequence)

    @property
    def _state_version(self) -> int:
        return int(_NativeState(self, 0).counters.state_version)

    @_state_version.setter
    def _state_version(self, value: int) -> None:
        N.check(N.lib.sf_cache_set_version(self._h, int(value)), "sf_cache_set_version")

    def source_keys(self) -> tuple:
        return self._keys

    def holds_any(self) -> bool:
        """Whether any expert is resident or in flight."""
        st = _NativeState(self, 0)
        return any(st.where[e] != _ABSENT for e in range(len(self._keys)))

    # ---------------------------------------------------------------- events
    def _fresh_event_handles(self, n: int):
        """``n`` created (not yet fill-bound) ready events; the manager records
        the ones it uses behind their fills."""
        while len(self._spare_events) < n:
            ev = torch.cuda.Event(blocking=False)
            ev.record(self._copy_stream)  # creates the CUDA event; re-recorded after the copy
            self._spare_events.append(ev)
        return (ctypes.c_uint64 * n)(*[ev.cuda_event for ev in self._spare_events[:n]])

    def _adopt_events(self, handles: Iterable[int]) -> None:
        used = set(handles)
        if not used:
            return
        keep = []
        for ev in self._spare_events:
            if ev.cuda_event in used:
                self._events[ev.cuda_event] = ev
            else:
                keep.append(ev)
        self._spare_events = keep
        if len(self._events) > 4 * self._n_slots + 64:
            self._prune_events()

    def _prune_events(self) -> None:
        """Drops the Python references to events the manager no longer holds
        (leases, snapshots and observers keep their own references)."""
        st = _NativeState(self, 0)
        live = {int(st.slots[s].ready_event) for s in range(self._n_slots)}
        live.update(int(f.ready_event) for f in self._native_fills())
        self._events = {h: ev for h, ev in self._events.items() if h in live}

    def _native_fills(self):
        n = ctypes.c_int()
        N.check(N.lib.sf_cache_fills(self._h, None, 0, ctypes.byref(n)), "sf_cache_fills")
        buf = (N.SfCacheFill * max(n.value, 1))()
        N.check(N.lib.sf_cache_fills(self._h, buf, len(buf), ctypes.byref(n)), "sf_cache_fills")
        return list(buf[: n.value])

    # --------------------------------------------------------------- acquire
    def _check_open(self) -> None:
        if self._closed or self._closing:
            raise RuntimeError("expert cache is closed")

    def _check_host_managed(self) -> None:
        self._check_open()
        if self._device_mode:
            raise RuntimeError("expert cache is device-managed: call leave_device_mode() first")

    def _indices(self, keys) -> list:
        out = []
        for key in keys:
            e = self._index.get(key)
            if e is None:
                raise KeyError(f"unknown expert {key!r}")
            out.append(e)
        return out

    def _grant(self, keys, mode: int, defer_touch: bool, probabilities=None) -> list:
        """Runs one native acquire over ``keys``; returns a lease per key
        (``None`` where nothing was granted), emitting the observer records
        of every hit, join, eviction and submission in order."""
        self._check_host_managed()
        idx = self._indices(keys)
        n = len(idx)
        if n == 0:
            return []
        experts = (ctypes.c_int32 * n)(*idx)
        fresh = self._fresh_event_handles(n) if mode != N.SF_CACHE_RESIDENT_ONLY else None
        probs = None
        if probabilities is not None:
            probs = (ctypes.c_float * len(self._keys))(*[float(probabilities.get(k, 0.0)) for k in self._keys])
        grants = (N.SfCacheGrant * n)()
        granted = ctypes.c_int()
        rc = N.lib.sf_cache_acquire(self._h, experts, n, mode, int(defer_touch), fresh, probs, grants,
                                    ctypes.byref(granted))
        if rc == N.SF_ERR_NO_SLOT:
            raise NoEvictableSlotError("all GPU expert slots have active leases")
        N.check(rc, "sf_cache_acquire")
        self._adopt_events(int(g.ready_event) for g in grants if g.kind == N.SF_GRANT_MISS)
        leases = []
        for key, g in zip(keys, grants):
            if g.kind == N.SF_GRANT_NONE:
                leases.append(None)
                continue
            ready = self._events.get(int(g.ready_event))
            if self._observer is not None:
                self._report_grant(key, g, ready)
            leases.append(ExpertLease(self, key, self._index[key], int(g.slot), int(g.generation), ready,
                                      defer_touch=defer_touch, grant=(int(g.kind), int(g.submission))))
        return leases

    def _report_grant(self, key, g, ready) -> None:
        slot, gen = int(g.slot), int(g.generation)
        if g.kind == N.SF_GRANT_HIT:
            self._emit(RuntimeEventKind.RESIDENT_HIT, key, slot, gen)
        elif g.kind == N.SF_GRANT_JOIN:
            self._emit(RuntimeEventKind.INFLIGHT_JOIN, key, slot, gen,
                       submission_sequence=int(g.submission), ready_event=ready)
        else:
            if g.victim >= 0:
                self._emit(RuntimeEventKind.EVICT, key, slot, gen, victim_expert_id=self._keys[g.victim])
            self._emit(RuntimeEventKind.H2D_SUBMIT, key, slot, gen, submission_sequence=int(g.submission),
                       ready_event=ready)

    def acquire(self, expert_id: Hashable) -> ExpertLease:
        with self._lock:
            return self._grant((expert_id,), N.SF_CACHE_ACQUIRE, False)[0]

    def acquire_many(self, expert_ids) -> list:
        """Leases for ``expert_ids`` in order, as consecutive ``acquire``
        calls would give them, with every miss submitted by one native call.
        Stops early (a shorter list) at the first expert for which every
        slot is leased; raises ``NoEvictableSlotError`` if that is the first."""
        with self._lock:
            return [l for l in self._grant(tuple(expert_ids), N.SF_CACHE_ACQUIRE, False) if l is not None]

    def _prefetch(self, expert_id: Hashable) -> ExpertLease:
        with self._lock:
            return self._grant((expert_id,), N.SF_CACHE_ACQUIRE, True)[0]

    def _prefetch_nonblocking(self, expert_id: Hashable, *, resident_only: bool = False,
                              eviction_probabilities: Mapping | None = None) -> ExpertLease | None:
        if resident_only:
            mode = N.SF_CACHE_RESIDENT_ONLY
        elif eviction_probabilities is not None:
            mode = N.SF_CACHE_PROBABILITY
        else:
            mode = N.SF_CACHE_NONBLOCKING
        with self._lock:
            return self._grant((expert_id,), mode, True, eviction_probabilities)[0]

    # ---------------------------------------------------------------- leases
    def _lease_wait(self, lease: ExpertLease, stream: torch.cuda.Stream, touch: bool) -> torch.Tensor:
        with self._lock:
            N.check(N.lib.sf_cache_wait(self._h, lease._index, lease.slot_id, lease.generation,
                                        stream.cuda_stream, int(touch)), "expert lease")
            if self._observer is not None:
                self._observer.record(kind=RuntimeEventKind.CONSUME_WAIT, cache_id=self.cache_id,
                                      queue_id=self.queue_id, expert_id=lease.expert_id,
                                      slot_id=lease.slot_id, generation=lease.generation,
                                      ready_event=lease.ready_event, stream_ids=(int(stream.cuda_stream),))
            return self._storage[lease.slot_id]

    def _lease_release(self, lease: ExpertLease, streams: tuple) -> None:
        with self._lock:
            N.check(N.lib.sf_cache_check(self._h, lease._index, lease.slot_id, lease.generation),
                    "expert lease")
            if self._observer is not None:
                self._emit(RuntimeEventKind.RELEASE, lease.expert_id, lease.slot_id, lease.generation,
                           stream_ids=tuple(sorted(int(s.cuda_stream) for s in streams)))
            handles = (ctypes.c_uint64 * max(len(streams), 1))(*[s.cuda_stream for s in streams])
            N.check(N.lib.sf_cache_release(self._h, lease._index, lease.slot_id, lease.generation, handles,
                                           len(streams)), "expert lease")

    def _emit(self, kind, expert_id, slot_id: int, generation: int, *, submission_sequence=None,
              victim_expert_id=None, ready_event=None, stream_ids=()) -> None:
        self._observer.record(kind=kind, cache_id=self.cache_id, queue_id=self.queue_id,
                              expert_id=expert_id, slot_id=slot_id, generation=generation,
                              submission_sequence=submission_sequence, victim_expert_id=victim_expert_id,
                              ready_event=ready_event, stream_ids=stream_ids)

    # ------------------------------------------------------------- fast path
    def device_slot_table(self, keys) -> torch.Tensor | None:
        """int32 device tensor with the slot of each key, or ``None`` unless
        the cache holds every source, all resident, none in flight (so no
        slot can change while the table is used)."""
        with self._lock:
            self._check_open()
            if self._device_mode or self._n_slots < len(self._keys):
                return None
            table = (ctypes.c_int32 * len(self._keys))()
            complete = ctypes.c_int()
            N.check(N.lib.sf_cache_resident_table(self._h, table, ctypes.byref(complete)),
                    "sf_cache_resident_table")
            if not complete.value:
                return None
            keys = tuple(keys)
            version = self._state_version
            if self._table is not None and self._table[0] == version and self._table[1] == keys:
                return self._table[2]
            slots = torch.tensor([table[self._index[k]] if k in self._index else -1 for k in keys],
                                 dtype=torch.int32).to(self.device)
            self._table = (version, keys, slots)
            return slots

    def device_hit_counter(self) -> torch.Tensor:
        """The device int64 scalar kernels add resident hits to
        (``ops.moe_dispatch(..., active_total=)``); read on the host only
        when the statistics are read."""
        if self._device_hits is None:
            self._device_hits = torch.zeros((), dtype=torch.int64, device=self.device)
        return self._device_hits

    def note_device_hits(self, count: torch.Tensor) -> None:
        """Adds a device-side count of resident hits (no host sync)."""
        self.device_hit_counter().add_(count.reshape(()))

    def _flush_device_hits(self) -> None:
        if self._device_hits is not None:
            N.check(N.lib.sf_cache_add_hits(self._h, int(self._device_hits.item())), "sf_cache_add_hits")
            self._device_hits.zero_()

    def prefill_all(self) -> None:
        """Leases and releases every source once (fills the empty ones)."""
        self._check_host_managed()
        for key in self._keys:
            if key in self._resident or key in self._inflight:
                continue
            self.acquire(key).release()

    # --------------------------------------------------- device-managed mode
    @property
    def device_managed(self) -> bool:
        return self._device_mode

    @property
    def directory(self) -> DeviceExpertDirectory | None:
        """The HBM bookkeeping while device-managed, else ``None``."""
        return self._directory if self._device_mode else None

    def enter_device_mode(self) -> DeviceExpertDirectory:
        """Moves the bookkeeping to the device (synchronises the device; needs
        no active lease and every fill complete).  The sources must be
        page-locked and device-mapped."""
        with self._lock:
            self._check_open()
            if self._device_mode:
                return self._directory
            torch.cuda.synchronize(self.device)
            self._flush_device_hits()
            S, E = self._n_slots, len(self._keys)
            slot_expert, slot_gen = (ctypes.c_int32 * S)(), (ctypes.c_int32 * S)()
            slot_stamp, expert_slot = (ctypes.c_int64 * S)(), (ctypes.c_int32 * E)()
            clock, counters = ctypes.c_int64(), (ctypes.c_int64 * 4)()
            N.check(N.lib.sf_cache_export_slots(self._h, slot_expert, slot_gen, slot_stamp, expert_slot,
                                                ctypes.byref(clock), counters), "device-managed mode")
            if self._directory is None:
                self._directory = DeviceExpertDirectory(self)
            self._directory.load(dict(
                slot_expert=torch.tensor(list(slot_expert), dtype=torch.int32),
                slot_gen=torch.tensor(list(slot_gen), dtype=torch.int32),
                slot_stamp=torch.tensor(list(slot_stamp), dtype=torch.int64),
                expert_slot=torch.tensor(list(expert_slot), dtype=torch.int32),
                clock=clock.value, counters=torch.tensor(list(counters), dtype=torch.int64)))
            torch.cuda.synchronize(self.device)
            self._device_mode = True
            self._table = None
            return self._directory

    def _mirror_device_state(self) -> None:
        """Installs the device bookkeeping in the host manager (synchronises
        the device); the device copy stays authoritative while the mode lasts."""
        if not self._device_mode:
            return
        torch.cuda.synchronize(self.device)
        st = self._directory.read()
        if st["status"]:
            raise RuntimeError(f"device expert directory failed (status {st['status']})")
        S = self._n_slots
        se = (ctypes.c_int32 * S)(*st["slot_expert"].tolist())
        sg = (ctypes.c_int32 * S)(*st["slot_gen"].tolist())
        ss = (ctypes.c_int64 * S)(*st["slot_stamp"].tolist())
        cn = (ctypes.c_int64 * 4)(*st["counters"].tolist())
        N.check(N.lib.sf_cache_adopt_slots(self._h, se, sg, ss, st["clock"], cn), "device-managed mode")
        self._events.clear()

    def leave_device_mode(self) -> None:
        """Returns the bookkeeping to the host manager (synchronises the device)."""
        with self._lock:
            if not self._device_mode:
                return
            self._mirror_device_state()
            self._device_mode = False
            self._table = None

    # ------------------------------------------------------------ inspection
    def stats(self) -> ExpertCacheStats:
        with self._lock:
            self._mirror_device_state()
            self._flush_device_hits()
            c = _NativeState(self, 3).counters
            return ExpertCacheStats(int(c.h2d_submissions), int(c.resident_hits), int(c.inflight_joins),
                                    int(c.evictions), int(c.pending_use_guards))

    def resident_expert_ids(self) -> tuple:
        with self._lock:
            self._mirror_device_state()
            st = _NativeState(self, 1)
            return tuple(k for e, k in enumerate(self._keys) if st.where[e] == _RESIDENT)

    def snapshot(self) -> GpuExpertCacheSnapshot:
        with self._lock:
            self._mirror_device_state()
            self._flush_device_hits()
            st = _NativeState(self, 0)
            fills = self._native_fills()
            done = {int(f.submission): bool(f.done) for f in fills}
            slots = []
            guards_total = 0
            for s in range(self._n_slots):
                row = st.slots[s]
                e = int(row.expert)
                if e < 0:
                    ready = False
                elif st.where[e] == _INFLIGHT and st.home[e] == s:
                    ready = done.get(int(st.fill_seq[e]), True)
                else:
                    ready = st.where[e] == _RESIDENT and st.home[e] == s
                guards_total += int(row.guards_pending)
                slots.append(CacheSlotSnapshot(s, None if e < 0 else self._keys[e], int(row.generation),
                                               int(row.leases), int(row.stamp), bool(ready),
                                               int(row.guards_pending)))
            pending = tuple(PendingTransferSnapshot(self._keys[f.expert], int(f.slot), int(f.generation),
                                                    int(f.submission), self._events.get(int(f.ready_event)),
                                                    False) for f in fills if not f.done)
            c = st.counters
            stats = ExpertCacheStats(int(c.h2d_submissions), int(c.resident_hits), int(c.inflight_joins),
                                     int(c.evictions), guards_total)
            return GpuExpertCacheSnapshot(self.cache_id, self.queue_id, self._n_slots, int(c.state_version),
                                          int(c.sequence), int(c.submission_sequence), tuple(slots),
                                          pending, stats)

    # ------------------------------------------------------- reset / restore
    def _quiescent(self) -> bool:
        q = ctypes.c_int()
        N.check(N.lib.sf_cache_quiescent(self._h, ctypes.byref(q)), "sf_cache_quiescent")
        return bool(q.value)

    def cold_reset(self) -> None:
        with self._lock:
            self._check_host_managed()
            if self.active_lease_count:
                raise RuntimeError("cold reset cannot run while an active lease exists")
            if not self._quiescent():
                raise RuntimeError("cold reset requires explicit CUDA synchronization")
            if self._device_hits is not None:
                self._device_hits.zero_()
            N.check(N.lib.sf_cache_reset(self._h, N.SF_CACHE_RESET_COLD), "sf_cache_reset")
            self._events.clear()
            self._table = None

    def invalidate_contents(self) -> None:
        """Forgets every slot's expert (each slot's generation advances, its
        last use and guards are cleared) while keeping the counters and the
        slot memory: the next access of any expert is a miss.  This is the
        reference's "0 slots" intervention (``discard_completed_experts``,
        main_comparison_runtime.py:7-32) as one call; it needs the same
        quiescent boundary as a checkpoint."""
        with self._lock:
            self._require_checkpoint_boundary()
            N.check(N.lib.sf_cache_reset(self._h, N.SF_CACHE_RESET_DISCARD), "sf_cache_reset")
            self._events.clear()
            self._table = None

    def _require_checkpoint_boundary(self) -> None:
        self._check_host_managed()
        if self._observer is not None:
            raise RuntimeError("checkpoint restoration requires no active cache observer")
        if self.active_lease_count:
            raise RuntimeError("checkpoint boundary cannot contain active leases")
        if not self._quiescent():
            raise RuntimeError("checkpoint boundary requires explicit CUDA synchronization")

    def _capture_checkpoint(self) -> _Checkpoint:
        with self._lock:
            self._require_checkpoint_boundary()
            self._flush_device_hits()
            need = ctypes.c_size_t()
            N.check(N.lib.sf_cache_export(self._h, None, 0, ctypes.byref(need)), "sf_cache_export")
            image = (ctypes.c_uint8 * need.value)()
            N.check(N.lib.sf_cache_export(self._h, image, need.value, ctypes.byref(need)), "sf_cache_export")
            weights = torch.empty_like(self._storage, device="cpu", pin_memory=True)
            weights.copy_(self._storage.detach())
            return _Checkpoint(self, weights, bytes(image), dict(self._events), 0)

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
            buf = (ctypes.c_uint8 * len(checkpoint.image)).from_buffer_copy(checkpoint.image)
            N.check(N.lib.sf_cache_import(self._h, buf, len(checkpoint.image)), "sf_cache_import")
            self._events = dict(checkpoint.events)
            self._table = None
            finished = perf_counter_ns()
            return dict(weight_bytes=checkpoint.weights.numel() * checkpoint.weights.element_size(),
                        weights_pinned=checkpoint.weights.is_pinned(),
                        total_wall_ns=finished - started,
                        timings_ns=dict(boundary_check=checked - started, weight_copy_call=copied - checked,
                                        stream_synchronize=synced - copied, metadata_restore=finished - synced))

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            if self._device_mode:
                self.leave_device_mode()
            if not self._closing and self.active_lease_count:
                raise RuntimeError("expert cache cannot close while an active lease exists")
            self._closing = True
            torch.cuda.synchronize(self.device)
            N.lib.sf_cache_destroy(self._h)
            self._h = None
            self._events.clear()
            self._spare_events.clear()
            # Release the device memory now (slots, directory, tables).
            self._storage = self._storage.new_empty((0,) + tuple(self._storage.shape[1:]))
            self._directory = None
            self._device_hits = None
            self._sources.clear()
            owner, self._source_owner = self._source_owner, None
            if owner is not None:
                owner.close()
            self._table = None
            self._closed = True
            self._closing = False

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order varies
        h = getattr(self, "_h", None)
        if h and not getattr(self, "_closed", True):
            try:
                N.lib.sf_cache_destroy(h)
            except Exception:
                pass
