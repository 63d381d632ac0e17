"""Expert leases: a caller's claim on one generation of one cache slot.

Interface of ``src/specfit/runtime/lease.py``: ``NoEvictableSlotError``
(:13), ``ExpertCacheStats`` (:18-23) and ``ExpertLease`` (:26-105) with
``wait(stream=None) -> Tensor``, ``release()``, the context-manager protocol,
``expert_id``, ``generation``, ``slot_id`` and ``ready_event``.

A lease here is a handle: its identity is (expert index, slot, generation),
and every operation is one call into the native slot manager that checks
that identity first (a lease whose slot was refilled is refused with the
reference's error).  ``wait`` orders the stream behind the slot's fill
unless the fill is already published, and applies a deferred LRU touch;
``release`` hands the manager the streams the lease was used on, which
become the slot's use guards.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, Hashable

import torch

if TYPE_CHECKING:  # pragma: no cover
    from .gpu_expert_cache import GpuExpertCache


class NoEvictableSlotError(RuntimeError):
    """Every slot of the cache is held by an active lease."""


@dataclass(frozen=True, slots=True)
class ExpertCacheStats:
    h2d_submissions: int
    resident_hits: int
    inflight_joins: int
    evictions: int
    pending_use_guards: int


class ExpertLease:
    __slots__ = ("_cache", "_key", "_index", "slot_id", "_generation", "ready_event", "_used",
                 "_touch_due", "_done", "grant")

    def __init__(self, cache: "GpuExpertCache", key: Hashable, index: int, slot_id: int, generation: int,
                 ready_event, *, defer_touch: bool = False, grant: tuple = (0, -1)) -> None:
        self._cache = cache
        self._key = key
        self._index = index
        self.slot_id = slot_id
        self._generation = generation
        self.ready_event = ready_event
        self._used: dict = {}          # cuda_stream handle -> stream the slot was read on
        self._touch_due = defer_touch  # a prefetched lease counts as a use at its first wait
        self._done = False
        # How the cache granted it: (SF_GRANT_HIT / _JOIN / _MISS, submission
        # number of the fill it joined or started, else -1).
        self.grant = grant

    @property
    def expert_id(self) -> Hashable:
        return self._key

    @property
    def generation(self) -> int:
        return self._generation

    def wait(self, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        if self._done:
            raise RuntimeError("cannot wait on a released expert lease")
        s = stream if stream is not None else torch.cuda.current_stream(self._cache.device)
        view = self._cache._lease_wait(self, s, self._touch_due)
        self._touch_due = False
        self._used.setdefault(s.cuda_stream, s)
        return view

    def release(self) -> None:
        if not self._done:
            self._cache._lease_release(self, tuple(self._used.values()))
            self._done = True

    def __enter__(self) -> "ExpertLease":
        if self._done:
            raise RuntimeError("cannot re-enter a released expert lease")
        return self

    def __exit__(self, exc_type, exc, tb) -> None:
        self.release()
