"""Expert leases: a caller's claim on one cache slot generation.

Mirrors ``src/specfit/runtime/lease.py``: ``NoEvictableSlotError`` (:13),
``ExpertCacheStats`` (:18-23) and ``ExpertLease`` (:26-105).  A lease pins
its slot against eviction until released; ``wait(stream)`` orders ``stream``
after the slot's fill and returns the slot tensor; ``release()`` records, on
every stream that waited, the event a later refill of the slot must wait for.
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
    __slots__ = ("_cache", "_expert_id", "_generation", "_released", "_streams", "_touch_pending",
                 "_ready_confirmed", "ready_event", "slot_id")

    def __init__(self, cache: "GpuExpertCache", expert_id: Hashable, slot_id: int, generation: int,
                 ready_event, *, _defer_touch: bool = False) -> None:
        self._cache = cache
        self._expert_id = expert_id
        self._generation = generation
        self._released = False
        self._streams: dict = {}
        self._touch_pending = _defer_touch
        # Set by the cache when the slot's fill is already known complete, so
        # a consumer need not wait on its event.
        self._ready_confirmed = False
        self.slot_id = slot_id
        self.ready_event = ready_event

    @property
    def expert_id(self) -> Hashable:
        return self._expert_id

    @property
    def generation(self) -> int:
        return self._generation

    def wait(self, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        if self._released:
            raise RuntimeError("cannot wait on a released expert lease")
        if stream is None:
            stream = torch.cuda.current_stream(self._cache.device)
        if not self._ready_confirmed and self.ready_event is not None:
            stream.wait_event(self.ready_event)
        self._streams[stream.cuda_stream] = stream
        tensor = self._cache._lease_tensor(self._expert_id, self.slot_id, self._generation,
                                           touch=self._touch_pending)
        self._touch_pending = False
        if self._cache._observer is not None:
            self._cache._record_consume_wait(expert_id=self._expert_id, slot_id=self.slot_id,
                                             generation=self._generation,
                                             ready_event=self.ready_event, stream=stream)
        return tensor

    def release(self) -> None:
        if self._released:
            return
        self._cache._release(self._expert_id, self.slot_id, self._generation,
                             tuple(self._streams.values()))
        self._released = True

    def __enter__(self) -> "ExpertLease":
        if self._released:
            raise RuntimeError("cannot re-enter a released expert lease")
        return self

    def __exit__(self, exc_type, exc, tb) -> None:
        self.release()
