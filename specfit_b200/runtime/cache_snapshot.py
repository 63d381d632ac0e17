"""Immutable views of an expert cache's state.

Field-for-field the snapshot types of ``src/specfit/runtime/cache_snapshot.py``
(``CacheSlotSnapshot``, ``PendingTransferSnapshot``,
``GpuExpertCacheSnapshot``) so tooling written against the reference reads
them unchanged.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Hashable

from .lease import ExpertCacheStats


def _nonneg(**values: int) -> None:
    for name, value in values.items():
        if isinstance(value, bool) or not isinstance(value, int):
            raise TypeError(f"{name} must be an integer")
        if value < 0:
            raise ValueError(f"{name} must be non-negative")


@dataclass(frozen=True, slots=True)
class CacheSlotSnapshot:
    slot_id: int
    expert_id: Hashable | None
    generation: int
    active_leases: int
    last_used_sequence: int
    ready: bool
    pending_use_guards: int

    def __post_init__(self) -> None:
        _nonneg(slot_id=self.slot_id, generation=self.generation, active_leases=self.active_leases,
                last_used_sequence=self.last_used_sequence,
                pending_use_guards=self.pending_use_guards)
        if not isinstance(self.ready, bool):
            raise TypeError("ready must be a boolean")
        if self.expert_id is None and (self.ready or self.active_leases or self.pending_use_guards):
            raise ValueError("an empty slot cannot be ready or in use")


@dataclass(frozen=True, slots=True)
class PendingTransferSnapshot:
    expert_id: Hashable
    slot_id: int
    generation: int
    submission_sequence: int
    ready_event: Any
    ready_event_completed: bool

    def __post_init__(self) -> None:
        _nonneg(slot_id=self.slot_id, generation=self.generation,
                submission_sequence=self.submission_sequence)
        if not isinstance(self.ready_event_completed, bool):
            raise TypeError("ready_event_completed must be a boolean")


@dataclass(frozen=True, slots=True)
class GpuExpertCacheSnapshot:
    cache_id: str
    queue_id: str
    capacity: int
    host_state_version: int
    lru_sequence: int
    submission_sequence: int
    slots: tuple
    pending_transfers: tuple
    stats: ExpertCacheStats

    def __post_init__(self) -> None:
        if not self.cache_id or not self.queue_id:
            raise ValueError("cache_id and queue_id must be non-empty")
        _nonneg(capacity=self.capacity, host_state_version=self.host_state_version,
                lru_sequence=self.lru_sequence, submission_sequence=self.submission_sequence)
        if len(self.slots) != self.capacity:
            raise ValueError("snapshot must describe every slot")
