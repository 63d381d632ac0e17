"""Cache-transition observers.

The observer protocol of ``src/specfit/runtime/cache_observer.py``: the cache
calls ``record(kind=..., cache_id=..., ...)`` at every resident hit, in-flight
join, eviction, H2D submission, consumer wait and release, in host order.
``RecordingCacheTransitionObserver`` keeps them in memory for tests.
"""
from __future__ import annotations

from dataclasses import dataclass
from threading import Lock
from time import perf_counter_ns
from typing import Any, Hashable, Protocol

from .state import RuntimeEventKind


class CacheTransitionObserver(Protocol):
    def record(self, *, kind: RuntimeEventKind, cache_id: str, queue_id: str, expert_id: Hashable,
               slot_id: int, generation: int, submission_sequence: int | None = None,
               victim_expert_id: Hashable | None = None, ready_event: Any = None,
               stream_ids: tuple = ()) -> None: ...


@dataclass(frozen=True, slots=True)
class CacheTransition:
    run_id: str
    sequence: int
    host_time_ns: int
    kind: RuntimeEventKind
    cache_id: str
    queue_id: str
    expert_id: Hashable
    slot_id: int
    generation: int
    submission_sequence: int | None = None
    victim_expert_id: Hashable | None = None
    ready_event: Any = None
    stream_ids: tuple = ()


class RecordingCacheTransitionObserver:
    def __init__(self, run_id: str = "specfit-b200") -> None:
        if not run_id:
            raise ValueError("run_id must be non-empty")
        self.run_id = run_id
        self._events: list = []
        self._lock = Lock()

    def record(self, *, kind, cache_id, queue_id, expert_id, slot_id, generation,
               submission_sequence=None, victim_expert_id=None, ready_event=None,
               stream_ids=()) -> None:
        with self._lock:
            self._events.append(CacheTransition(
                run_id=self.run_id, sequence=len(self._events), host_time_ns=perf_counter_ns(),
                kind=RuntimeEventKind(kind), cache_id=cache_id, queue_id=queue_id,
                expert_id=expert_id, slot_id=slot_id, generation=generation,
                submission_sequence=submission_sequence, victim_expert_id=victim_expert_id,
                ready_event=ready_event, stream_ids=tuple(stream_ids)))

    def events(self) -> tuple:
        with self._lock:
            return tuple(self._events)

    def reset(self) -> None:
        with self._lock:
            self._events.clear()
