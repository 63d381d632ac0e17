"""Keys and event kinds shared by the expert cache and its observers.

``ExpertKey`` mirrors ``specfit.state.ExpertKey`` (``src/specfit/state.py:8-15``)
and ``RuntimeEventKind`` the cache-transition kinds of
``src/specfit/trace.py:900-906``; the values are the same strings so traces
from either implementation compare equal.
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum


@dataclass(frozen=True, slots=True, order=True)
class ExpertKey:
    layer_id: int
    expert_id: int

    def __post_init__(self) -> None:
        if self.layer_id < 0 or self.expert_id < 0:
            raise ValueError("layer_id and expert_id must be non-negative")


class RuntimeEventKind(str, Enum):
    RESIDENT_HIT = "resident_hit"
    INFLIGHT_JOIN = "inflight_join"
    H2D_SUBMIT = "h2d_submit"
    EVICT = "evict"
    CONSUME_WAIT = "consume_wait"
    RELEASE = "release"
