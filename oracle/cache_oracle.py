"""CPU oracle of the expert cache's slot state (test infrastructure only).

Restates the reference's logical LRU replay, ``_LayerState.access`` and
``_choose_lru_slot`` (src/specfit/replay.py:156-285), which re-derives a
cache layer's state from the sequence of expert accesses: a resident expert
is a hit; a miss takes the replaceable slot that is empty first, else least
recently used, ties by lower slot id (``replay.py:214-227``), evicting its
expert and counting one H2D submission; every access leases and releases
the slot, touching its LRU stamp twice (``replay.py:229-272``).

Used by the tests and by ``bench.py --mode sweep`` to predict the misses of
configuration 3's slot sweep from the routes alone.  Parity of this
restatement: it follows the reference function line by line; the GPU cache
(``GpuExpertCache``) is checked against it on the same access sequences.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class LruLayer:
    capacity: int
    expert: list = field(default_factory=list)     # slot -> expert id or None
    last_used: list = field(default_factory=list)  # slot -> LRU stamp
    sequence: int = 0
    h2d_submissions: int = 0
    resident_hits: int = 0
    evictions: int = 0

    def __post_init__(self) -> None:
        if self.capacity <= 0:
            raise ValueError("capacity must be positive")
        self.expert = [None] * self.capacity
        self.last_used = [0] * self.capacity

    def _touch(self, slot: int) -> None:
        self.sequence += 1
        self.last_used[slot] = self.sequence

    def access(self, expert_id: int) -> bool:
        """One acquire + release; returns True on a miss (an H2D fill)."""
        try:
            slot = self.expert.index(expert_id)
            self.resident_hits += 1
            miss = False
        except ValueError:
            slot = min(range(self.capacity),
                       key=lambda s: (self.expert[s] is not None, self.last_used[s], s))
            if self.expert[slot] is not None:
                self.evictions += 1
            self.expert[slot] = expert_id
            self.h2d_submissions += 1
            miss = True
        self._touch(slot)  # lease
        self._touch(slot)  # release
        return miss

    def resident(self) -> tuple:
        """Resident experts in slot order."""
        return tuple(e for e in self.expert if e is not None)


def pass_accesses(routes, order: str = "expert_id_ascending", resident=()) -> list:
    """The experts one layer's forward acquires for one pass: the distinct
    experts of ``routes`` (any iterable of expert ids) in execution order --
    ascending id, or (``resident_first``) the residents first, each group
    ascending (``qwen3_offloaded_experts.py:262-292``)."""
    active = sorted({int(e) for e in routes})
    if order == "expert_id_ascending":
        return active
    if order == "resident_first":
        res = set(resident)
        return [e for e in active if e in res] + [e for e in active if e not in res]
    raise ValueError(f"unknown execution order {order!r}")


def replay_passes(capacity: int, layer_routes: list, passes: int) -> list:
    """Misses per pass of ``passes`` identical forwards over layers whose
    routes are ``layer_routes[l]``, starting from empty caches."""
    layers = [LruLayer(capacity) for _ in layer_routes]
    out = []
    for _ in range(passes):
        misses = 0
        for lay, routes in zip(layers, layer_routes):
            for e in pass_accesses(routes):
                misses += lay.access(e)
        out.append(misses)
    return out
