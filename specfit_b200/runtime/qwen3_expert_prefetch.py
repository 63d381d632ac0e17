"""Predicted cross-layer expert prefetch for one eager target forward.

Drop-in for ``Qwen3ExpertPrefetch`` (``src/specfit/runtime/
qwen3_expert_prefetch.py:34-418``): same constructor arguments, validation
messages, context protocol, and the same ``stats()`` / ``events()`` records,
which the reference's runner reads — so every scheduling decision (what is
leased, copied or computed, and when) is the reference's.

How it is organised here:

* ``_LayerPlan`` — one per decoder layer: the keys still to place, the
  leases held for the layer, its speculation cap and its statistics row;
* ``_CopyLedger`` — the scheduler's own fills still running (the
  ``max_inflight`` credits), with a memo of events known complete;
* ``Qwen3ExpertPrefetch`` itself walks a window of plans (the current layer plus ``lookahead_layers``) whenever the forward
  reaches an attention block or finishes an expert, and ``experts()`` hands
  the router's experts out one at a time: a completed fill first, else the
  oldest running one, else a credit is waited for or a blocking fill forced.

How a fill was granted comes from the lease itself (``lease.grant``: hit,
join of a running fill, or a new fill with its submission number), so no
cache state is re-read to classify it.  Eviction for speculation is LRU, or
with ``eviction_policy="probability"`` the lowest predicted probability
below the incoming expert's.
"""
from __future__ import annotations

import math
from collections import deque
from contextlib import ExitStack
from dataclasses import asdict, dataclass, field
from numbers import Real
from typing import Mapping, Sequence

import torch

from .. import _native as N
from .qwen3_offloaded_experts import Qwen3OffloadedExperts, ReductionMode
from .state import ExpertKey


@dataclass(slots=True)
class _LayerStats:
    layer_id: int
    predicted_experts: int
    actual_experts: int = 0
    ready_at_router: int = 0
    inflight_at_router: int = 0
    missing_at_router: int = 0
    prediction_copies: int = 0
    demand_copies: int = 0
    unused_prediction_copies: int = 0
    computed_experts: int = 0
    compute_waits: int = 0


@dataclass(slots=True)
class _LayerPlan:
    layer: int
    cache: object
    limit: int                       # speculative leases allowed before the router runs
    queue: deque                     # keys still to place, in placement order
    probabilities: dict | None
    row: _LayerStats
    held: dict = field(default_factory=dict)   # key -> (lease, rank, lease number)
    routed: bool = False             # the router has run: the queue is real demand
    guarded: bool = False            # predicted residents protected once
    speculated: set = field(default_factory=set)  # keys this plan copied on prediction


class _CopyLedger:
    """Fills the scheduler started (or found running) that are not known
    complete; their count is bounded by ``max_inflight``."""

    def __init__(self, limit: int) -> None:
        self.limit = limit
        self.running: list = []
        self.finished: set = set()
        self.peak = 0

    def done(self, event) -> bool:
        if event in self.finished:
            return True
        if event.query():
            self.finished.add(event)
            return True
        return False

    def sweep(self) -> None:
        self.running = [ev for ev in self.running if not self.done(ev)]

    def add(self, event) -> None:
        self.running.append(event)
        self.peak = max(self.peak, len(self.running))

    @property
    def full(self) -> bool:
        return len(self.running) >= self.limit


def _int_at_least(name: str, value, low: int) -> None:
    if type(value) is not int or value < low:
        raise ValueError(f"{name} must be an integer >= {low}")


def _layer_probabilities(layer: int, supplied, keys: dict) -> tuple:
    """(scores by expert id, probabilities by key) of one layer, validated."""
    if not isinstance(supplied, Mapping):
        raise TypeError("each probability layer must map expert IDs to probabilities")
    scores, by_key = {}, {}
    for e, p in supplied.items():
        if (type(e) is not int or e not in keys or type(p) is bool or not isinstance(p, Real)
                or not math.isfinite(p) or not 0 <= p <= 1):
            raise ValueError(f"invalid expert probability in layer {layer}")
        scores[e] = by_key[keys[e]] = float(p)
    return scores, by_key


class Qwen3ExpertPrefetch:
    """Scheduling for exactly one complete eager forward of ``loaded.model``.

    Enter and exit at a host-quiescent point with no outside leases; not
    reentrant, not reusable.  Streams, hooks and leases are restored on exit,
    including on exceptions."""

    def __init__(self, loaded, predictions: Mapping[int, Sequence[int]], *,
                 lookahead_layers: int = 1, max_inflight: int = 2,
                 max_prefetch_per_layer: int | None = None, trace: bool = False,
                 prediction_probabilities: Mapping[int, Mapping[int, float]] | None = None,
                 eviction_policy: str = "lru") -> None:
        _int_at_least("lookahead_layers", lookahead_layers, 0)
        _int_at_least("max_inflight", max_inflight, 1)
        if max_prefetch_per_layer is not None and (type(max_prefetch_per_layer) is not int
                                                   or max_prefetch_per_layer < 0):
            raise ValueError("max_prefetch_per_layer must be a non-negative integer or None")
        if type(trace) is not bool:
            raise ValueError("trace must be a boolean")
        if not isinstance(predictions, Mapping):
            raise TypeError("predictions must map layer IDs to expert IDs")
        if eviction_policy not in ("lru", "probability"):
            raise ValueError("eviction_policy must be 'lru' or 'probability'")
        if prediction_probabilities is None and eviction_policy != "lru":
            raise ValueError("probability eviction requires prediction_probabilities")
        if prediction_probabilities is not None and not isinstance(prediction_probabilities, Mapping):
            raise TypeError("prediction_probabilities must map layers to expert probabilities")
        layers = tuple(loaded.model.model.layers)
        caches = tuple(loaded.expert_caches)
        if not layers or len(layers) != len(caches):
            raise ValueError("decoder layers and expert caches must match")
        for mapping, what in ((predictions, "prediction"), (prediction_probabilities or {}, "probability")):
            if any(type(l) is not int or not 0 <= l < len(layers) for l in mapping):
                raise ValueError(f"{what} layer is outside the loaded model")

        self._plans = []
        for layer, cache in enumerate(caches):
            cap = cache.slot_count - 1  # one slot stays free for the real demand
            if max_prefetch_per_layer is not None:
                cap = min(cap, max_prefetch_per_layer)
            ids = tuple(predictions.get(layer, ()))
            keys = {}
            if ids or prediction_probabilities is not None:
                keys = {k.expert_id: k for k in cache.source_keys()
                        if type(k) is ExpertKey and k.layer_id == layer}
            if any(type(e) is not int or e not in keys for e in ids):
                raise ValueError(f"invalid predicted expert in layer {layer}")
            by_key = None
            if prediction_probabilities is None:
                order = sorted(set(ids))
            else:
                scores, by_key = _layer_probabilities(layer, prediction_probabilities.get(layer, {}), keys)
                if any(e not in scores for e in ids):
                    raise ValueError("every predicted expert needs an explicit probability")
                order = sorted((e for e in set(ids) if scores[e] > 0), key=lambda e: (-scores[e], e))[:cap]
            self._plans.append(_LayerPlan(layer, cache, cap, deque(keys[e] for e in order), by_key,
                                          _LayerStats(layer, len(order))))
        if len({c.device for c in caches}) != 1:
            raise ValueError("prefetch requires all layers on one GPU")

        self._layers = layers
        self._caches = caches
        self.predictions = tuple(tuple(k.expert_id for k in p.queue) for p in self._plans)
        self.lookahead_layers = lookahead_layers
        self.max_inflight = max_inflight
        self.eviction_policy = eviction_policy
        self._trace = trace
        self._log: list = []
        self._stack = ExitStack()
        self._ledger = _CopyLedger(max_inflight)
        self._copies_started = 0          # order of the scheduler's own fills
        self._leases_taken = 0            # order of every lease the scheduler took
        self._speculative = 0             # leases held for layers whose router has not run
        self._peak_speculative = 0
        self._credit_waits = 0
        self._forced_fills = 0
        self._cursor = 0                  # layer whose attention opens next
        self._open = None                 # layer between attention and its last expert
        self._at = 0                      # layer of the latest attention (record field)
        self._state = "new"               # new -> active -> closed

    # ------------------------------------------------------------- context
    def __enter__(self):
        if self._state != "new":
            raise RuntimeError("a prefetch context cannot be reused")
        modules = tuple(layer.mlp.experts for layer in self._layers)
        for lid, (m, cache) in enumerate(zip(modules, self._caches, strict=True)):
            if not isinstance(m, Qwen3OffloadedExperts) or m.cache is not cache or m.layer_id != lid:
                raise RuntimeError("every decoder layer must contain its offloaded expert cache")
        if any(m.reduction_mode is not ReductionMode.CANONICAL for m in modules):
            raise ValueError("predicted prefetch requires canonical reduction")
        if any(m._prediction_scheduler is not None for m in modules):
            raise RuntimeError("another predicted prefetch context is active")
        if any(c.closed or c.active_lease_count for c in self._caches):
            raise RuntimeError("prefetch requires open caches without active leases")
        self._state = "active"
        try:
            shared = torch.cuda.Stream(device=self._caches[0].device)
            for cache in self._caches:
                own = cache.copy_stream
                shared.wait_stream(own)
                # Fills already queued count against the credits until done.
                for t in cache._outstanding_transfers:
                    if not t.ready_event.query():
                        self._ledger.running.append(t.ready_event)
                cache.copy_stream = shared
                self._stack.callback(self._give_back_stream, cache, own, shared)
            for lid, (layer, m) in enumerate(zip(self._layers, modules, strict=True)):
                m._prediction_scheduler = self
                self._stack.callback(setattr, m, "_prediction_scheduler", None)
                hook = layer.self_attn.register_forward_pre_hook(lambda mod, args, l=lid: self._attention(l))
                self._stack.callback(hook.remove)
            self._note("prediction_available")
            self._advance()
            return self
        except BaseException:
            self._release_all()
            self._stack.close()
            raise

    @staticmethod
    def _give_back_stream(cache, own, shared) -> None:
        own.wait_stream(shared)
        cache.copy_stream = own

    def __exit__(self, exc_type, exc, tb) -> None:
        try:
            self._release_all()
        finally:
            self._stack.close()
        finished = self._cursor == len(self._layers)
        self._state = "complete" if exc_type is None and finished else "closed"
        if exc_type is None and not finished:
            raise RuntimeError("prefetch context requires exactly one complete target forward")

    def _release_all(self) -> None:
        """Releases every lease still held, oldest lease first."""
        held = sorted(((entry[2], plan, key) for plan in self._plans for key, entry in plan.held.items()),
                      key=lambda t: t[0])
        for _, plan, key in held:
            self._unhold(plan, key).release()

    # ------------------------------------------------------------- records
    def _note(self, action, *, layer=None, expert=None, **values) -> None:
        if self._trace:
            self._log.append(dict(sequence=len(self._log), action=action, current_layer=self._at,
                                  layer_id=layer, expert_id=expert, **values))

    def _attention(self, layer: int) -> None:
        if self._state != "active" or self._open is not None or layer != self._cursor:
            raise RuntimeError("predicted prefetch requires one ordered eager layer traversal")
        self._at = self._open = layer
        self._note("attention", layer=layer)
        self._advance()

    # -------------------------------------------------------------- leases
    def _unhold(self, plan: _LayerPlan, key):
        lease = plan.held.pop(key)[0]
        if not plan.routed:
            self._speculative -= 1
        return lease

    def _lease(self, plan: _LayerPlan, key, how: str) -> bool:
        """Lease ``key`` for ``plan``: ``how`` is "resident" (hits and joins
        only), "predict" / "demand" (a fill only into a slot nobody is still
        reading, and only with a free credit checked by the caller), or
        "force" (a blocking fill that may queue behind a slot's readers)."""
        cache = plan.cache
        if how == "force":
            lease = cache._prefetch(key)
        elif how == "predict" and self.eviction_policy == "probability":
            lease = cache._prefetch_nonblocking(key, eviction_probabilities=plan.probabilities)
        else:
            lease = cache._prefetch_nonblocking(key, resident_only=how == "resident")
        if lease is None:
            return False
        kind, submission = lease.grant
        if kind == N.SF_GRANT_HIT:
            self._ledger.finished.add(lease.ready_event)  # published only after its fill completed
        if kind == N.SF_GRANT_MISS:
            rank = (0, self._copies_started)
            self._copies_started += 1
            self._ledger.add(lease.ready_event)
            if how == "predict":
                plan.speculated.add(key)
                plan.row.prediction_copies += 1
            else:
                plan.row.demand_copies += 1
            self._note("copy", layer=plan.layer, expert=key.expert_id, prediction=how == "predict",
                       slot_wait=how == "force")
        else:
            rank = (-1, submission if kind == N.SF_GRANT_JOIN else -1)
        plan.held[key] = (lease, rank, self._leases_taken)
        self._leases_taken += 1
        if not plan.routed:
            self._speculative += 1
            self._peak_speculative = max(self._peak_speculative, self._speculative)
        return True

    # ---------------------------------------------------------- placement
    def _window(self):
        stop = min(len(self._plans), self._at + self.lookahead_layers + 1)
        return self._plans[self._at:stop]

    def _guard_residents(self, plan: _LayerPlan) -> None:
        """Before any miss of a not-yet-routed layer, lease its predicted
        experts that are already resident or in flight (once per layer), so
        an earlier miss cannot evict them."""
        plan.guarded = True
        if not plan.cache.holds_any():
            return
        for key in plan.queue:
            if len(plan.held) >= plan.limit:
                return
            if key not in plan.held:
                self._lease(plan, key, "resident")

    def _place(self, plan: _LayerPlan) -> bool:
        """Leases the plan's queued keys in order; False when the walk must
        stop here (speculation cap, no credit, or no writable slot)."""
        q = plan.queue
        while q:
            key = q[0]
            if key in plan.held:
                q.popleft()
            elif not plan.routed and len(plan.held) >= plan.limit:
                return False
            elif self._lease(plan, key, "resident"):
                q.popleft()
            elif self._ledger.full or not self._lease(plan, key, "demand" if plan.routed else "predict"):
                return False
            else:
                q.popleft()
        return True

    def _advance(self) -> None:
        self._ledger.sweep()
        for plan in self._window():
            if not plan.routed and not plan.guarded:
                self._guard_residents(plan)
            if not self._place(plan):
                return  # a farther layer waits until this one is placed

    # ------------------------------------------------------------ schedule
    def _next_expert(self, plan: _LayerPlan, todo: dict):
        """(key, waited) of the expert to run next, or None when none of the
        remaining experts is leased."""
        oldest = None
        for key in todo:
            held = plan.held.get(key)
            if held is None:
                continue
            if self._ledger.done(held[0].ready_event):
                return key, False
            if oldest is None or held[1] < plan.held[oldest][1]:
                oldest = key
        return None if oldest is None else (oldest, True)

    def experts(self, layer: int, active_experts: tuple):
        """Yield ``(expert_id, lease)`` for every actual expert of ``layer``
        once, completed transfers first."""
        plan = self._plans[layer] if 0 <= layer < len(self._plans) else None
        if self._state != "active" or self._open != layer or plan is None or plan.routed:
            raise RuntimeError("expert scheduling must follow this layer's Attention exactly once")
        routed = set(active_experts)
        self._speculative -= len(plan.held)
        plan.routed = True
        row = plan.row
        row.actual_experts = len(routed)
        self._note("router", layer=layer, experts=list(active_experts))
        todo = dict.fromkeys(ExpertKey(layer, e) for e in sorted(routed))
        for key in [k for k in plan.held if k.expert_id not in routed]:  # wrong predictions
            self._unhold(plan, key).release()
        row.unused_prediction_copies = sum(k.expert_id not in routed for k in plan.speculated)
        for key in todo:
            if key not in plan.held:
                self._lease(plan, key, "resident")
            held = plan.held.get(key)
            if held is None:
                row.missing_at_router += 1
            elif self._ledger.done(held[0].ready_event):
                row.ready_at_router += 1
            else:
                row.inflight_at_router += 1
        plan.queue = deque(k for k in todo if k not in plan.held)
        while todo:
            self._advance()
            pick = self._next_expert(plan, todo)
            if pick is None:
                self._ledger.sweep()
                if self._ledger.full:
                    # Only other layers' fills are running: wait for a credit.
                    self._credit_waits += 1
                    self._ledger.running[0].synchronize()
                else:
                    # Every writable slot may still be read by queued kernels;
                    # only real demand may queue a fill behind them.
                    self._lease(plan, next(iter(todo)), "force")
                    self._forced_fills += 1
                continue
            key, waited = pick
            if waited:
                row.compute_waits += 1
            lease = self._unhold(plan, key)
            del todo[key]
            self._note("compute", layer=layer, expert=key.expert_id, waited=waited)
            try:
                yield key.expert_id, lease
                row.computed_experts += 1
            finally:
                lease.release()
        self._advance()
        self._open = None
        self._cursor = layer + 1
        self._note("layer_complete", layer=layer)

    # ------------------------------------------------------------- records
    def stats(self) -> dict:
        """Host-side statistics (no GPU synchronisation)."""
        return dict(complete=self._state == "complete", lookahead_layers=self.lookahead_layers,
                    max_inflight=self.max_inflight, prefetch_slot_limits=[p.limit for p in self._plans],
                    peak_inflight=self._ledger.peak, peak_speculative_leases=self._peak_speculative,
                    queue_capacity_waits=self._credit_waits, slot_wait_copies=self._forced_fills,
                    layers=[asdict(p.row) for p in self._plans])

    def events(self) -> tuple:
        return tuple(dict(row) for row in self._log)
