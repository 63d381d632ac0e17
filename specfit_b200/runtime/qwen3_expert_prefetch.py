"""Predicted cross-layer expert prefetch for one eager target forward.

Drop-in for ``Qwen3ExpertPrefetch`` (``src/specfit/runtime/
qwen3_expert_prefetch.py:34-418``): same constructor arguments, validation
and messages, context protocol, ``stats()`` / ``events()`` records.

What it schedules.  Before the forward, each layer has a list of predicted
experts.  All caches share one copy stream for the duration of the context.
Whenever the forward reaches a layer's attention (a forward pre-hook) and
whenever an expert of the current layer has been computed, ``_pump`` walks
the layers from the current one up to ``lookahead_layers`` ahead and, for
each, leases its requested experts in order:

* an expert already resident or in flight is held at no cost;
* otherwise a copy is submitted if fewer than ``max_inflight`` scheduler
  copies are still running, into a slot whose previous readers are done
  (speculation never queues behind a busy slot);
* speculative leases of a layer are capped at ``slots - 1`` (or
  ``max_prefetch_per_layer``), leaving one slot for the real demand.

When the router has run, ``experts(layer, active)`` replaces the layer's
prediction queue with the real demand, drops wrong predictions, and yields
each real expert once: a ready one if any, else the oldest in flight (a
compute wait), else — when nothing the layer needs is in flight — it frees a
queue credit or forces a blocking fill.  The caller computes the yielded
expert while later copies continue, and reduces all contributions in
canonical order, so the result is bit-identical to the plain forward.

Eviction for speculation is LRU, or with ``eviction_policy="probability"``
the lowest predicted probability below the incoming expert's
(``GpuExpertCache._choose_probability_slot``).
"""
from __future__ import annotations

import math
from collections import deque
from contextlib import ExitStack
from dataclasses import asdict, dataclass
from numbers import Real
from typing import Mapping, Sequence

import torch

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


def _check_count(name: str, value, minimum: int) -> None:
    if type(value) is not int or value < minimum:
        raise ValueError(f"{name} must be an integer >= {minimum}")


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
        _check_count("lookahead_layers", lookahead_layers, 0)
        _check_count("max_inflight", max_inflight, 1)
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
        n = len(layers)
        for mapping, what in ((predictions, "prediction"), (prediction_probabilities or {}, "probability")):
            if any(type(l) is not int or not 0 <= l < n for l in mapping):
                raise ValueError(f"{what} layer is outside the loaded model")

        slots = [len(c._slots) - 1 for c in caches]
        self._limits = tuple(s if max_prefetch_per_layer is None else min(s, max_prefetch_per_layer)
                             for s in slots)
        self._probabilities: list = []
        self._requests: list = []
        ordered = []
        for layer, cache in enumerate(caches):
            ids = tuple(predictions.get(layer, ()))
            need_keys = bool(ids) or prediction_probabilities is not None
            keys = ({k.expert_id: k for k in cache._sources
                     if type(k) is ExpertKey and k.layer_id == layer} if need_keys else {})
            if any(type(e) is not int or e not in keys for e in ids):
                raise ValueError(f"invalid predicted expert in layer {layer}")
            probs = None
            if prediction_probabilities is not None:
                supplied = prediction_probabilities.get(layer, {})
                if not isinstance(supplied, Mapping):
                    raise TypeError("each probability layer must map expert IDs to probabilities")
                score: dict = {}
                probs = {}
                for e, p in supplied.items():
                    if (type(e) is not int or e not in keys or type(p) is bool
                            or not isinstance(p, Real) or not math.isfinite(p) or not 0 <= p <= 1):
                        raise ValueError(f"invalid expert probability in layer {layer}")
                    score[e] = float(p)
                    probs[keys[e]] = score[e]
                if any(e not in score for e in ids):
                    raise ValueError("every predicted expert needs an explicit probability")
                ids = tuple(sorted((e for e in set(ids) if score[e] > 0),
                                   key=lambda e: (-score[e], e)))[: self._limits[layer]]
            else:
                ids = tuple(sorted(set(ids)))
            self._probabilities.append(probs)
            ordered.append(ids)
            self._requests.append(deque(keys[e] for e in ids))
        if len({c.device for c in caches}) != 1:
            raise ValueError("prefetch requires all layers on one GPU")

        self._loaded = loaded
        self._layers = layers
        self._caches = caches
        self.predictions = tuple(ordered)
        self.lookahead_layers = lookahead_layers
        self.max_inflight = max_inflight
        self.eviction_policy = eviction_policy
        self._trace = trace
        self._events: list = []
        self._stack = ExitStack()
        self._leases: dict = {}           # ExpertKey -> lease held by the scheduler
        self._held = [0] * n              # leases held per layer
        self._speculative = 0             # leases of layers whose router has not run
        self._rank: dict = {}             # ExpertKey -> (0, copy order) or (-1, joined submission)
        self._pending: list = []          # scheduler copy events not known complete
        self._done_events: set = set()
        self._prediction_copies: set = set()
        self._residents_protected: set = set()
        self._actual: dict = {}
        self._layer_stats = [_LayerStats(i, len(ids)) for i, ids in enumerate(ordered)]
        self._copy_order = 0
        self._next_layer = 0
        self._open_layer = None
        self._current_layer = 0
        self._entered = self._used = self._complete = False
        self._peak_inflight = self._peak_speculative = 0
        self._queue_capacity_waits = self._slot_wait_copies = 0

    # ------------------------------------------------------------ context
    def __enter__(self):
        if self._used:
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
        self._used = True
        try:
            self._copy_stream = torch.cuda.Stream(device=self._caches[0].device)
            for cache in self._caches:
                previous = cache.copy_stream
                self._copy_stream.wait_stream(previous)
                # Copies already queued count against the credits until done.
                self._pending.extend(t.ready_event for t in cache._outstanding_transfers
                                     if not t.ready_event.query())
                cache.copy_stream = self._copy_stream
                self._stack.callback(self._restore_stream, cache, previous)
            for lid, (layer, m) in enumerate(zip(self._layers, modules, strict=True)):
                m._prediction_scheduler = self
                self._stack.callback(setattr, m, "_prediction_scheduler", None)
                handle = layer.self_attn.register_forward_pre_hook(self._attention_hook(lid))
                self._stack.callback(handle.remove)
            self._entered = True
            self._record("prediction_available")
            self._pump()
            return self
        except BaseException:
            for key in tuple(self._leases):
                self._drop(key).release()
            self._entered = False
            self._stack.close()
            raise

    def _restore_stream(self, cache, previous) -> None:
        previous.wait_stream(self._copy_stream)
        cache.copy_stream = previous

    def __exit__(self, exc_type, exc, tb) -> None:
        try:
            for key in tuple(self._leases):
                self._drop(key).release()
        finally:
            self._entered = False
            self._stack.close()
        self._complete = exc_type is None and self._next_layer == len(self._layers)
        if exc_type is None and not self._complete:
            raise RuntimeError("prefetch context requires exactly one complete target forward")

    # ------------------------------------------------------------ helpers
    def _record(self, action, *, layer=None, expert=None, **values) -> None:
        if self._trace:
            self._events.append(dict(sequence=len(self._events), action=action,
                                     current_layer=self._current_layer, layer_id=layer,
                                     expert_id=expert, **values))

    def _attention_hook(self, layer: int):
        def hook(module, inputs):
            self._begin_layer(layer)
        return hook

    def _begin_layer(self, layer: int) -> None:
        if not self._entered or self._open_layer is not None or layer != self._next_layer:
            raise RuntimeError("predicted prefetch requires one ordered eager layer traversal")
        self._current_layer = self._open_layer = layer
        self._record("attention", layer=layer)
        self._pump()

    def _ready(self, event) -> bool:
        if event in self._done_events:
            return True
        if event.query():
            self._done_events.add(event)
            return True
        return False

    def _reap(self) -> None:
        self._pending = [ev for ev in self._pending if not self._ready(ev)]

    def _drop(self, key):
        lease = self._leases.pop(key)
        self._rank.pop(key, None)
        self._held[key.layer_id] -= 1
        if key.layer_id not in self._actual:
            self._speculative -= 1
        return lease

    def _hold(self, key, *, resident_only=False, force=False, prediction=False) -> bool:
        """Lease ``key`` (blocking fill when ``force``); False if it would need
        a copy that is not allowed now."""
        cache = self._caches[key.layer_id]
        submitted_before = cache._submission_sequence
        if force:
            lease = cache._prefetch(key)
        elif prediction and self.eviction_policy == "probability":
            lease = cache._prefetch_nonblocking(key, resident_only=resident_only,
                                                eviction_probabilities=self._probabilities[key.layer_id])
        else:
            lease = cache._prefetch_nonblocking(key, resident_only=resident_only)
        if lease is None:
            return False
        self._leases[key] = lease
        self._held[key.layer_id] += 1
        if key.layer_id not in self._actual:
            self._speculative += 1
        if key in cache._resident:  # published only after its copy completed
            self._done_events.add(lease.ready_event)
        if cache._submission_sequence != submitted_before:
            self._pending.append(lease.ready_event)
            self._rank[key] = (0, self._copy_order)
            self._copy_order += 1
            st = self._layer_stats[key.layer_id]
            if prediction:
                self._prediction_copies.add(key)
                st.prediction_copies += 1
            else:
                st.demand_copies += 1
            self._peak_inflight = max(self._peak_inflight, len(self._pending))
            self._record("copy", layer=key.layer_id, expert=key.expert_id, prediction=prediction,
                         slot_wait=force)
        else:
            transfer = cache._inflight.get(key)
            self._rank[key] = (-1, transfer.submission_sequence if transfer else -1)
        self._peak_speculative = max(self._peak_speculative, self._speculative)
        return True

    def _protect_predicted_residents(self, layer: int) -> None:
        """Lease the predicted experts of ``layer`` that are already resident
        or in flight before any miss of the layer can evict them (once)."""
        if layer in self._residents_protected:
            return
        cache = self._caches[layer]
        if cache._resident or cache._inflight:
            for key in self._requests[layer]:
                if self._held[layer] >= self._limits[layer]:
                    break
                if key not in self._leases:
                    self._hold(key, resident_only=True)
        self._residents_protected.add(layer)

    def _pump(self) -> None:
        self._reap()
        end = min(len(self._layers), self._current_layer + self.lookahead_layers + 1)
        for layer in range(self._current_layer, end):
            demand = layer in self._actual
            if not demand:
                self._protect_predicted_residents(layer)
            queue = self._requests[layer]
            while queue:
                key = queue[0]
                if key in self._leases:
                    queue.popleft()
                    continue
                if not demand and self._held[layer] >= self._limits[layer]:
                    return
                if self._hold(key, resident_only=True):
                    queue.popleft()
                    continue
                if len(self._pending) >= self.max_inflight:
                    return
                if not self._hold(key, prediction=not demand):
                    return
                queue.popleft()
            # A farther layer is only considered once this one is placed.

    # ------------------------------------------------------------ schedule
    def experts(self, layer: int, active_experts: tuple):
        """Yield ``(expert_id, lease)`` for every actual expert of ``layer``
        once, completed transfers first."""
        if not self._entered or self._open_layer != layer or layer in self._actual:
            raise RuntimeError("expert scheduling must follow this layer's Attention exactly once")
        actual = set(active_experts)
        self._speculative -= self._held[layer]
        self._actual[layer] = actual
        remaining = dict.fromkeys(ExpertKey(layer, e) for e in sorted(actual))
        st = self._layer_stats[layer]
        st.actual_experts = len(actual)
        self._record("router", layer=layer, experts=list(active_experts))
        for key in tuple(self._leases):  # wrong predictions go first
            if key.layer_id == layer and key.expert_id not in actual:
                self._drop(key).release()
        st.unused_prediction_copies = sum(k.layer_id == layer and k.expert_id not in actual
                                          for k in self._prediction_copies)
        for key in remaining:
            if key not in self._leases:
                self._hold(key, resident_only=True)
            lease = self._leases.get(key)
            if lease is None:
                st.missing_at_router += 1
            elif self._ready(lease.ready_event):
                st.ready_at_router += 1
            else:
                st.inflight_at_router += 1
        self._requests[layer] = deque(k for k in remaining if k not in self._leases)
        while remaining:
            self._pump()
            ready = oldest = None
            for key in remaining:
                lease = self._leases.get(key)
                if lease is None:
                    continue
                if self._ready(lease.ready_event):
                    ready = key
                    break
                if oldest is None or self._rank[key] < self._rank[oldest]:
                    oldest = key
            if ready is not None:
                key, waited = ready, False
            elif oldest is not None:
                key, waited = oldest, True
                st.compute_waits += 1
            else:
                self._reap()
                if len(self._pending) >= self.max_inflight:
                    # Only earlier or speculative copies are running and none of
                    # this layer's experts is leased: wait for one credit.
                    self._queue_capacity_waits += 1
                    self._pending[0].synchronize()
                    continue
                # Every reusable slot may still be read by submitted kernels;
                # only the real demand may queue a fill behind them.
                self._hold(next(iter(remaining)), force=True)
                self._slot_wait_copies += 1
                continue
            lease = self._drop(key)
            del remaining[key]
            self._record("compute", layer=layer, expert=key.expert_id, waited=waited)
            try:
                yield key.expert_id, lease
                st.computed_experts += 1
            finally:
                lease.release()
        self._pump()
        self._open_layer = None
        self._next_layer = layer + 1
        self._record("layer_complete", layer=layer)

    # ------------------------------------------------------------- records
    def stats(self) -> dict:
        """Host-side statistics (no GPU synchronisation)."""
        return dict(complete=self._complete, lookahead_layers=self.lookahead_layers,
                    max_inflight=self.max_inflight, prefetch_slot_limits=list(self._limits),
                    peak_inflight=self._peak_inflight,
                    peak_speculative_leases=self._peak_speculative,
                    queue_capacity_waits=self._queue_capacity_waits,
                    slot_wait_copies=self._slot_wait_copies,
                    layers=[asdict(row) for row in self._layer_stats])

    def events(self) -> tuple:
        return tuple(dict(row) for row in self._events)
