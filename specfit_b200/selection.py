"""SpecFit exact subtree selection on the native search.

Drop-ins for the reference's selection entry points:

* ``SelectionCostModel`` (``src/specfit/selection_methods.py:26-66``) and
  ``CacheCostModel`` (``src/specfit/selection_refinement.py:83-113``): same
  fields, validation and ``predict_ns``;
* ``exact_specfit_selection(pool, atlas, model, resident_mask=0)``
  (``src/specfit/specfit_exact.py:58-65``): same arguments, validation and
  result (the selected raw ids in increasing order);
* ``LevelSpecFit`` (``src/specfit/main_comparison.py:63-103``): per-cycle
  level-prefix selection with the adaptive-depth stop rule.

Routes are packed into 48 x 128-bit footprints per token (one bit per
(layer, expert)) with numpy and searched by ``sf_specfit_select`` (C++).
Beyond the reference, pools need not have 2/6/10/14/18 nodes (up to 63).
"""
from __future__ import annotations

import ctypes
from dataclasses import asdict, dataclass
from math import isfinite

import numpy as np

from . import _native as N

LAYERS = 48
EXPERTS = 128
WORDS = LAYERS * EXPERTS // 64
MAX_DRAFT_NODES = 7


def _finite_nonneg(x) -> bool:
    return not isinstance(x, bool) and isinstance(x, (int, float)) and isfinite(x) and x >= 0


@dataclass(frozen=True)
class SelectionCostModel:
    """Intercept per selected-node count plus one slope per distinct
    (layer, expert) in the verification footprint."""

    size_mean_ns: tuple
    size_intercept_ns: tuple
    expert_ns: float

    def __post_init__(self):
        if (len(self.size_mean_ns) != MAX_DRAFT_NODES + 1
                or len(self.size_intercept_ns) != MAX_DRAFT_NODES + 1
                or any(isinstance(x, bool) or not isfinite(x) or x <= 0 for x in self.size_mean_ns)
                or any(not _finite_nonneg(x) for x in (*self.size_intercept_ns, self.expert_ns))
                or any(b + 384 * self.expert_ns <= 0 for b in self.size_intercept_ns)):
            raise ValueError("invalid calibrated selection cost model")

    def predict_ns(self, node_count: int, expert_union: int | None = None) -> float:
        if type(node_count) is not int or not 0 <= node_count <= MAX_DRAFT_NODES:
            raise ValueError("draft node count is outside the calibrated range")
        if expert_union is None:
            return self.size_mean_ns[node_count]
        if type(expert_union) is not int or expert_union < 384:
            raise ValueError("expert union must include the mandatory seed in all layers")
        return self.size_intercept_ns[node_count] + self.expert_ns * expert_union

    def to_dict(self) -> dict:
        return {**asdict(self), "size_mean_ns": list(self.size_mean_ns),
                "size_intercept_ns": list(self.size_intercept_ns)}

    @classmethod
    def from_dict(cls, value: dict) -> "SelectionCostModel":
        if set(value) != {"size_mean_ns", "size_intercept_ns", "expert_ns"}:
            raise ValueError("unexpected cost-model fields")
        return cls(tuple(value["size_mean_ns"]), tuple(value["size_intercept_ns"]), value["expert_ns"])


@dataclass(frozen=True)
class CacheCostModel:
    """Size intercepts plus compute work and initially missing expert work."""

    size_intercept_ns: tuple
    expert_ns: float
    missing_ns: float

    def __post_init__(self):
        if (len(self.size_intercept_ns) != MAX_DRAFT_NODES + 1
                or any(not _finite_nonneg(x) for x in
                       (*self.size_intercept_ns, self.expert_ns, self.missing_ns))
                or any(b + 384 * self.expert_ns <= 0 for b in self.size_intercept_ns)):
            raise ValueError("invalid cache-aware cost coefficients")

    def predict_ns(self, count, footprint, missing):
        if (type(count) is not int or not 0 <= count <= MAX_DRAFT_NODES
                or type(footprint) is not int or footprint < 384
                or type(missing) is not int or not 0 <= missing <= footprint):
            raise ValueError("invalid cache-aware query features")
        return self.size_intercept_ns[count] + self.expert_ns * footprint + self.missing_ns * missing

    def to_dict(self):
        return dict(size_intercept_ns=list(self.size_intercept_ns), expert_ns=self.expert_ns,
                    missing_ns=self.missing_ns)

    @classmethod
    def from_dict(cls, value):
        if set(value) != {"size_intercept_ns", "expert_ns", "missing_ns"}:
            raise ValueError("unexpected cache model fields")
        return cls(tuple(value["size_intercept_ns"]), value["expert_ns"], value["missing_ns"])


def _footprint_rows(routes: np.ndarray) -> np.ndarray:
    """``routes`` int [tokens, 48, 8] -> uint64 [tokens, 96] footprint bitsets
    (native packer; raises ValueError on invalid or repeated expert ids)."""
    r = np.ascontiguousarray(routes, dtype=np.int32)
    if r.ndim != 3 or r.shape[1:] != (LAYERS, 8):
        raise ValueError("invalid atlas raw/layer/Top-8")
    out = np.empty((r.shape[0], WORDS), dtype=np.uint64)
    N.check(N.lib.sf_specfit_pack_routes(r.ctypes.data, r.shape[0], LAYERS, 8, EXPERTS,
                                         out.ctypes.data, WORDS), "sf_specfit_pack_routes")
    return out


def footprints(routes: np.ndarray, experts: int = EXPERTS) -> np.ndarray:
    """Any-shape packing: ``routes`` int [tokens, layers, top_k] ->
    uint64 [tokens, ceil(layers * experts / 64)] with bit layer*experts+expert."""
    r = np.ascontiguousarray(routes, dtype=np.int32)
    if r.ndim != 3:
        raise ValueError("routes must be [tokens, layers, top_k]")
    words = (r.shape[1] * experts + 63) // 64
    out = np.empty((r.shape[0], words), dtype=np.uint64)
    N.check(N.lib.sf_specfit_pack_routes(r.ctypes.data, r.shape[0], r.shape[1], r.shape[2], experts,
                                         out.ctypes.data, words), "sf_specfit_pack_routes")
    return out


def footprints_device(routes, experts: int = EXPERTS, out=None):
    """``footprints`` as device work (graph-capturable torch ops): ``routes``
    int64 ``[tokens, layers, top_k]`` with distinct experts per (token,
    layer) -> int64 ``[tokens, words]`` with the same bits (bit layer*experts
    + expert).  Distinct bits make the scatter-add an OR (no carries); no
    validation is done here (the native packer validates)."""
    import torch

    n, layers, k = routes.shape
    words = (layers * experts + 63) // 64
    bit = (torch.arange(layers, device=routes.device, dtype=torch.int64).view(1, layers, 1) * experts
           + routes).reshape(n, layers * k)
    res = out if out is not None else torch.empty(n, words, dtype=torch.int64, device=routes.device)
    res.zero_()
    res.scatter_add_(1, bit >> 6, torch.ones_like(bit) << (bit & 63))
    return res


def pack_routes(pool, atlas) -> np.ndarray:
    """Validate complete top-8 routes of the seed (raw 0) and every node and
    pack them (cf. ``_pack_routes``, ``specfit_exact.py:18-49``)."""
    count = len(pool.nodes)
    expected = tuple(range(count + 1))
    if ((0, *(n.raw_id for n in pool.nodes)) != expected
            or tuple(atlas.position_to_raw) != expected
            or len(atlas.expert_ids_by_raw_layer) != (count + 1) * LAYERS):
        raise ValueError("atlas must cover every candidate and all 48 layers")
    try:
        table = np.array([(raw, layer, *experts) for raw, layer, experts in atlas.expert_ids_by_raw_layer])
    except ValueError:
        raise ValueError("invalid atlas raw/layer/Top-8") from None
    if table.ndim != 2 or table.shape[1] != 10:
        raise ValueError("invalid atlas raw/layer/Top-8")
    if table.dtype.kind not in "iu":
        raise ValueError("invalid expert ID")
    raws, layers = table[:, 0], table[:, 1]
    if raws.min() < 0 or raws.max() > count or layers.min() < 0 or layers.max() >= LAYERS:
        raise ValueError("invalid atlas raw/layer/Top-8")
    cell = raws * LAYERS + layers
    if np.unique(cell).size != cell.size:
        raise ValueError("duplicate atlas raw/layer")
    routes = np.empty((count + 1, LAYERS, 8), dtype=np.int64)
    routes[raws, layers] = table[:, 2:]
    return _footprint_rows(routes)


def resident_words(resident_mask: int) -> np.ndarray:
    if type(resident_mask) is not int or not 0 <= resident_mask < 1 << (LAYERS * EXPERTS):
        raise ValueError("invalid resident bitmap")
    raw = resident_mask.to_bytes(LAYERS * EXPERTS // 8, "little")
    return np.frombuffer(raw, dtype=np.uint64).copy()


def _model_terms(model):
    if isinstance(model, CacheCostModel):
        return np.asarray(model.size_intercept_ns, np.float64), float(model.expert_ns), float(model.missing_ns)
    if isinstance(model, SelectionCostModel):
        return np.asarray(model.size_intercept_ns, np.float64), float(model.expert_ns), 0.0
    raise ValueError("a frozen SpecFit cost model is required")


def search(parents, cum_logp, footprints: np.ndarray, model, resident: np.ndarray | None = None,
           max_nodes: int = MAX_DRAFT_NODES) -> tuple:
    """Run the native search on packed footprints ``[n + 1, words]``."""
    intercept, slope, missing = _model_terms(model)
    n = len(parents)
    par = np.ascontiguousarray(parents, dtype=np.int32)
    cum = np.ascontiguousarray(cum_logp, dtype=np.float64)
    fp = np.ascontiguousarray(footprints, dtype=np.uint64)
    if fp.shape[0] != n + 1:
        raise ValueError("one footprint per node plus the seed is required")
    res = None if resident is None else np.ascontiguousarray(resident, dtype=np.uint64)
    out = np.zeros(max(max_nodes, 1), dtype=np.int32)
    count = ctypes.c_int32(0)
    score = ctypes.c_double(0.0)
    N.check(N.lib.sf_specfit_select(
        n, par.ctypes.data if n else None, cum.ctypes.data if n else None, fp.ctypes.data,
        fp.shape[1], None if res is None else res.ctypes.data, intercept.ctypes.data, max_nodes,
        slope, missing, out.ctypes.data, ctypes.byref(count), ctypes.byref(score)),
        "sf_specfit_select")
    return tuple(int(i) for i in out[: count.value])


def select_from_routes(parents, cum_logp, routes: np.ndarray, model, resident_mask: int = 0,
                       max_nodes: int = MAX_DRAFT_NODES) -> tuple:
    """Same search from array inputs: ``routes`` int [n + 1, 48, 8] (seed
    first), e.g. the per-layer top-8 indices captured from the verify pass."""
    return search(parents, cum_logp, _footprint_rows(routes), model, resident_words(resident_mask),
                  max_nodes)


def exact_specfit_selection(pool, atlas, model, resident_mask: int = 0) -> tuple:
    """Selected raw ids (increasing) of the score-maximising ancestor-closed
    subtree (``specfit_exact.py:58-94``)."""
    if not isinstance(model, (SelectionCostModel, CacheCostModel)):
        raise ValueError("a frozen SpecFit cost model is required")
    res = resident_words(resident_mask)
    footprints = pack_routes(pool, atlas)
    parents = [n.parent_raw_id for n in pool.nodes]
    cum = [n.cumulative_log_probability for n in pool.nodes]
    return search(parents, cum, footprints, model, res)


class LevelSpecFit:
    """Selection over one cycle's level prefixes: each new level's routes are
    packed once, then the exact search runs on the prefix
    (``main_comparison.py:63-103``)."""

    def __init__(self, model, atlas):
        if len(atlas) != LAYERS:
            raise ValueError("route atlas must cover 48 layers")
        self.model, self.atlas = model, atlas
        self._rows: list = []

    def pack(self, nodes) -> np.ndarray:
        count = len(nodes)
        if any(n.raw_id != raw for raw, n in enumerate(nodes, 1)):
            raise ValueError("invalid level-prefix candidate pool")
        for raw in range(len(self._rows), count + 1):
            per_layer = []
            for matrix in self.atlas:
                if len(matrix) <= raw or len(matrix[raw]) != 8:
                    raise ValueError("route atlas does not cover the candidate prefix")
                per_layer.append(tuple(matrix[raw]))
            self._rows.append(_footprint_rows(np.asarray([per_layer], dtype=np.int64))[0])
        return np.stack(self._rows[: count + 1])

    def select(self, nodes) -> tuple:
        footprints = self.pack(nodes)
        return search([n.parent_raw_id for n in nodes], [n.cumulative_log_probability for n in nodes],
                      footprints, self.model, None)

    def stop(self, nodes):
        """Adaptive depth: stop when the selection on the depth<=d prefix
        takes no node of depth d; returns (stop, selection)."""
        ids = self.select(nodes)
        depth = nodes[-1].depth
        return all(nodes[raw - 1].depth != depth for raw in ids), ids
