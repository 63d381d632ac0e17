"""SpecFit exact selection (C++ search behind the reference API).  CPU only.

* Selected subtrees and adaptive-depth stops equal the reference's own
  ``exact_specfit_selection`` / ``LevelSpecFit`` on 93 seeded pools
  (tests/golden/selection.json, made by tests/golden/make_golden.py),
  including its compensated-summation tie case.
* The reward sum equals CPython's builtin ``sum`` bit for bit.
* On pool shapes the reference does not accept (any size, any topology) the
  search equals an independent brute-force enumeration of the objective."""
import itertools
import json
import math
from types import SimpleNamespace

import numpy as np
import pytest

from specfit_b200 import _native as N
from specfit_b200 import selection as sel
from specfit_b200 import synthetic


def objects(case):
    n = len(case.parents)
    nodes = [SimpleNamespace(raw_id=i + 1, parent_raw_id=case.parents[i], depth=case.depths[i],
                             cumulative_log_probability=case.cum_logp[i]) for i in range(n)]
    pool = SimpleNamespace(nodes=nodes)
    atlas = SimpleNamespace(position_to_raw=tuple(range(n + 1)), expert_ids_by_raw_layer=tuple(
        (raw, layer, tuple(int(e) for e in case.routes[raw, layer]))
        for raw in range(n + 1) for layer in range(48)))
    atlas48 = [tuple(tuple(int(e) for e in case.routes[raw, layer]) for raw in range(n + 1))
               for layer in range(48)]
    resident = 0
    for layer in range(48):
        for e in np.nonzero(case.resident[layer])[0]:
            resident |= 1 << (128 * layer + int(e))
    return pool, atlas, atlas48, resident


def build_model(m):
    if m["kind"] == "cache":
        return sel.CacheCostModel(tuple(m["intercept"]), m["expert_ns"], m["missing_ns"])
    return sel.SelectionCostModel(tuple(m["intercept"]), tuple(m["intercept"]), m["expert_ns"])


def load_cases(golden_dir):
    return json.loads((golden_dir / "selection.json").read_text())


def test_selection_matches_reference_golden(golden_dir):
    cases = load_cases(golden_dir)
    assert len(cases) == 93
    for c in cases:
        case = synthetic.selection_case(c["seed"], c["n"], shared_routes=c["shared"],
                                        level_prob=c["level_prob"])
        pool, atlas, atlas48, resident = objects(case)
        model = build_model(c["model"])
        got = sel.exact_specfit_selection(pool, atlas, model, resident if c["resident"] else 0)
        assert list(got) == c["selected"], c
        if "stops" in c:
            level = sel.LevelSpecFit(model, atlas48)
            for prefix, stop, ids in c["stops"]:
                s, i = level.stop(pool.nodes[:prefix])
                assert (bool(s), list(i)) == (stop, ids), (c["seed"], c["n"], prefix)


def test_compensated_sum_equals_python_sum():
    import ctypes

    rng = np.random.default_rng(0)
    probes = [rng.uniform(0, 1, size=k) for k in range(1, 9) for _ in range(200)]
    probes += [np.array([1e16, 1.0, -1e16]), np.array([0.1] * 7), np.array([1.0, 1e-16, 1e-16] * 2),
               np.exp(rng.normal(-3, 2, size=7))]
    for xs in probes:
        xs = np.ascontiguousarray(xs, dtype=np.float64)
        got = N.lib.sf_compensated_sum(xs.ctypes.data_as(ctypes.c_void_p), len(xs))
        assert got == sum(xs.tolist(), start=0.0), xs


def brute(parents, cum, routes, model, resident_bits, max_nodes=7):
    """Independent enumeration of the objective (cf. the reference's
    exhaustive_specfit_choice, main_comparison.py:173-189)."""
    n = len(parents)
    probs = [0.0] + [math.exp(c) for c in cum]
    masks = [set((l, int(e)) for l in range(48) for e in routes[raw, l]) for raw in range(n + 1)]
    intercept, slope, missing = sel._model_terms(model)
    best = None
    for k in range(min(max_nodes, n) + 1):
        for ids in itertools.combinations(range(1, n + 1), k):
            if any(parents[i - 1] not in (0, *ids) for i in ids):
                continue
            union = set(masks[0])
            for i in ids:
                union |= masks[i]
            elapsed = intercept[k] + slope * len(union)
            if missing:
                elapsed += missing * len(union - resident_bits)
            reward = 1.0 + sum((probs[i] for i in ids), start=0.0)
            key = (-reward / elapsed, -reward, len(union), k, ids)
            if best is None or key < best:
                best = key
    return best[-1]


@pytest.mark.parametrize("seed,n", [(1, 5), (2, 9), (3, 12), (4, 11), (5, 8)])
def test_generic_pools_equal_brute_force(seed, n):
    rng = np.random.default_rng(seed)
    parents = [int(rng.integers(0, raw)) for raw in range(1, n + 1)]
    cum = []
    for raw, p in enumerate(parents, start=1):
        cum.append((0.0 if p == 0 else cum[p - 1]) + float(np.log(rng.uniform(0.05, 0.95))))
    # A few distinct route patterns so footprints overlap (ties are possible).
    patterns = [np.stack([rng.permutation(128)[:8] for _ in range(48)]) for _ in range(4)]
    routes = np.stack([patterns[int(rng.integers(0, 4))] for _ in range(n + 1)])
    resident = set((l, int(e)) for l in range(48) for e in rng.permutation(128)[:30])
    res_words = np.zeros(96, dtype=np.uint64)
    for l, e in resident:
        b = 128 * l + e
        res_words[b // 64] |= np.uint64(1) << np.uint64(b % 64)
    fp = sel._footprint_rows(routes)
    for model in (sel.SelectionCostModel(synthetic.SELECTION_INTERCEPT_NS, synthetic.SELECTION_INTERCEPT_NS,
                                         synthetic.SELECTION_EXPERT_NS),
                  sel.CacheCostModel(synthetic.SELECTION_INTERCEPT_NS, synthetic.SELECTION_EXPERT_NS,
                                     0.5 * synthetic.SELECTION_EXPERT_NS),
                  sel.SelectionCostModel((1.0,) * 8, (1.0,) * 8, 0.0)):
        got = sel.search(parents, cum, fp, model, res_words)
        assert got == brute(parents, cum, routes, model, resident), (seed, n, model)


@pytest.mark.parametrize("seed", [11, 12, 13])
def test_pruned_search_on_decode_like_pools(seed):
    """Pools of 15 nodes with a B200-fitted-style model (intercepts of a
    few ms nearly flat in the size, 1.44 us per expert), where the search's
    bound prunes most subtrees: the result equals the brute force."""
    rng = np.random.default_rng(seed)
    n = 15
    parents = [0, 0, 0] + [int(rng.integers(1, raw)) for raw in range(4, n + 1)]
    cum = []
    for raw, p in enumerate(parents, start=1):
        cum.append((0.0 if p == 0 else cum[p - 1]) + float(np.log(rng.uniform(0.3, 0.99))))
    routes = np.stack([np.stack([rng.permutation(128)[:8] for _ in range(48)]) for _ in range(n + 1)])
    fp = sel._footprint_rows(routes)
    ic = tuple(float(x) for x in 5.4e6 + np.sort(rng.uniform(0, 5e5, 8)))
    model = sel.SelectionCostModel(ic, ic, 1439.6)
    assert sel.search(parents, cum, fp, model, None) == brute(parents, cum, routes, model, set())


def test_route_validation_errors(golden_dir):
    case = synthetic.selection_case(3, 6)
    pool, atlas, _, _ = objects(case)
    model = sel.SelectionCostModel((1.0,) * 8, (1.0,) * 8, 0.0)
    bad = list(atlas.expert_ids_by_raw_layer)
    raw, layer, experts = bad[5]
    bad[5] = (raw, layer, (experts[0],) * 8)
    with pytest.raises(ValueError, match="duplicate expert"):
        sel.exact_specfit_selection(pool, SimpleNamespace(position_to_raw=atlas.position_to_raw,
                                                          expert_ids_by_raw_layer=tuple(bad)), model)
    bad[5] = (raw, layer, (128,) + experts[1:])
    with pytest.raises(ValueError, match="invalid expert ID"):
        sel.exact_specfit_selection(pool, SimpleNamespace(position_to_raw=atlas.position_to_raw,
                                                          expert_ids_by_raw_layer=tuple(bad)), model)
    with pytest.raises(ValueError, match="cover every candidate"):
        sel.exact_specfit_selection(pool, SimpleNamespace(position_to_raw=atlas.position_to_raw,
                                                          expert_ids_by_raw_layer=atlas.expert_ids_by_raw_layer[:-1]),
                                    model)
    with pytest.raises(ValueError, match="resident bitmap"):
        sel.exact_specfit_selection(pool, atlas, model, resident_mask=-1)
    with pytest.raises(ValueError, match="cost model"):
        sel.exact_specfit_selection(pool, atlas, object())
