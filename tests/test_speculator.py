"""Speculative-decoding pieces on the CPU: the simulated acceptance walk,
candidate-pool validation and sub-tree extraction (reference rules of
eagle3_types.py:86-300), the per-token route function, and KV compaction of
the accepted rows (``_compact_tree_cache``, eagle3_tree.py:833-858) on the
reserved cache against a plain DynamicCache."""
import math

import numpy as np
import pytest
import torch

from specfit_b200 import synthetic
from specfit_b200.runtime.eagle3_types import Eagle3DraftCandidate, Eagle3DraftCandidatePool
from specfit_b200.runtime.kv_cache import ReservedCache, compact_tree_cache_
from specfit_b200.runtime.qwen3_verifier import qwen3_moe_config
from specfit_b200.runtime.speculator import BernoulliAcceptance


def cand(raw, parent, depth, tok, lp, cum, path):
    return Eagle3DraftCandidate(raw, parent, depth, tok, lp, cum, raw - 1, path)


def small_pool():
    l = math.log
    c = [cand(1, 0, 1, 10, l(.5), l(.5), (10,)), cand(2, 0, 1, 11, l(.25), l(.25), (11,)),
         cand(3, 1, 2, 12, l(.5), l(.25), (10, 12)), cand(4, 3, 3, 13, l(.5), l(.125), (10, 12, 13))]
    return Eagle3DraftCandidatePool(9, 2, 3, tuple(c), 3, 3)


def test_pool_to_tree_and_validation():
    pool = small_pool()
    tree = pool.to_tree((1, 3, 4))
    assert tree.token_ids == (10, 12, 13) and tree.parent_ids == (0, 1, 2) and tree.source_raw_ids == (1, 3, 4)
    with pytest.raises(ValueError, match="ancestor-closed"):
        pool.to_tree((3,))
    with pytest.raises(ValueError, match="absent"):
        pool.to_tree((7,))
    bad = list(pool.candidates)
    bad[2] = cand(3, 1, 2, 12, math.log(.5), math.log(.3), (10, 12))
    with pytest.raises(ValueError, match="cumulative score"):
        Eagle3DraftCandidatePool(9, 2, 3, tuple(bad), 3, 3)
    bad[2] = cand(3, 0, 1, 10, math.log(.5), math.log(.5), (10,))
    with pytest.raises(ValueError, match="distinct token"):
        Eagle3DraftCandidatePool(9, 2, 3, tuple(bad[:3]), 3, 3)


def test_tree_from_arrays_matches_pool_to_tree():
    """The array form of to_tree (the device-drafting fast path) builds the
    same tree and refuses the same selections."""
    from specfit_b200.runtime.eagle3_types import tree_from_arrays

    pool = small_pool()
    c = pool.candidates
    arrays = (np.array([x.target_token_id for x in c]), np.array([x.parent_raw_id for x in c]),
              np.array([x.depth for x in c]), np.array([x.conditional_log_probability for x in c]),
              np.array([x.cumulative_log_probability for x in c]))
    for sel_ids in ((1, 3, 4), (4, 3, 1), (2,), (1, 2, 3)):
        a, b = pool.to_tree(sel_ids), tree_from_arrays(sel_ids, *arrays)
        assert a.token_ids == b.token_ids and a.parent_ids == b.parent_ids and a.depths == b.depths
        assert a.source_raw_ids == b.source_raw_ids
        assert np.allclose(a.conditional_probabilities, b.conditional_probabilities)
        assert np.allclose(a.cumulative_log_probabilities, b.cumulative_log_probabilities)
    for bad, msg in (((3,), "ancestor-closed"), ((7,), "absent"), ((1, 1), "unique"), ([1], "tuple")):
        with pytest.raises(ValueError, match=msg):
            tree_from_arrays(bad, *arrays)


def test_device_footprints_match_native_packer():
    """footprints_device (the in-graph packing) sets the bits of the native
    packer sf_specfit_pack_routes."""
    from specfit_b200 import selection as sel

    r = synthetic.token_routes(torch.arange(61) * 977 + 5, 48, experts=128, top_k=8, seed=3)
    assert np.array_equal(sel.footprints(r.numpy(), 128),
                          sel.footprints_device(r, 128).numpy().view(np.uint64))


def test_acceptance_walk_follows_first_accepted_child():
    tree = small_pool().to_tree((1, 2, 3, 4))
    acc = BernoulliAcceptance(seed=3)
    acc.p[:] = 1.0
    assert acc.path(tree) == (1, 3, 4)  # node 1 is the first accepted child of the seed
    acc.p[:] = 0.0
    assert acc.path(tree) == ()
    acc.p[:] = [1.0, 0.0, 1.0, 1, 1, 1, 1, 1]
    assert acc.path(tree) == (1,)
    draws = BernoulliAcceptance(seed=5).p
    assert np.all((draws > 0) & (draws < 1)) and len(draws) == 8


def test_token_routes_are_per_token_and_distinct():
    t = torch.tensor([3, 3, 151935, 0])
    r = synthetic.token_routes(t, 4)
    assert r.shape == (4, 4, 8) and torch.equal(r[0], r[1]) and not torch.equal(r[0], r[2])
    assert all(len(set(r[i, l].tolist())) == 8 for i in range(4) for l in range(4))
    assert int(r.min()) >= 0 and int(r.max()) < 128


def test_compaction_matches_dynamic_cache():
    from transformers import DynamicCache

    cfg = qwen3_moe_config(2)
    g = torch.Generator().manual_seed(1)
    caches = [DynamicCache(config=cfg), ReservedCache(config=cfg, capacity=40)]
    for n in (20, 6):
        for layer in range(2):
            k = torch.randn(1, 4, n, 8, generator=g)
            v = torch.randn(1, 4, n, 8, generator=g)
            for c in caches:
                c.update(k, v, layer)
    ref, res = caches
    for layer in ref.layers:  # the reference's compaction, restated on the DynamicCache
        src = torch.tensor([20, 22, 25])
        keys, values = layer.keys.index_select(-2, src), layer.values.index_select(-2, src)
        layer.keys[..., 20:23, :].copy_(keys)
        layer.values[..., 20:23, :].copy_(values)
    ref.crop(23)
    compact_tree_cache_(res, base_kv_length=20, verification_positions=(0, 2, 5), verification_node_count=6)
    assert res.get_seq_length() == 23
    for a, b in zip(ref.layers, res.layers):
        assert torch.equal(a.keys, b.keys) and torch.equal(a.values, b.values)
    with pytest.raises(RuntimeError, match="unexpected length"):
        compact_tree_cache_(res, base_kv_length=20, verification_positions=(0,), verification_node_count=6)


def test_static_mode_writes_at_the_device_offset():
    cfg = qwen3_moe_config(1)
    c = ReservedCache(config=cfg, capacity=16)
    k = torch.arange(4 * 5 * 2, dtype=torch.float32).view(1, 4, 5, 2)
    c.update(k, k + 1, 0)
    off = torch.tensor(7)
    c.set_static(off, reported_length=13)
    assert c.get_seq_length() == 13
    kk, vv = c.update(k[..., :3, :] * 10, k[..., :3, :] * 20, 0)
    assert kk.shape[-2] == 16  # the whole reserved buffer
    assert torch.equal(kk[..., 7:10, :], k[..., :3, :] * 10) and torch.equal(vv[..., 7:10, :], k[..., :3, :] * 20)
    assert torch.equal(kk[..., :5, :], k) and torch.count_nonzero(kk[..., 10:, :]) == 0
    c.set_static(None)
    c.set_length(10)
    assert c.get_seq_length() == 10 and c.layers[0].keys.shape[-2] == 10


def test_verify_inputs_restate_the_tree_rows():
    """The graph path's [3, q] input block and its device-side visibility
    rule reproduce Eagle3DraftTree's positions and verification mask."""
    from specfit_b200.runtime.eagle3_types import Eagle3DraftTree
    from specfit_b200.runtime.speculator import verify_input_rows, visibility_from_ancestors

    rng = np.random.default_rng(4)
    for n in (0, 1, 3, 7):
        parents = tuple(int(rng.integers(0, i + 1)) for i in range(n))
        depths = []
        for p in parents:
            depths.append(1 if p == 0 else depths[p - 1] + 1)
        tree = Eagle3DraftTree(tuple(range(10, 10 + n)), parents, tuple(depths), (0.5,) * n,
                               tuple(math.log(0.5) * d for d in depths), tuple(range(5, 5 + n)))
        base, cap = 37, 37 + 8 + 5
        rows = verify_input_rows(tree, base)
        assert [r[0] for r in rows] == [0] + list(range(5, 5 + n))
        assert [r[1] for r in rows] == tree.verification_position_ids(base_kv_length=base, device="cpu")[0].tolist()
        anc = torch.tensor([r[2] for r in rows])
        vis = visibility_from_ancestors(anc, torch.tensor(base), cap)
        ref = tree.verification_attention_mask(base_kv_length=base, device="cpu")[0, 0]
        assert torch.equal(vis[:, : base + 1 + n], ref)
        assert not vis[:, base + 1 + n:].any()
