"""End-to-end speculative decoding on the GPU (configuration 4 pieces).

* The drafter stand-in grows a valid candidate pool (4 + 8 per level, depth
  <= 8) whose scores are its own log-probabilities.
* ``B200TreeSpeculator.generate`` commits exactly the requested number of
  tokens; after every cycle's in-place compaction the KV cache holds the
  context plus every committed token but the pending one.
* Commit audit: the compacted cache rows equal, within bf16 tolerance, the
  rows a plain causal forward over the same committed sequence produces
  (the reference's commit audit compares the same rows), with eager verify
  passes and with the per-tree-size CUDA graphs over the static cache."""
import pytest
import torch

from specfit_b200 import synthetic
from specfit_b200.runtime.eagle3_drafter import build_random_drafter
from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3, qwen3_moe_config
from specfit_b200.runtime.speculator import B200TreeSpeculator, BernoulliAcceptance
from specfit_b200.selection import SelectionCostModel

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def small():
    cfg = qwen3_moe_config(3, hidden=256, experts=16, top_k=4, moe_inter=128, heads=8, kv_heads=2,
                           head_dim=128, vocab=512)
    m = build_random_offloaded_qwen3(device=DEV, slots_per_layer=16, config=cfg, seed=6, std=0.05)
    m.warm_all_caches()
    d = build_random_drafter(m.model, seed=9, std=0.05, inter=512, aux_layers=(0, 1, 2))
    return cfg, m, d


def cost():
    return SelectionCostModel(synthetic.SELECTION_SIZE_MEAN_NS, synthetic.SELECTION_INTERCEPT_NS,
                              synthetic.SELECTION_EXPERT_NS)


def test_drafter_pool_shape():
    cfg, m, d = small()
    try:
        ids = torch.randint(0, 512, (1, 30), generator=torch.Generator().manual_seed(1)).to(DEV)
        d.begin_generation(200)
        aux = torch.randn(30, 3 * 256, device=DEV).to(torch.bfloat16)
        pool = d.build_candidate_pool(fed_ids=ids, aux_history=aux, pending_seed=ids[:, -1:],
                                      top_k=4, max_depth=8, first_width=4, level_width=8)
        assert len(pool.candidates) == 4 + 8 * 7
        assert pool.actual_depth == 8
        assert sum(c.depth == 1 for c in pool.candidates) == 4
        assert all(c.cumulative_log_probability <= 0 for c in pool.candidates)
        assert d._len == 31  # committed rows + the seed row
        d.end_generation()
    finally:
        m.close()


@pytest.mark.parametrize("graphs", [False, True])
def test_generate_commits_and_audit_matches_causal_forward(graphs):
    from transformers import DynamicCache

    import specfit_b200.runtime.speculator as sp

    cfg, m, d = small()
    try:
        ctx = torch.randint(0, 512, (1, 40), generator=torch.Generator().manual_seed(2)).to(DEV)
        spec = B200TreeSpeculator(m, d, cost_model=cost(), acceptance=BernoulliAcceptance(3),
                                  graphs=graphs)
        keep = {}
        real = sp.compact_tree_cache_

        def spy(cache, **kw):  # keep the cache of the last compaction
            real(cache, **kw)
            keep["cache"] = cache
        sp.compact_tree_cache_ = spy
        try:
            res = spec.generate(ctx, 24)
        finally:
            sp.compact_tree_cache_ = real
        assert res.committed == 24
        assert all(c.selected <= 7 and c.accepted <= c.selected for c in res.cycles)
        assert sum(c.selected for c in res.cycles) > 0  # SpecFit verifies drafted nodes
        cache = keep["cache"]
        n = cache.get_seq_length() - 40
        assert 0 < n <= 24
        # Causal forward over the context + the committed tokens held in the
        # cache, with the per-token routes the verify passes used.
        seq = torch.cat((ctx, torch.tensor([res.tokens[:n]], device=DEV)), dim=1)
        routes = synthetic.token_routes(seq[0], cfg.num_hidden_layers, experts=16, top_k=4)
        hooks = [layer.mlp.gate.register_forward_hook(
            lambda mod, a, out, l=l: (out[0], out[1], routes[40:, l, :]) if out[2].shape[0] == n else None)
            for l, layer in enumerate(m.model.model.layers)]
        try:
            ref = DynamicCache(config=m.model.config)
            with torch.no_grad():
                m.model(input_ids=seq[:, :40], past_key_values=ref, use_cache=True)
                m.model(input_ids=seq[:, 40:], past_key_values=ref, use_cache=True)
        finally:
            for h in hooks:
                h.remove()
        for a, b in zip(cache.layers, ref.layers):
            assert torch.allclose(a.keys[..., 40:, :].float(), b.keys[..., 40:, :].float(), atol=2e-2, rtol=0)
            assert torch.allclose(a.values[..., 40:, :].float(), b.values[..., 40:, :].float(), atol=2e-2, rtol=0)
        spec.release_graphs()
    finally:
        m.close()


def test_device_drafting_matches_eager_drafting():
    """From the same drafter state, the graph-replayed device drafting grows
    the pool the eager drafting grows: the same level-1 tokens, log-probs
    within bf16 tolerance, and (nearly) the same (parent, token) pairs
    (scores computed in a different order may swap exact near-ties)."""
    from specfit_b200.runtime.eagle3_drafter import DeviceDraft

    cfg, m, d = small()
    try:
        g = torch.Generator().manual_seed(5)
        ids = torch.randint(0, 512, (1, 33), generator=g).to(DEV)
        aux = torch.randn(33, 3 * 256, generator=g).to(DEV).to(torch.bfloat16)
        d.begin_generation(256)
        d.build_candidate_pool(fed_ids=ids[:, :30], aux_history=aux[:30], pending_seed=ids[:, 30:31])
        state = (d._k.clone(), d._v.clone(), d._len, d._fed)
        kw = dict(fed_ids=ids[:, :33], aux_history=aux[:33], pending_seed=ids[:, 32:33] * 0 + 7)
        eager = d.build_candidate_pool(top_k=4, max_depth=8, first_width=4, level_width=8, **kw)
        d._k.copy_(state[0]); d._v.copy_(state[1]); d._len, d._fed = state[2], state[3]
        dd = DeviceDraft(d, top_k=4, max_depth=8, first_width=4, level_width=8, max_new=9)
        dev_pool = dd.pool(**kw)
        assert d._fed == 34 and d._len == state[2] + 3  # 2 new committed rows + the new seed row
        a, b = eager.candidates, dev_pool.candidates
        assert len(a) == len(b) == 60
        assert [c.target_token_id for c in a[:4]] == [c.target_token_id for c in b[:4]]
        for x, y in zip(a[:4], b[:4]):
            assert abs(x.conditional_log_probability - y.conditional_log_probability) < 5e-2
        pairs = lambda p: {(c.parent_raw_id, c.target_token_id) for c in p}
        assert len(pairs(a) & pairs(b)) >= 0.8 * 60
        dd.release()
    finally:
        m.close()


def test_native_compaction_matches_generic():
    """All-layer KV compaction in two launches (sf_kv_compact) moves the same
    rows as per-layer index_select + copy, including overlapping moves."""
    from specfit_b200.runtime.kv_cache import ReservedCache, compact_tree_cache_

    cfg = qwen3_moe_config(3)
    g = torch.Generator(device="cuda").manual_seed(3)
    caches = [ReservedCache(config=cfg, capacity=64) for _ in range(2)]
    for n in (30, 8):
        for layer in range(3):
            k = torch.randn(1, 4, n, 128, generator=g, device="cuda").to(torch.bfloat16)
            v = torch.randn(1, 4, n, 128, generator=g, device="cuda").to(torch.bfloat16)
            for c in caches:
                c.update(k, v, layer)
    pos = (0, 1, 3, 4, 7)
    compact_tree_cache_(caches[0], base_kv_length=30, verification_positions=pos, verification_node_count=8)
    ref = caches[1]
    for layer in ref.layers:
        src = torch.tensor([30 + p for p in pos], device="cuda")
        kk, vv = layer.keys.index_select(-2, src), layer.values.index_select(-2, src)
        layer.keys[..., 30:35, :].copy_(kk)
        layer.values[..., 30:35, :].copy_(vv)
    ref.crop(35)
    for a, b in zip(caches[0].layers, ref.layers):
        assert torch.equal(a.keys, b.keys) and torch.equal(a.values, b.values)


def test_cycle_calibration_forces_every_tree_size():
    """The reference-style fit times whole cycles at each forced tree size:
    one intercept per size, every size actually verified, and the fitted
    model selects drafted nodes again afterwards."""
    cfg, m, d = small()
    try:
        ctx = torch.randint(0, 512, (1, 40), generator=torch.Generator().manual_seed(4)).to(DEV)
        spec = B200TreeSpeculator(m, d, cost_model=cost(), acceptance=BernoulliAcceptance(5), graphs=True)
        model = spec.calibrate_cycle_cost_model(ctx, expert_ns=500.0, tokens=32)
        assert len(model.size_intercept_ns) == 8 and all(x >= 0 for x in model.size_intercept_ns)
        assert all(x > 0 for x in model.size_mean_ns)
        assert spec.cost_model is not model  # the speculator's own model is restored
        spec.cost_model = model
        res = spec.generate(ctx, 24)
        assert res.committed == 24 and all(c.experts > 0 for c in res.cycles)
        spec.release_graphs()
    finally:
        m.close()


def test_draft_level_kernel_matches_the_eager_sort():
    """sf_draft_level picks the level's nodes by the eager builder's rule
    (score desc, parent asc, token asc; exact ties included) and writes the
    pool rows, ancestor sets, positions and parent hidden rows."""
    import numpy as np

    from specfit_b200 import _native as N

    g = torch.Generator().manual_seed(11)
    rows, k, width, H = 8, 4, 8, 256
    v = -torch.rand(rows, k, generator=g).sort(dim=1, descending=True).values
    v[2, 1] = v[5, 0] = -0.5                       # equal log-probs ...
    cum = (-torch.rand(rows, generator=g)).double()
    cum[5] = cum[2]                                # ... and equal scores across parents
    t = torch.randint(0, 1000, (rows, k), generator=g)
    vis = torch.randint(1, 1 << 20, (rows,), generator=g)
    hid = torch.randn(rows, H, generator=g).to(torch.bfloat16)
    dev = [x.to(DEV) for x in (v, t, cum, vis, hid)]
    seed_pos = torch.tensor(100, device=DEV)
    nt, nc, nv, npos = (torch.zeros(width, dtype=dt, device=DEV)
                        for dt in (torch.long, torch.float64, torch.long, torch.long))
    nh = torch.zeros(width, H, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros(width, 5, dtype=torch.float64, device=DEV)
    rc = N.lib.sf_draft_level(dev[0].data_ptr(), dev[1].data_ptr(), rows, k, dev[2].data_ptr(),
                              dev[3].data_ptr(), dev[4].data_ptr(), H, width, 12, 3, 20,
                              seed_pos.data_ptr(), nt.data_ptr(), nc.data_ptr(), nv.data_ptr(),
                              npos.data_ptr(), nh.data_ptr(), out.data_ptr(),
                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    opts = sorted(((float(cum[j]) + float(v[j, r]), j, int(t[j, r]), float(v[j, r]))
                   for j in range(rows) for r in range(k)), key=lambda o: (-o[0], o[1], o[2]))[:width]
    o = out.cpu().numpy()
    for s, (score, j, tok, cond) in enumerate(opts):
        assert int(nt[s]) == tok and float(nc[s]) == score
        assert int(nv[s]) == int(vis[j]) | (1 << (20 + s)) and int(npos[s]) == 104
        assert torch.equal(nh[s].cpu(), hid[j])
        assert np.array_equal(o[s], [tok, 12 + j, cond, score, 4])
