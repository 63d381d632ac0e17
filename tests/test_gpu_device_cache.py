"""Device-managed expert caches on the GPU.

In device-managed mode a layer's cache bookkeeping runs on the device
(``csrc/expert_directory.cu``): the plan kernel takes the host wave loop's
lease / eviction / fill decisions and a kernel copies the missing experts
from page-locked host memory.  The bar: outputs bit-identical to the
host-managed path on the same passes, and afterwards the same slots,
generations, LRU stamps and counters as the host-managed cache (both
execution policies, waves when a layer needs more experts than slots); a
verify pass with misses captured in one CUDA graph replays the eager
logits bit for bit.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _layer_pool(layer_id, experts, seed):
    from specfit_b200 import synthetic
    from specfit_b200.runtime.qwen3_verifier import ExpertHostPool

    weights, x = synthetic.bf16_layer_inputs(seed=seed, tokens=65, experts=experts)
    pool = ExpertHostPool(1, experts, 3 * 2048 * 768)
    for e in range(experts):
        pool.data[0, e].copy_(weights.packed(e))
    return pool, x


def _slot_view(snap):
    return [(s.expert_id, s.generation, s.last_used_sequence, s.ready) for s in snap.slots]


@pytest.mark.parametrize("slots,policy", [(24, "expert_id_ascending"), (24, "resident_first"),
                                          (5, "expert_id_ascending"), (5, "resident_first"),
                                          (128, "expert_id_ascending")])
def test_device_managed_layer_equals_host_managed(slots, policy):
    from specfit_b200 import runtime as rt

    pool, x = _layer_pool(2, 128, seed=51)
    xd = x.to(DEV)
    caches, modules = [], []
    for _ in range(2):
        c = rt.GpuExpertCache({rt.ExpertKey(2, e): pool.data[0, e] for e in range(128)}, slot_count=slots,
                              device=DEV, adopt_pinned_sources=True)
        caches.append(c)
        modules.append(rt.Qwen3OffloadedExperts(layer_id=2, cache=c, hidden_size=2048, intermediate_size=768,
                                                execution_policy=policy))
    try:
        caches[1].enter_device_mode()
        rng = np.random.default_rng(slots)
        for step in range(5):
            # Skewed routes over a drifting expert subset: hits, misses and evictions.
            lo = 7 * step
            idx = np.stack([lo + rng.permutation(40)[:8] for _ in range(65)]) % 128
            w = rng.dirichlet(np.ones(8), size=65).astype(np.float32)
            it, wt = torch.from_numpy(idx).to(DEV), torch.from_numpy(w).to(DEV)
            host = modules[0](xd, it, wt)
            dev = modules[1](xd, it, wt)
            torch.cuda.synchronize()
            assert torch.equal(host, dev), step
            a, b = caches[0].stats(), caches[1].stats()
            assert (a.h2d_submissions, a.resident_hits, a.inflight_joins, a.evictions) == \
                (b.h2d_submissions, b.resident_hits, b.inflight_joins, b.evictions), step
            assert _slot_view(caches[0].snapshot()) == _slot_view(caches[1].snapshot()), step
        assert caches[0].stats().h2d_submissions > 0
        caches[1].leave_device_mode()
        assert not caches[1].device_managed
        # Host-managed again: the next pass continues from the same state.
        idx = np.stack([rng.permutation(128)[:8] for _ in range(65)])
        it = torch.from_numpy(idx).to(DEV)
        wt = torch.full((65, 8), 0.125, device=DEV)
        assert torch.equal(modules[0](xd, it, wt), modules[1](xd, it, wt))
        assert _slot_view(caches[0].snapshot()) == _slot_view(caches[1].snapshot())
    finally:
        for c in caches:
            c.close()
        pool.close()


def test_device_managed_mode_refuses_host_leases():
    from specfit_b200 import runtime as rt

    pool, _ = _layer_pool(0, 4, seed=3)
    c = rt.GpuExpertCache({rt.ExpertKey(0, e): pool.data[0, e] for e in range(4)}, slot_count=2,
                          device=DEV, adopt_pinned_sources=True)
    try:
        c.acquire(rt.ExpertKey(0, 1)).release()
        c.enter_device_mode()
        with pytest.raises(RuntimeError, match="device-managed"):
            c.acquire(rt.ExpertKey(0, 0))
        assert c.resident_expert_ids() == (rt.ExpertKey(0, 1),)
        c.leave_device_mode()
        c.acquire(rt.ExpertKey(0, 0)).release()
    finally:
        c.close()
        pool.close()


def test_device_managed_verify_pass_graph_replays_eager():
    """A small target with 3 slots per 16-expert layer: the eager verify
    pass with host-managed caches, the same pass with device-managed caches,
    and its CUDA-graph replay give the same logits and leave the caches in
    the same state."""
    from test_gpu_model import make_tree, small_config

    from specfit_b200.runtime.kv_cache import ReservedCache
    from specfit_b200.runtime.lean_forward import LeanQwen3Forward
    from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3
    from specfit_b200.runtime.verify_graph import VerifyGraph

    models = [build_random_offloaded_qwen3(device=DEV, slots_per_layer=3, config=small_config(), seed=5,
                                           std=0.05) for _ in range(2)]
    try:
        ctx = torch.randint(0, 512, (1, 37), generator=torch.Generator().manual_seed(2)).to(DEV)
        tree = make_tree(nodes=9, depth=4, seed=1)
        ids = tree.verification_token_ids(torch.tensor([[5]], device=DEV))
        mask = tree.verification_attention_mask(base_kv_length=37, device=DEV)
        pos = tree.verification_position_ids(base_kv_length=37, device=DEV)
        kv, fwd = [], []
        for m in models:
            lean = LeanQwen3Forward(m.model)
            cache = ReservedCache(config=m.model.config, capacity=47)
            with torch.no_grad():
                lean(input_ids=ctx, past_key_values=cache, use_cache=True)
            kv.append(cache)
            fwd.append(lean)
        models[1].enter_device_managed_caches()
        host, dev = [], []
        for i in range(3):
            for m, lean, cache, out in zip(models, fwd, kv, (host, dev)):
                with torch.no_grad():
                    out.append(lean(input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=cache,
                                    use_cache=True).logits.clone())
                cache.crop(37)
            torch.cuda.synchronize()
            assert torch.equal(host[i], dev[i]), i
        assert models[0].cache_stats() == models[1].cache_stats()
        vg = VerifyGraph(models[1].model, kv[1], q_len=10, device=DEV, forward=fwd[1])
        vg.capture(ids, mask, pos)  # two warm-up passes run for real
        for i in range(2):
            with torch.no_grad():
                fwd[0](input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=kv[0], use_cache=True)
            kv[0].crop(37)
        ref = None
        for i in range(3):
            with torch.no_grad():
                ref = fwd[0](input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=kv[0],
                             use_cache=True).logits.clone()
            kv[0].crop(37)
            vg.load(ids, mask, pos)
            vg.replay()
            torch.cuda.synchronize()
            assert torch.equal(vg.logits, ref), i
        assert models[0].cache_stats() == models[1].cache_stats()
        assert models[1].cache_stats()["h2d_submissions"] > 0
    finally:
        for m in models:
            m.close()


@pytest.mark.parametrize("slots", [3, 6, 16])
def test_sweep_fills_follow_the_lru_replay(slots):
    """Configuration 3's shape on a small target: per-layer Zipf(1.1) routes
    replace the router for a 33-row verify pass; from empty caches, the fills
    of each of four passes equal the reference's logical LRU replay
    (src/specfit/replay.py:156-285, oracle/cache_oracle.py) — with
    host-managed caches and with device-managed ones, where a layer needs
    more experts than it has slots (waves) or fewer."""
    from test_gpu_model import make_tree

    from oracle.cache_oracle import replay_passes
    from specfit_b200 import synthetic
    from specfit_b200.runtime.kv_cache import ReservedCache
    from specfit_b200.runtime.lean_forward import LeanQwen3Forward
    from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3, qwen3_moe_config

    cfg = qwen3_moe_config(3, hidden=256, experts=16, top_k=4, moe_inter=128, heads=8, kv_heads=2,
                           head_dim=128, vocab=512)
    m = build_random_offloaded_qwen3(device=DEV, slots_per_layer=slots, config=cfg, seed=9, std=0.05)
    try:
        tree = make_tree(nodes=32, depth=6, seed=3)
        T = 33
        routes = [torch.from_numpy(synthetic.zipf_routes(T, l, seed=4, experts=16, top_k=4)).to(DEV)
                  for l in range(3)]
        for l, layer in enumerate(m.model.model.layers):
            layer.mlp.gate.register_forward_hook(
                lambda mod, a, out, l=l: (out[0], out[1], routes[l]) if out[2].shape[0] == T else None)
        expected = replay_passes(slots, [r.cpu().numpy().reshape(-1) for r in routes], passes=4)
        lean = LeanQwen3Forward(m.model)
        cache = ReservedCache(config=m.model.config, capacity=20 + T)
        ctx = torch.randint(0, 512, (1, 20), generator=torch.Generator().manual_seed(6)).to(DEV)
        with torch.no_grad():
            lean(input_ids=ctx, past_key_values=cache, use_cache=True)
        ids = tree.verification_token_ids(torch.tensor([[9]], device=DEV))
        mask = tree.verification_attention_mask(base_kv_length=20, device=DEV)
        pos = tree.verification_position_ids(base_kv_length=20, device=DEV)
        outs = {}
        for mode in ("host", "device"):
            m.cold_reset_caches()
            if mode == "device":
                m.enter_device_managed_caches()
            fills, logits = [], []
            for _ in range(4):
                before = m.cache_stats()["h2d_submissions"]
                with torch.no_grad():
                    logits.append(lean(input_ids=ids, attention_mask=mask, position_ids=pos,
                                       past_key_values=cache, use_cache=True).logits.clone())
                cache.crop(20)
                torch.cuda.synchronize()
                fills.append(m.cache_stats()["h2d_submissions"] - before)
            assert fills == expected, (mode, fills, expected)
            outs[mode] = logits
            m.leave_device_managed_caches()
        for a, b in zip(outs["host"], outs["device"]):
            assert torch.equal(a, b)
    finally:
        m.close()


def test_captured_later_waves_run_only_when_needed():
    """The waves after a layer's first are captured behind a conditional
    node that the plan kernel opens only when the layer's experts do not fit
    its slots.  Routes held in a device buffer (read by the captured pass)
    switch each layer between 4 experts (one wave with 6 slots) and ~16
    (three waves) from one replay to the next: every replay gives the eager
    host-managed pass's logits bit for bit, the caches end in the same state,
    and the directories show which layers used later waves."""
    from test_gpu_model import make_tree

    from specfit_b200 import synthetic
    from specfit_b200.runtime.kv_cache import ReservedCache
    from specfit_b200.runtime.lean_forward import LeanQwen3Forward
    from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3, qwen3_moe_config
    from specfit_b200.runtime.verify_graph import VerifyGraph

    cfg = qwen3_moe_config(3, hidden=256, experts=16, top_k=4, moe_inter=128, heads=8, kv_heads=2,
                           head_dim=128, vocab=512)
    T, L = 13, 3
    rng = np.random.default_rng(11)
    few = [torch.from_numpy(np.stack([rng.permutation(4) for _ in range(T)])).to(DEV) for _ in range(L)]
    many = [torch.from_numpy(synthetic.zipf_routes(T, l, seed=8, experts=16, top_k=4)).to(DEV)
            for l in range(L)]
    routes = torch.empty(L, T, 4, dtype=torch.int64, device=DEV)
    plans = [("few", "many", "few"), ("many", "few", "many"), ("few", "few", "few"), ("many", "many", "many"),
             ("many", "few", "few")]

    def set_routes(plan):
        for l, kind in enumerate(plan):
            routes[l].copy_((few if kind == "few" else many)[l])

    set_routes(plans[0])
    models = [build_random_offloaded_qwen3(device=DEV, slots_per_layer=6, config=cfg, seed=12, std=0.05)
              for _ in range(2)]
    try:
        for m in models:
            for l, layer in enumerate(m.model.model.layers):
                layer.mlp.gate.register_forward_hook(
                    lambda mod, a, out, l=l: (out[0], out[1], routes[l]) if out[2].shape[0] == T else None)
        ctx = torch.randint(0, 512, (1, 21), generator=torch.Generator().manual_seed(3)).to(DEV)
        tree = make_tree(nodes=T - 1, depth=4, seed=2)
        ids = tree.verification_token_ids(torch.tensor([[7]], device=DEV))
        mask = tree.verification_attention_mask(base_kv_length=21, device=DEV)
        pos = tree.verification_position_ids(base_kv_length=21, device=DEV)
        kv, fwd = [], []
        for m in models:
            lean = LeanQwen3Forward(m.model)
            cache = ReservedCache(config=m.model.config, capacity=21 + T)
            with torch.no_grad():
                lean(input_ids=ctx, past_key_values=cache, use_cache=True)
            kv.append(cache)
            fwd.append(lean)
        models[1].enter_device_managed_caches()
        vg = VerifyGraph(models[1].model, kv[1], q_len=T, device=DEV, forward=fwd[1])
        vg.capture(ids, mask, pos)  # two warm-up passes run for real
        for _ in range(2):
            with torch.no_grad():
                fwd[0](input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=kv[0], use_cache=True)
            kv[0].crop(21)
        for plan in plans:
            set_routes(plan)
            with torch.no_grad():
                ref = fwd[0](input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=kv[0],
                             use_cache=True).logits.clone()
            kv[0].crop(21)
            vg.load(ids, mask, pos)
            vg.replay()
            torch.cuda.synchronize()
            assert torch.equal(vg.logits, ref), plan
            later = [int(c.directory.wave_count[1:].sum()) > 0 for c in models[1].caches]
            assert later == [kind == "many" for kind in plan], (plan, later)
        assert models[0].cache_stats() == models[1].cache_stats()
        from specfit_b200 import _native as N

        assert N.device_status(reset=True) == 0
    finally:
        for m in models:
            m.close()
