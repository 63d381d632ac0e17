"""Drop-in runtime on the GPU: GpuExpertCache and Qwen3OffloadedExperts.

Scenarios follow the reference's GPU tests (tests/gpu/test_gpu_expert_cache.py
and tests/gpu/test_qwen3_offloaded_experts.py of SpecFit): event order, stats
deltas, LRU victims, in-flight joins, lease protection, snapshots, reset,
close, and the expert math against the oracle."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def rt():
    from specfit_b200 import runtime

    return runtime


def make_sources(n=3, shape=(64, 96), seed=0):
    g = torch.Generator().manual_seed(seed)
    return {e: torch.randn(*shape, generator=g).to(torch.bfloat16) for e in range(n)}


def test_one_slot_102_switches(rt):
    sources = make_sources()
    x = torch.linspace(-1, 1, 4 * 96, device=DEV, dtype=torch.bfloat16).reshape(4, 96)
    expected = {e: F.linear(x, s.to(DEV)) for e, s in sources.items()}
    cache = rt.GpuExpertCache(sources, slot_count=1, device=DEV)
    assert cache.sources_are_pinned
    assert cache.copy_stream.cuda_stream != torch.cuda.default_stream(DEV).cuda_stream
    outs = []
    for i in range(102):
        with cache.acquire(i % 3) as lease:
            outs.append((i % 3, F.linear(x, lease.wait()).clone()))
    torch.cuda.synchronize()
    for e, o in outs:
        torch.testing.assert_close(o, expected[e], rtol=1.6e-2, atol=1.6e-2)
    st = cache.stats()
    assert (st.h2d_submissions, st.evictions) == (102, 101)
    assert cache.resident_expert_ids() == (2,)
    cache.close()


def test_two_acquires_join_one_inflight_copy(rt):
    cache = rt.GpuExpertCache(make_sources(), slot_count=1, device=DEV)
    with torch.cuda.stream(cache.copy_stream):
        torch.cuda._sleep(10_000_000)
    first = cache.acquire(0)
    second = cache.acquire(0)
    try:
        assert cache.stats().h2d_submissions == 1 and cache.stats().inflight_joins == 1
        assert first.slot_id == second.slot_id and first.ready_event is second.ready_event
        assert first.wait().data_ptr() == second.wait().data_ptr()
    finally:
        second.release()
        first.release()
    torch.cuda.synchronize()
    with cache.acquire(0) as lease:
        lease.wait()
    assert cache.stats().resident_hits == 1


def test_active_lease_protects_slot(rt):
    cache = rt.GpuExpertCache(make_sources(), slot_count=1, device=DEV)
    lease = cache.acquire(0)
    with pytest.raises(rt.NoEvictableSlotError):
        cache.acquire(1)
    lease.release()
    with cache.acquire(1) as nxt:
        nxt.wait()
    torch.cuda.synchronize()
    assert cache.resident_expert_ids() == (1,)
    with pytest.raises(KeyError):
        cache.acquire(7)


def test_lru_victim_and_guards(rt):
    cache = rt.GpuExpertCache(make_sources(), slot_count=2, device=DEV)
    for e in (0, 1, 0, 2):
        with cache.acquire(e) as lease:
            lease.wait()
    torch.cuda.synchronize()
    assert cache.resident_expert_ids() == (0, 2)
    assert cache.stats().evictions == 1
    assert cache.stats().pending_use_guards == 0


def test_snapshot_cold_reset_and_close(rt):
    obs = rt.RecordingCacheTransitionObserver("snap")

    class Owner:
        closed = False

        def close(self):
            Owner.closed = True

    srcs = {k: v.pin_memory() for k, v in make_sources().items()}
    cache = rt.GpuExpertCache(srcs, slot_count=2, device=DEV, observer=obs,
                              adopt_pinned_sources=True, source_owner=Owner())
    snap0 = cache.snapshot()
    assert snap0.capacity == 2 and all(s.expert_id is None for s in snap0.slots)
    with cache.acquire(0) as lease:
        lease.wait()
    torch.cuda.synchronize()
    snap = cache.snapshot()
    assert [s.expert_id for s in snap.slots] == [0, None] and snap.slots[0].ready
    kinds = [e.kind for e in obs.events()]
    assert kinds == [rt.RuntimeEventKind.H2D_SUBMIT, rt.RuntimeEventKind.CONSUME_WAIT,
                     rt.RuntimeEventKind.RELEASE]
    held = cache.acquire(1)
    with pytest.raises(RuntimeError, match="active lease"):
        cache.cold_reset()
    with pytest.raises(RuntimeError, match="active lease"):
        cache.close()
    held.release()
    torch.cuda.synchronize()
    cache.cold_reset()
    assert cache.stats() == rt.ExpertCacheStats(0, 0, 0, 0, 0)
    assert cache.snapshot().lru_sequence == 0
    cache.close()
    assert cache.closed and Owner.closed
    with pytest.raises(RuntimeError, match="closed"):
        cache.acquire(0)


def test_checkpoint_roundtrip(rt):
    cache = rt.GpuExpertCache(make_sources(), slot_count=2, device=DEV)
    for e in (0, 1):
        with cache.acquire(e) as lease:
            lease.wait()
    torch.cuda.synchronize()
    ckpt = cache._capture_checkpoint()
    with cache.acquire(2) as lease:
        lease.wait()
    torch.cuda.synchronize()
    assert cache.resident_expert_ids() == (1, 2)
    info = cache._restore_checkpoint(ckpt)
    assert info["weights_pinned"] and cache.resident_expert_ids() == (0, 1)
    with cache.acquire(0) as lease:
        w = lease.wait().clone()
    torch.cuda.synchronize()
    assert torch.equal(w.cpu(), make_sources()[0])


# ---------------------------------------------------------------- experts


def packed(gate, up, down):
    return torch.cat((gate.flatten(), up.flatten(), down.flatten()))


def test_canonical_output_invariant_to_execution_order(rt):
    hid, inter = 4, 3
    g = torch.Generator().manual_seed(29)
    gate_up = torch.randn(3, 2 * inter, hid, dtype=torch.bfloat16, generator=g)
    down = torch.randn(3, hid, inter, dtype=torch.bfloat16, generator=g)
    srcs = {rt.ExpertKey(0, e): packed(gate_up[e, :inter], gate_up[e, inter:], down[e]) for e in range(3)}
    x = torch.randn(2, hid, dtype=torch.bfloat16, generator=g).to(DEV)
    idx = torch.tensor([[0, 1, 2], [2, 0, 1]], device=DEV)
    w = torch.tensor([[0.5, 0.3, 0.2], [0.45, 0.35, 0.2]], dtype=torch.bfloat16, device=DEV)
    cache = rt.GpuExpertCache(srcs, slot_count=1, device=DEV)
    experts = rt.Qwen3OffloadedExperts(layer_id=0, cache=cache, hidden_size=hid, intermediate_size=inter)
    fwd = experts(x, idx, w, execution_order=(0, 1, 2))
    torch.cuda.synchronize()
    assert cache.resident_expert_ids() == (rt.ExpertKey(0, 2),)
    rev = experts(x, idx, w, execution_order=(2, 1, 0))
    torch.cuda.synchronize()
    assert cache.resident_expert_ids() == (rt.ExpertKey(0, 0),)
    assert torch.equal(fwd, rev)
    pk = {e: srcs[rt.ExpertKey(0, e)].float().numpy() for e in range(3)}
    ref = mo.moe_experts(x.float().cpu().numpy(), idx.cpu().numpy(), w.float().cpu().numpy(), pk, hid, inter, "bf16")
    np.testing.assert_allclose(fwd.float().cpu().numpy(), ref, rtol=1.6e-2, atol=1.6e-2)


def test_resident_first_events_and_stats(rt):
    hid, inter = 4, 3
    g = torch.Generator().manual_seed(101)
    srcs = {rt.ExpertKey(0, e): torch.randn(3 * hid * inter, dtype=torch.bfloat16, generator=g) for e in range(3)}
    x = torch.randn(2, hid, dtype=torch.bfloat16, generator=g).to(DEV)
    idx = torch.tensor([[0, 1, 2], [2, 0, 1]], device=DEV)
    w = torch.tensor([[0.5, 0.3, 0.2], [0.45, 0.35, 0.2]], dtype=torch.bfloat16, device=DEV)
    acq = {rt.RuntimeEventKind.H2D_SUBMIT, rt.RuntimeEventKind.RESIDENT_HIT}

    def case(policy, order=None):
        obs = rt.RecordingCacheTransitionObserver(f"rf-{policy}")
        cache = rt.GpuExpertCache(srcs, slot_count=2, device=DEV, observer=obs)
        for e in (1, 2):
            with cache.acquire(rt.ExpertKey(0, e)) as lease:
                lease.wait()
        torch.cuda.synchronize()
        obs.reset()
        kw = {} if policy is None else {"execution_policy": policy}
        ex = rt.Qwen3OffloadedExperts(layer_id=0, cache=cache, hidden_size=hid, intermediate_size=inter, **kw)
        before = cache.stats()
        out = ex(x, idx, w, execution_order=order)
        torch.cuda.synchronize()
        after = cache.stats()
        delta = tuple(getattr(after, f) - getattr(before, f)
                      for f in ("h2d_submissions", "resident_hits", "inflight_joins", "evictions"))
        events = tuple((ev.kind, ev.expert_id.expert_id) for ev in obs.events() if ev.kind in acq)
        return out, delta, events

    legacy, d_legacy, ev_legacy = case(None)
    resident, d_res, ev_res = case(rt.ExpertExecutionPolicy.RESIDENT_FIRST)
    explicit, d_exp, ev_exp = case(rt.ExpertExecutionPolicy.RESIDENT_FIRST, order=(0, 1, 2))
    assert [e for _, e in ev_legacy] == [0, 1, 2]
    assert ev_res == ((rt.RuntimeEventKind.RESIDENT_HIT, 1), (rt.RuntimeEventKind.RESIDENT_HIT, 2),
                      (rt.RuntimeEventKind.H2D_SUBMIT, 0))
    assert [e for _, e in ev_exp] == [0, 1, 2]
    assert d_legacy == (3, 0, 0, 3) and d_res == (1, 2, 0, 1) and d_exp == (3, 0, 0, 3)
    assert torch.equal(legacy, resident) and torch.equal(legacy, explicit)


def test_arrival_order_reduction_kat(rt):
    silu_one = F.silu(torch.tensor(1.0, dtype=torch.bfloat16)).item()
    srcs = {rt.ExpertKey(0, e): packed(torch.ones(1, 1, dtype=torch.bfloat16),
                                       torch.ones(1, 1, dtype=torch.bfloat16),
                                       torch.tensor([[v / silu_one]], dtype=torch.bfloat16))
            for e, v in enumerate((1.0, 2.0 ** -8, -1.0))}
    x = torch.ones(1, 1, dtype=torch.bfloat16, device=DEV)
    idx = torch.tensor([[0, 1, 2]], device=DEV)
    w = torch.ones(1, 3, dtype=torch.bfloat16, device=DEV)
    mk = lambda mode: rt.Qwen3OffloadedExperts(
        layer_id=0, cache=rt.GpuExpertCache(srcs, slot_count=1, device=DEV), hidden_size=1,
        intermediate_size=1, reduction_mode=mode)
    arrival = mk(rt.ReductionMode.ARRIVAL_ORDER)
    canonical = mk(rt.ReductionMode.CANONICAL)
    assert arrival(x, idx, w, execution_order=(0, 1, 2)).item() == 0.0
    assert canonical(x, idx, w, execution_order=(0, 2, 1)).item() == 0.0
    assert arrival(x, idx, w, execution_order=(0, 2, 1)).item() == 2.0 ** -8


def test_validation_messages(rt):
    srcs = {rt.ExpertKey(0, 0): torch.zeros(3 * 4 * 3, dtype=torch.bfloat16)}
    cache = rt.GpuExpertCache(srcs, slot_count=1, device=DEV)
    ex = rt.Qwen3OffloadedExperts(layer_id=0, cache=cache, hidden_size=4, intermediate_size=3)
    x = torch.zeros(2, 4, dtype=torch.bfloat16, device=DEV)
    i = torch.zeros(2, 1, dtype=torch.long, device=DEV)
    w = torch.ones(2, 1, device=DEV)
    with pytest.raises(ValueError, match=r"hidden_states width is 5, expected 4"):
        ex(torch.zeros(2, 5, dtype=torch.bfloat16, device=DEV), i, w)
    with pytest.raises(ValueError, match="torch.long"):
        ex(x, i.int(), w)
    with pytest.raises(ValueError, match="must match top_k_index shape"):
        ex(x, i, torch.ones(2, 2, device=DEV))
    with pytest.raises(ValueError, match="every active expert exactly once"):
        ex(x, i, w, execution_order=(0, 1))
    with pytest.raises(KeyError):
        ex(x, torch.full((2, 1), 3, dtype=torch.long, device=DEV), w)


@pytest.mark.parametrize("slots", [24, 128])
def test_full_layer_cache_paths_match_oracle(rt, slots):
    """H=2048, I=768, 128 experts, T=65: waves through a 24-slot cache and the
    fully resident path of a 128-slot cache give the same result as the
    oracle; stats count every active expert once."""
    from specfit_b200 import synthetic

    weights, x = synthetic.bf16_layer_inputs(seed=31, tokens=65)
    srcs = {rt.ExpertKey(3, e): weights.packed(e) for e in range(128)}
    cache = rt.GpuExpertCache(srcs, slot_count=slots, device=DEV)
    ex = rt.Qwen3OffloadedExperts(layer_id=3, cache=cache, hidden_size=2048, intermediate_size=768)
    if slots == 128:
        cache.prefill_all()
        torch.cuda.synchronize()
        cache.stats()
    rng = np.random.default_rng(3)
    idx_np = np.stack([rng.permutation(128)[:8] for _ in range(65)])
    w_np = rng.dirichlet(np.ones(8), size=65).astype(np.float32)
    before = cache.stats()
    out = ex(x.to(DEV), torch.from_numpy(idx_np).to(DEV), torch.from_numpy(w_np).to(DEV))
    torch.cuda.synchronize()
    after = cache.stats()
    n_active = len(np.unique(idx_np))
    hits = after.resident_hits - before.resident_hits
    subs = after.h2d_submissions - before.h2d_submissions
    assert hits + subs == n_active
    if slots == 128:
        assert subs == 0 and hits == n_active
    pk = {e: weights.packed(e).float().numpy() for e in np.unique(idx_np)}
    ref = mo.moe_experts(x.float().numpy(), idx_np, w_np, pk, 2048, 768, "bf16")
    got = out.float().cpu().numpy()
    assert np.abs(got - ref).max() <= 2e-2


@pytest.mark.parametrize("slots,experts,seed", [(4, 12, 0), (1, 3, 1), (6, 8, 2), (12, 12, 3)])
def test_cache_state_follows_the_lru_replay_oracle(rt, slots, experts, seed):
    """Access by access, the cache's fills, evictions and resident set equal
    the reference's logical LRU replay (src/specfit/replay.py:156-285,
    restated in oracle/cache_oracle.py) on Zipf-skewed random accesses."""
    from oracle.cache_oracle import LruLayer

    rng = np.random.default_rng(seed)
    weights = 1.0 / np.arange(1, experts + 1) ** 1.1
    seq = rng.choice(experts, size=150, p=weights / weights.sum())
    cache = rt.GpuExpertCache(make_sources(experts, shape=(8, 16), seed=seed), slot_count=slots, device=DEV)
    ref = LruLayer(slots)
    for i, e in enumerate(seq):
        with cache.acquire(int(e)) as lease:
            lease.wait()
        torch.cuda.synchronize()  # each fill lands before the next access, as in the replay
        ref.access(int(e))
        st = cache.stats()
        assert (st.h2d_submissions, st.resident_hits, st.evictions) == \
            (ref.h2d_submissions, ref.resident_hits, ref.evictions), i
        assert set(cache.resident_expert_ids()) == set(ref.resident()), i
    cache.close()


def test_reference_cache_off_edits_invalidate_the_cache(rt):
    """The reference's "0 slots" intervention edits private members in place
    (src/specfit/main_comparison_runtime.py:7-32: clear the resident and
    in-flight maps and the transfer queue, empty every slot, advance its
    generation, reset its last use, drop its ready event and use guards,
    bump the state version).  Those edits work on this cache's views, keep
    the counters, and make the next access a fill into an empty slot;
    ``invalidate_contents`` does the same in one call."""
    cache = rt.GpuExpertCache(make_sources(4), slot_count=2, device=DEV)
    try:
        for e in (0, 1):
            with cache.acquire(e) as lease:
                lease.wait()
        torch.cuda.synchronize()
        before = cache.stats()
        gens = [s.generation for s in cache._slots]
        version = cache._state_version
        with cache._lock:
            cache._require_checkpoint_boundary()
            cache._resident.clear()
            cache._inflight.clear()
            cache._outstanding_transfers.clear()
            for slot in cache._slots:
                slot.expert_id = None
                slot.generation += 1
                slot.last_used_sequence = 0
                slot.ready_event = None
                if slot.use_events is not None:
                    slot.use_events.clear()
            cache._state_version += 1
        assert cache._state_version > version
        assert cache.resident_expert_ids() == ()
        assert [s.generation for s in cache._slots] == [g + 1 for g in gens]
        assert all(s.expert_id is None and s.last_used_sequence == 0 for s in cache._slots)
        after = cache.stats()
        assert (after.h2d_submissions, after.resident_hits, after.evictions) == \
            (before.h2d_submissions, before.resident_hits, before.evictions)
        with cache.acquire(0) as lease:
            lease.wait()
        st = cache.stats()
        assert st.h2d_submissions == before.h2d_submissions + 1 and st.evictions == before.evictions
        torch.cuda.synchronize()
        cache.invalidate_contents()
        assert cache.resident_expert_ids() == ()
        with cache.acquire(3) as lease:
            lease.wait()
        assert cache.stats().evictions == before.evictions
    finally:
        cache.close()
