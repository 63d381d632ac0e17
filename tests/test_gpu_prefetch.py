"""Predicted cross-layer prefetch (``Qwen3ExpertPrefetch``, a9) on the GPU.

Scenarios follow the reference's own GPU tests of the scheduler
(tests/gpu/test_qwen3_expert_prefetch.py, test_qwen3_probability_prefetch.py):
outputs bit-identical to the plain forward for right, wrong, missing and
repeated predictions at every slot count and lookahead; real misses are
submitted before ready experts are computed; predictions start before the
first attention; streams, hooks and leases are restored, also on errors;
bad configurations fail before touching a cache; probability eviction."""
from types import SimpleNamespace

import pytest
import torch
from torch import nn

from specfit_b200.runtime import ExpertKey, GpuExpertCache, Qwen3OffloadedExperts
from specfit_b200.runtime.qwen3_verifier import LoadedOffloadedQwen3

pytestmark = pytest.mark.gpu

H, I, E = 16, 12, 6


class _Attention(nn.Module):
    def forward(self, hidden):
        return hidden.clone()


class _Model(nn.Module):
    """Layers of (attention stand-in, offloaded experts), as the scheduler sees
    a decoder: one ``self_attn`` pre-hook per layer, then ``mlp.experts``."""

    def __init__(self, experts):
        super().__init__()
        self.model = nn.Module()
        self.model.layers = nn.ModuleList()
        self.config = SimpleNamespace(num_hidden_layers=len(experts))
        for m in experts:
            layer = nn.Module()
            layer.self_attn = _Attention()
            layer.mlp = nn.Module()
            layer.mlp.experts = m
            self.model.layers.append(layer)

    def forward(self, hidden, idx, w):
        for layer in self.model.layers:
            hidden = layer.self_attn(hidden)
            hidden = layer.mlp.experts(hidden, idx, w)
        return hidden


def make_case(slots=3, layers=2, seed=909):
    g = torch.Generator().manual_seed(seed)
    caches, experts = [], []
    for lid in range(layers):
        sources = {ExpertKey(lid, e): torch.randn(3 * H * I, generator=g, dtype=torch.bfloat16) / 16
                   for e in range(E)}
        cache = GpuExpertCache(sources, slot_count=slots, device="cuda:0")
        caches.append(cache)
        experts.append(Qwen3OffloadedExperts(layer_id=lid, cache=cache, hidden_size=H,
                                             intermediate_size=I, h2d_prefetch=False))
    loaded = LoadedOffloadedQwen3(_Model(experts), tuple(caches), None)
    inputs = (torch.randn(4, H, generator=g, dtype=torch.bfloat16).cuda(),
              torch.tensor([[4, 0, 2], [1, 4, 3], [2, 0, 1], [4, 3, 0]], device="cuda:0"),
              torch.rand(4, 3, generator=g, dtype=torch.bfloat16).cuda())
    return loaded, inputs


def assert_restored(loaded, streams):
    torch.cuda.synchronize()
    for layer, cache, stream in zip(loaded.model.model.layers, loaded.expert_caches, streams):
        assert cache.copy_stream is stream
        assert layer.mlp.experts._prediction_scheduler is None
        snap = cache.snapshot()
        assert not snap.pending_transfers
        assert all(not s.active_leases and not s.pending_use_guards for s in snap.slots)


@pytest.mark.parametrize("slots", [1, 2, 3, 6])
def test_outputs_bitwise_for_any_prediction(slots):
    loaded, inputs = make_case(slots)
    try:
        expected = loaded.model(*inputs)
        streams = tuple(c.copy_stream for c in loaded.expert_caches)
        for prediction in ((), (0, 1, 2, 3, 4), (5,), (4, 0, 4, 2, 5)):
            for depth in (0, 1):
                loaded.cold_reset_expert_caches()
                with loaded.prefetch_experts({i: prediction for i in range(2)},
                                             lookahead_layers=depth, max_inflight=2) as sched:
                    actual = loaded.model(*inputs)
                assert torch.equal(actual, expected), (prediction, depth)
                assert_restored(loaded, streams)
                st = sched.stats()
                assert st["complete"] and st["peak_inflight"] <= 2
                for lid, row in enumerate(st["layers"]):
                    assert row["computed_experts"] == row["actual_experts"] == 5
                    assert row["ready_at_router"] + row["inflight_at_router"] + row["missing_at_router"] == 5
                    assert (row["prediction_copies"] + row["demand_copies"]
                            == loaded.expert_caches[lid].stats().h2d_submissions)
    finally:
        loaded.close()


@pytest.mark.parametrize("tokens", [0, 1, 4])
def test_repeated_noncontiguous_and_empty_inputs(tokens):
    for slots in (1, 6):
        loaded, (hidden, idx, w) = make_case(slots)
        try:
            idx[0, 2] = idx[0, 0]  # a repeated expert in one token
            inputs = tuple(t[:tokens].t().contiguous().t() for t in (hidden, idx, w))
            originals = tuple(t.clone() for t in inputs)
            expected = loaded.model(*inputs)
            streams = tuple(c.copy_stream for c in loaded.expert_caches)
            for depth in (0, 1):
                loaded.cold_reset_expert_caches()
                with loaded.prefetch_experts({0: (0, 4, 5), 1: (0, 4, 5)}, lookahead_layers=depth):
                    actual = loaded.model(*inputs)
                assert torch.equal(actual, expected)
                assert all(torch.equal(a, b) for a, b in zip(inputs, originals))
                assert_restored(loaded, streams)
        finally:
            loaded.close()


def test_real_misses_are_submitted_before_ready_experts_are_computed():
    loaded, inputs = make_case(slots=4, layers=1)
    try:
        cache = loaded.expert_caches[0]
        for e in (3, 4):
            with cache.acquire(ExpertKey(0, e)) as lease:
                lease.wait()
        torch.cuda.synchronize()
        with torch.cuda.stream(cache.copy_stream):
            torch.cuda._sleep(50_000_000)  # keep the next copies in flight
        with loaded.prefetch_experts({}, trace=True) as sched:
            loaded.model(*inputs)
        ev = sched.events()
        copies = [e for e in ev if e["action"] == "copy"]
        computed = [e for e in ev if e["action"] == "compute"]
        assert copies[0]["sequence"] < computed[0]["sequence"]
        assert [e["expert_id"] for e in computed[:2]] == [3, 4]  # the residents first
        assert all(not e["waited"] for e in computed[:2])
        assert {e["expert_id"] for e in computed} == set(range(5))
    finally:
        loaded.close()


def test_predictions_start_before_the_first_attention():
    loaded, inputs = make_case(slots=3)
    try:
        with loaded.prefetch_experts({0: (1, 2), 1: (3,)}, trace=True) as sched:
            first = sched.events()
            loaded.model(*inputs)
        assert [e["action"] for e in first[:1]] == ["prediction_available"]
        assert any(e["action"] == "copy" and e["prediction"] for e in first)
        actions = [e["action"] for e in sched.events()]
        assert actions.index("copy") < actions.index("attention")
    finally:
        loaded.close()


def test_exceptions_restore_streams_hooks_and_leases():
    loaded, (hidden, idx, w) = make_case(slots=3)
    try:
        streams = tuple(c.copy_stream for c in loaded.expert_caches)
        bad = idx.clone()
        bad[1, 1] = 99
        with pytest.raises(KeyError):
            with loaded.prefetch_experts({0: (0, 1, 2), 1: (3, 4)}):
                loaded.model(hidden, bad, w)
        assert_restored(loaded, streams)
        with pytest.raises(RuntimeError, match="exactly one complete target forward"):
            with loaded.prefetch_experts({0: (0,)}):
                pass
        assert_restored(loaded, streams)
        sched = loaded.prefetch_experts({})
        with sched:
            loaded.model(hidden, idx, w)
        with pytest.raises(RuntimeError, match="cannot be reused"):
            with sched:
                pass
    finally:
        loaded.close()


def test_invalid_configurations_fail_before_any_cache_change():
    loaded, inputs = make_case(slots=3)
    try:
        before = [c.stats() for c in loaded.expert_caches]
        cases = [
            (dict(predictions={0: (9,)}), ValueError, "invalid predicted expert"),
            (dict(predictions={5: (0,)}), ValueError, "outside the loaded model"),
            (dict(predictions={}, lookahead_layers=-1), ValueError, "lookahead_layers"),
            (dict(predictions={}, max_inflight=0), ValueError, "max_inflight"),
            (dict(predictions={}, max_prefetch_per_layer=-1), ValueError, "max_prefetch_per_layer"),
            (dict(predictions={}, eviction_policy="mru"), ValueError, "eviction_policy"),
            (dict(predictions={}, eviction_policy="probability"), ValueError, "requires prediction_probabilities"),
            (dict(predictions={0: (1,)}, prediction_probabilities={0: {1: 1.5}}), ValueError, "invalid expert probability"),
            (dict(predictions={0: (1, 2)}, prediction_probabilities={0: {1: 0.5}}), ValueError, "explicit probability"),
            (dict(predictions=[(0,)]), TypeError, "map layer IDs"),
        ]
        for kw, exc, msg in cases:
            preds = kw.pop("predictions")
            with pytest.raises(exc, match=msg):
                loaded.prefetch_experts(preds, **kw)
        assert [c.stats() for c in loaded.expert_caches] == before
        with loaded.prefetch_experts({}):
            with pytest.raises(RuntimeError, match="another predicted prefetch"):
                loaded.prefetch_experts({}).__enter__()
            with pytest.raises(RuntimeError, match="cannot switch execution policy"):
                loaded.set_expert_execution_policy("resident_first")
            loaded.model(*inputs)
    finally:
        loaded.close()


def test_probability_eviction_prefers_the_least_likely_resident():
    loaded, inputs = make_case(slots=3, layers=1)
    try:
        cache = loaded.expert_caches[0]
        for e in (0, 1, 2):  # fill every slot; LRU order 0, 1, 2
            with cache.acquire(ExpertKey(0, e)) as lease:
                lease.wait()
        torch.cuda.synchronize()
        probs = {0: {0: 0.9, 1: 0.1, 2: 0.8, 5: 0.5}}
        with loaded.prefetch_experts({0: (5,)}, prediction_probabilities=probs,
                                     eviction_policy="probability", trace=True) as sched:
            first = [e for e in sched.events() if e["action"] == "copy"]
            resident_after = set(cache.resident_expert_ids())
            loaded.model(*inputs)
        assert first and first[0]["expert_id"] == 5
        # expert 1 (p = 0.1) was replaced, not the least recently used expert 0 (p = 0.9)
        assert ExpertKey(0, 0) in resident_after and ExpertKey(0, 2) in resident_after
        assert ExpertKey(0, 1) not in resident_after
    finally:
        loaded.close()


def test_real_qwen3_logits_match_without_prefetch():
    """Two-layer Qwen3-MoE target (random weights): logits with predicted
    prefetch equal the plain forward's bit for bit."""
    from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3, qwen3_moe_config

    cfg = qwen3_moe_config(2, hidden=256, experts=16, top_k=4, moe_inter=128, heads=8, kv_heads=2,
                           head_dim=128, vocab=512)
    m = build_random_offloaded_qwen3(device="cuda:0", slots_per_layer=5, config=cfg, seed=4, std=0.05)
    try:
        ids = torch.randint(0, 512, (1, 24), generator=torch.Generator().manual_seed(3)).cuda()
        with torch.no_grad():
            plain = m.model(input_ids=ids).logits
            routes = {}
            hooks = [layer.mlp.gate.register_forward_hook(
                lambda mod, a, out, l=l: routes.__setitem__(l, sorted(set(out[2].reshape(-1).tolist()))))
                for l, layer in enumerate(m.model.model.layers)]
            m.model(input_ids=ids)
            for h in hooks:
                h.remove()
            for preds in ({l: tuple(r) for l, r in routes.items()}, {}, {0: (0, 1, 2), 1: (15,)}):
                m.cold_reset_expert_caches()
                with m.prefetch_experts(preds, lookahead_layers=1, max_inflight=2) as sched:
                    got = m.model(input_ids=ids).logits
                assert torch.equal(got, plain)
                assert sched.stats()["complete"]
    finally:
        m.close()
