"""Expert-parallel MoE block on the GPU (K7).

* ``sf_ep_send_pack`` writes the same rows, counts and route rows as the
  numpy restatement (byte for byte) for 1-8 ranks, including no tokens.
* ``sf_ep_recv_group`` groups received slots exactly like the restatement.
* W ranks emulated on one GPU (each rank's send / compute / combine phases,
  the all-to-all done by slicing) reproduce the single-GPU MoE block bit for
  bit at the Qwen3-30B-A3B expert shape, with ragged and empty ranks.
* With two or more GPUs, the NCCL path on two ranks does the same."""
import socket

import numpy as np
import pytest
import torch

from oracle import ep_oracle as ep
from specfit_b200 import ops, synthetic
from specfit_b200.runtime.expert_parallel import ExpertParallelMoE

pytestmark = pytest.mark.gpu

E, K, H, I = 128, 8, 2048, 768


def _routes(T, seed):
    return torch.from_numpy(synthetic.zipf_routes(T, 0, seed)).cuda()


@pytest.mark.parametrize("world,T,wdt", [(1, 33, torch.float32), (2, 65, torch.float32),
                                         (4, 130, torch.bfloat16), (8, 512, torch.float32),
                                         (8, 0, torch.float32)])
def test_send_pack_matches_restatement(world, T, wdt):
    g = torch.Generator(device="cuda").manual_seed(T + world)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    idx = _routes(T, world)
    w = torch.rand(T, K, generator=g, device="cuda").to(wdt)
    s = ops.ep_send_pack(x, idx, w, E, world)
    torch.cuda.synchronize()
    assert int(s.error.item()) == 0
    hb = x.view(torch.uint8).reshape(T, 2 * H).cpu().numpy() if T else np.zeros((0, 2 * H), np.uint8)
    rows, counts, route_row = ep.send_pack(hb, idx.cpu().numpy(), w.float().cpu().numpy(), E, world)
    assert np.array_equal(s.counts.cpu().numpy(), counts)
    P = int(counts[:, 0].sum())
    assert np.array_equal(s.rows[:P].cpu().numpy(), rows)
    assert np.array_equal(s.route_row.cpu().numpy(), route_row)


def test_send_pack_flags_invalid_expert():
    x = torch.zeros(4, H, dtype=torch.bfloat16, device="cuda")
    idx = _routes(4, 1)
    idx[2, 3] = E  # out of range
    s = ops.ep_send_pack(x, idx, torch.ones(4, K, device="cuda"), E, 2)
    torch.cuda.synchronize()
    assert int(s.error.item()) == 1
    assert int(s.route_row[2 * K + 3].item()) == -1
    assert int(s.counts[:, 1].sum().item()) == 4 * K - 1


@pytest.mark.parametrize("world", [2, 8])
def test_recv_group_matches_restatement(world):
    T = 97
    g = torch.Generator(device="cuda").manual_seed(world)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    idx = _routes(T, 5)
    w = torch.rand(T, K, generator=g, device="cuda")
    hb = x.view(torch.uint8).reshape(T, 2 * H).cpu().numpy()
    # Three "sources" with different token slices all send to rank 1.
    cuts = [0, 40, 41, T]
    blocks = []
    for a, b in zip(cuts[:-1], cuts[1:]):
        rows, counts, _ = ep.send_pack(hb[a:b], idx[a:b].cpu().numpy(), w[a:b].cpu().numpy(), E, world)
        off = int(counts[:1, 0].sum())
        blocks.append(rows[off: off + int(counts[1, 0])])
    recv = np.concatenate(blocks)
    per = E // world
    cnt, offs, order, ret = ep.recv_group(recv, 2 * H, K, per)
    d, return_src = ops.ep_recv_group(torch.from_numpy(recv).cuda(), recv.shape[0], H, K, per,
                                      torch.bfloat16)
    torch.cuda.synchronize()
    R = int(cnt.sum())
    assert int(d.error.item()) == 0
    assert np.array_equal(d.counts.cpu().numpy(), cnt)
    assert np.array_equal(d.offsets.cpu().numpy(), offs)
    assert np.array_equal(d.sorted_pos[:R].cpu().numpy(), order)
    assert np.array_equal(return_src[:R].cpu().numpy(), ret)


def _single_gpu_block(x, idx, w, storage):
    d = ops.moe_dispatch(idx, E)
    xs, ws = ops.moe_gather(x, w, d)
    slot = torch.arange(E, dtype=torch.int32, device=x.device)
    ys = ops.grouped_swiglu(xs, ws, d, slot, storage, H, I)
    return ops.moe_combine(ys, d, idx)


@pytest.fixture(scope="module")
def expert_storage():
    g = torch.Generator(device="cuda").manual_seed(7)
    return (torch.randn(E, 3 * H * I, generator=g, device="cuda") * 0.02).to(torch.bfloat16)


@pytest.mark.parametrize("world,tokens", [(1, [65]), (2, [65, 64]), (4, [30, 0, 65, 1]),
                                          (8, [64] * 8)])
def test_emulated_ranks_equal_single_gpu(world, tokens, expert_storage):
    T = sum(tokens)
    g = torch.Generator(device="cuda").manual_seed(world)
    x = (torch.randn(T, H, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    idx = _routes(T, 3 + world)
    w = torch.rand(T, K, generator=g, device="cuda")
    want = _single_gpu_block(x, idx, w, expert_storage)
    per = E // world
    ranks = [ExpertParallelMoE(num_experts=E, top_k=K, hidden_size=H, intermediate_size=I,
                               local_storage=expert_storage[r * per:(r + 1) * per], rank=r,
                               world=world) for r in range(world)]
    cuts = np.concatenate([[0], np.cumsum(tokens)]).astype(int)
    sends = [ranks[r].send(x[cuts[r]:cuts[r + 1]], idx[cuts[r]:cuts[r + 1]], w[cuts[r]:cuts[r + 1]])
             for r in range(world)]
    counts = [s.counts.cpu().numpy() for s in sends]  # [src][dst] -> (pairs, routes)
    pair_off = [np.concatenate([[0], np.cumsum(c[:, 0])]) for c in counts]
    outs = []
    for dst in range(world):
        recv = torch.cat([sends[src].rows[pair_off[src][dst]: pair_off[src][dst + 1]]
                          for src in range(world)])
        pairs = sum(int(counts[src][dst, 0]) for src in range(world))
        routes = sum(int(counts[src][dst, 1]) for src in range(world))
        outs.append(ranks[dst].compute(recv, pairs, routes, torch.bfloat16))
    # route offsets of each source's block inside each destination's output
    got = []
    for src in range(world):
        parts = []
        for dst in range(world):
            before = sum(int(counts[s][dst, 1]) for s in range(src))
            parts.append(outs[dst][before: before + int(counts[src][dst, 1])])
        returned = torch.cat(parts)
        got.append(ranks[src].combine(returned, sends[src], idx[cuts[src]:cuts[src + 1]]))
    got = torch.cat(got)
    torch.cuda.synchronize()
    assert all(int(s.error.item()) == 0 for s in sends)
    assert torch.equal(got, want)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_two_ranks_equal_single_gpu():
    import torch.multiprocessing as mp

    import ep_ranks

    mp.start_processes(ep_ranks.nccl_rank, args=(2, _free_port(), 21, [65, 40]), nprocs=2, join=True,
                       start_method="spawn")


def test_one_rank_ep_model_equals_single_gpu_model():
    """A one-rank expert-parallel verifier (2 layers) gives the same logits,
    bit for bit, as the single-GPU verifier with every expert resident."""
    from transformers import DynamicCache

    from specfit_b200.runtime.ep_verifier import build_random_ep_qwen3
    from specfit_b200.runtime.qwen3_verifier import build_random_offloaded_qwen3, qwen3_moe_config

    dev = torch.device("cuda", 0)
    cfg = qwen3_moe_config(2)
    single = build_random_offloaded_qwen3(device=dev, slots_per_layer=E, config=cfg, seed=3)
    single.warm_all_caches()
    epm = build_random_ep_qwen3(device=dev, rank=0, world=1, config=qwen3_moe_config(2), seed=3)
    gen = torch.Generator().manual_seed(4)
    ids = torch.randint(0, cfg.vocab_size, (2, 40), generator=gen).to(dev)
    outs = []
    for model in (single.model, epm.model):
        cache = DynamicCache(config=cfg)
        with torch.no_grad():
            outs.append(model(input_ids=ids, past_key_values=cache, use_cache=True).logits)
    single.close()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("fused_return", [True, False])
@pytest.mark.parametrize("tokens", [65, 520, 0])
def test_peer_exchange_one_rank_equals_single_gpu(tokens, fused_return, expert_storage):
    """The peer-memory exchange run with oneself (push, bounded wait,
    grouping, gather, SwiGLU, return, wait, combine) gives the single-GPU
    block bit for bit, repeatedly (arrival counters advance per layer) —
    with the return stored by the SwiGLU's epilogue and with the separate
    return kernel."""
    from specfit_b200.runtime.ep_peer import PeerExchange

    g = torch.Generator(device="cuda").manual_seed(tokens)
    moe = ExpertParallelMoE(num_experts=E, top_k=K, hidden_size=H, intermediate_size=I,
                            local_storage=expert_storage, rank=0, world=1)
    peer = PeerExchange(rank=0, world=1, max_tokens=520, hidden_size=H, top_k=K, local_experts=E,
                        device="cuda", fused_return=fused_return)
    moe.peer, moe.use_peer = peer, True
    try:
        for rep in range(3):
            x = (torch.randn(tokens, H, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
            idx = _routes(tokens, rep)
            w = torch.rand(tokens, K, generator=g, device="cuda")
            got = moe.forward(x, idx, w)
            want = _single_gpu_block(x, idx, w, expert_storage) if tokens else got
            torch.cuda.synchronize()
            assert torch.equal(got, want)
        assert peer.status() == (0, 0)
        assert int(peer._ticket.item()) == 0  # every fused launch leaves its ticket at zero
    finally:
        peer.close()


def test_peer_wait_gives_up_and_reports():
    """A receive wait whose arrivals never come (no push was issued) returns
    after its limit with the site and the missing rank recorded; the GPU
    stays usable."""
    import ctypes

    from specfit_b200 import _native as N
    from specfit_b200.runtime.ep_peer import PeerExchange

    peer = PeerExchange(rank=0, world=1, max_tokens=8, hidden_size=H, top_k=K, local_experts=16,
                        device="cuda", wait_limit_ms=100)
    try:
        n = peer.desc.cap_pairs * K
        i32 = torch.zeros(16 + 17 + 3 * n + 16 + 2, dtype=torch.int32, device="cuda")
        xs = torch.empty(peer.desc.cap_routes, H, dtype=torch.bfloat16, device="cuda")
        ws = torch.empty(peer.desc.cap_routes, dtype=torch.float32, device="cuda")
        p = i32.data_ptr()
        ptr = lambda off: p + 4 * off
        rc = N.lib.sf_ep_peer_recv(ctypes.byref(peer.desc), ptr(0), ptr(16), ptr(33), ptr(33 + n),
                                   ptr(33 + 3 * n), ptr(33 + 3 * n + 16), ptr(33 + 2 * n),
                                   ptr(33 + 3 * n + 17), xs.data_ptr(), ws.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream)
        assert rc == N.SF_OK
        torch.cuda.synchronize()
        assert peer.status() == (1, 1)
        with pytest.raises(RuntimeError, match="receive wait gave up"):
            peer.check()
        assert torch.ones(4, device="cuda").sum().item() == 4.0  # the context is fine
    finally:
        peer.close()
