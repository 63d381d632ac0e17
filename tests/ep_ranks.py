"""Rank bodies for the multi-process expert-parallel tests (spawned workers).

``cpu_rank`` runs the whole expert-parallel flow of one MoE layer on CPU
ranks over gloo with the numpy restatement (oracle/ep_oracle.py) and checks
that each rank's output equals the single-process oracle block bit for bit.
``nccl_rank`` runs the CUDA path (specfit_b200.runtime.expert_parallel) on
one GPU per rank and checks it against the single-GPU CUDA block.
"""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def _init(rank: int, world: int, port: int, backend: str, device=None):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    kw = dict(device_id=device) if device is not None else {}
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=60), **kw)
    return dist


def cpu_case(seed: int, tokens_per_rank, num_experts: int, top_k: int, hidden: int, inter: int):
    """Seeded global inputs, identical on every rank: bf16-representable
    hidden states [T, H] and packed experts, distinct top-k ids, fp32 weights."""
    from oracle import moe_oracle as mo

    rng = np.random.default_rng(seed)
    T = int(sum(tokens_per_rank))
    x = mo.bf16_round(rng.normal(0, 1, size=(T, hidden)).astype(np.float32))
    idx = np.stack([rng.permutation(num_experts)[:top_k] for _ in range(T)]).astype(np.int64).reshape(T, top_k)
    w = rng.uniform(0.05, 1.0, size=(T, top_k)).astype(np.float32)
    packed = {e: mo.bf16_round(rng.normal(0, 0.05, size=3 * hidden * inter).astype(np.float32))
              for e in range(num_experts)}
    return x, idx, w, packed


def bf16_bytes(x: np.ndarray) -> np.ndarray:
    """Raw bf16 bytes of bf16-representable float32 values [T, H] -> [T, 2H]."""
    bits = (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    return bits.view(np.uint8).reshape(x.shape[0], 2 * x.shape[1])


def bf16_values(b: np.ndarray, hidden: int) -> np.ndarray:
    bits = np.ascontiguousarray(b[:, : 2 * hidden]).view(np.uint16).astype(np.uint32) << 16
    return bits.view(np.float32).reshape(b.shape[0], hidden)


def cpu_rank(rank: int, world: int, port: int, seed: int, tokens_per_rank, num_experts: int,
             top_k: int, hidden: int, inter: int) -> None:
    import torch

    from oracle import ep_oracle as ep
    from oracle import moe_oracle as mo

    dist = _init(rank, world, port, "gloo")
    try:
        x, idx, w, packed = cpu_case(seed, tokens_per_rank, num_experts, top_k, hidden, inter)
        lo = int(sum(tokens_per_rank[:rank]))
        hi = lo + int(tokens_per_rank[rank])
        per = num_experts // world

        # 1. source: one row per (token, destination rank)
        rows, counts, route_row = ep.send_pack(bf16_bytes(x[lo:hi]), idx[lo:hi], w[lo:hi],
                                               num_experts, world)
        send_counts = torch.from_numpy(counts.copy())
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts)
        sp, sr = counts[:, 0].tolist(), counts[:, 1].tolist()
        rp, rr = recv_counts[:, 0].tolist(), recv_counts[:, 1].tolist()
        recv = torch.empty(sum(rp), rows.shape[1], dtype=torch.uint8)
        dist.all_to_all_single(recv, torch.from_numpy(rows), output_split_sizes=rp, input_split_sizes=sp)
        recv = recv.numpy()

        # 2. destination: group by local expert, expert forward, weight, return rows
        counts_l, offsets, order, return_src = ep.recv_group(recv, 2 * hidden, top_k, per)
        assert int(counts_l.sum()) == sum(rr) == return_src.size
        _, ws = ep.unpack_meta(recv, 2 * hidden, top_k)
        xs = bf16_values(recv, hidden)
        ys = np.zeros((order.size, hidden), dtype=np.float32)
        for le in range(per):
            a, b = offsets[le], offsets[le + 1]
            if a == b:
                continue
            pos = order[a:b]
            y = mo.expert_forward(xs[pos // top_k], packed[rank * per + le], hidden, inter, "bf16")
            ys[a:b] = mo.weight_rows(y, ws.reshape(-1)[pos], "bf16")
        ret = torch.from_numpy(np.ascontiguousarray(ys[return_src]))
        back = torch.empty(sum(sr), hidden, dtype=torch.float32)
        dist.all_to_all_single(back, ret, output_split_sizes=sr, input_split_sizes=rr)
        back = back.numpy()

        # 3. source: the single-GPU combine order (ascending expert id)
        out = np.zeros((hi - lo, hidden), dtype=np.float32)
        for t in range(hi - lo):
            for k in np.argsort(idx[lo + t], kind="stable"):
                out[t] = mo.bf16_round((out[t] + back[route_row[t * top_k + k]]).astype(np.float32))

        want = mo.moe_experts(x, idx, w, packed, hidden, inter, "bf16")[lo:hi]
        assert np.array_equal(out, want), f"rank {rank}: expert-parallel output differs"
    finally:
        dist.destroy_process_group()


def nccl_rank(rank: int, world: int, port: int, seed: int, tokens_per_rank) -> None:
    import torch

    from specfit_b200 import ops, synthetic
    from specfit_b200.runtime.expert_parallel import ExpertParallelMoE

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist = _init(rank, world, port, "nccl", device)
    try:
        E, K, H, I = 128, 8, 2048, 768
        g = torch.Generator(device="cpu").manual_seed(seed)
        T = int(sum(tokens_per_rank))
        x = (torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16).to(device)
        idx = torch.from_numpy(synthetic.zipf_routes(T, 0, seed)).to(device)
        w = torch.rand(T, K, generator=g).to(device)
        gd = torch.Generator(device=device).manual_seed(seed)
        storage = (torch.randn(E, 3 * H * I, generator=gd, device=device) * 0.02).to(torch.bfloat16)
        per = E // world
        lo = int(sum(tokens_per_rank[:rank]))
        hi = lo + int(tokens_per_rank[rank])
        moe = ExpertParallelMoE(num_experts=E, top_k=K, hidden_size=H, intermediate_size=I,
                                local_storage=storage[rank * per:(rank + 1) * per], rank=rank,
                                world=world)
        got = moe.forward(x[lo:hi], idx[lo:hi], w[lo:hi])
        from specfit_b200.runtime.ep_peer import PeerExchange

        peer = PeerExchange(rank=rank, world=world, max_tokens=max(tokens_per_rank), hidden_size=H,
                            top_k=K, local_experts=per, device=device)
        moe.peer, moe.use_peer = peer, True
        got_peer = [moe.forward(x[lo:hi], idx[lo:hi], w[lo:hi]) for _ in range(3)]
        torch.cuda.synchronize()
        peer.check()
        d = ops.moe_dispatch(idx, E)
        xs, ws = ops.moe_gather(x, w, d)
        slot = torch.arange(E, dtype=torch.int32, device=device)
        ys = ops.grouped_swiglu(xs, ws, d, slot, storage, H, I)
        want = ops.moe_combine(ys, d, idx)[lo:hi]
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"rank {rank}: NCCL expert-parallel output differs"
        for gp in got_peer:
            assert torch.equal(gp, want), f"rank {rank}: peer-memory expert-parallel output differs"
        peer.close()
    finally:
        dist.destroy_process_group()
