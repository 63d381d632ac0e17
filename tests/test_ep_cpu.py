"""Expert-parallel exchange on CPU ranks (gloo), no GPU.

* The numpy restatement of the send plan keeps every route exactly once,
  groups rows by destination then token, and sorts each row's local ids.
* 2 and 4 gloo ranks with ragged token counts (one rank with no tokens)
  run the whole exchange — count all-to-all, row all-to-all, per-expert
  forward on the owner, return all-to-all, combine — and each rank's output
  equals the single-process oracle MoE block bit for bit."""
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import ep_ranks
from oracle import ep_oracle as ep


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_send_plan_invariants(world):
    rng = np.random.default_rng(world)
    T, E, K, hb = 37, 16, 4, 64
    idx = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int64)
    w = rng.uniform(size=(T, K)).astype(np.float32)
    hidden = rng.integers(0, 256, size=(T, hb), dtype=np.uint8)
    rows, counts, route_row = ep.send_pack(hidden, idx, w, E, world)
    per = E // world
    assert counts[:, 1].sum() == T * K
    assert sorted(route_row.tolist()) == list(range(T * K))  # a permutation of the return rows
    ids, ws = ep.unpack_meta(rows, hb, K)
    i = 0
    for r in range(world):
        toks = [t for t in range(T) if (idx[t] // per == r).any()]
        assert counts[r, 0] == len(toks)
        for t in toks:
            mine = sorted(int(e) - r * per for e in idx[t] if e // per == r)
            assert ids[i, :len(mine)].tolist() == mine and (ids[i, len(mine):] == -1).all()
            assert np.array_equal(rows[i, :hb], hidden[t])
            i += 1


def test_recv_group_is_stable():
    rng = np.random.default_rng(3)
    T, E, K, hb = 20, 8, 3, 32
    idx = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int64)
    rows, counts, _ = ep.send_pack(np.zeros((T, hb), np.uint8), idx, np.ones((T, K), np.float32), E, 2)
    mine = rows[: counts[0, 0]]
    cnt, off, order, ret = ep.recv_group(mine, hb, K, E // 2)
    ids, _ = ep.unpack_meta(mine, hb, K)
    flat = ids.reshape(-1)
    for e in range(E // 2):
        pos = order[off[e]:off[e + 1]]
        assert (flat[pos] == e).all() and (np.diff(pos) > 0).all()
    assert sorted(ret.tolist()) == list(range(int(cnt.sum())))


@pytest.mark.parametrize("world,tokens", [(2, [7, 5]), (4, [6, 0, 9, 3])])
def test_gloo_ranks_equal_single_process_block(world, tokens):
    mp.start_processes(ep_ranks.cpu_rank, args=(world, free_port(), 11, tokens, 16, 4, 64, 32),
                       nprocs=world, join=True, start_method="spawn")
