"""Seeded synthetic inputs for the verification-path workloads.

No dataset or checkpoint is used anywhere: weights are random-init with the
Qwen3-30B-A3B shapes, tokens are uniform over the vocabulary, and trees and
routes come from fixed seeds.  Generation order is part of the contract (the
committed golden fixtures were produced from exactly these draws), so do not
reorder draws.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

# Qwen3-30B-A3B shapes (the reference's target model).
HIDDEN = 2048
NUM_EXPERTS = 128
TOP_K = 8
MOE_INTER = 768
NUM_LAYERS = 48
NUM_HEADS = 32
NUM_KV_HEADS = 4
HEAD_DIM = 128
VOCAB = 151936
ROPE_THETA = 1.0e6
RMS_EPS = 1.0e-6


@dataclass(frozen=True)
class MoeLayerWeights:
    router: torch.Tensor  # [E, H]
    gate_up: torch.Tensor  # [E, 2I, H]
    down: torch.Tensor  # [E, H, I]

    def packed(self, expert: int) -> torch.Tensor:
        """One packed slot ``[gate | up | down]`` flattened (the packed-v1
        expert row, ``adapters/qwen3_packed_checkpoint.py:20-23``)."""
        inter = self.down.shape[2]
        return torch.cat(
            (
                self.gate_up[expert, :inter].reshape(-1),
                self.gate_up[expert, inter:].reshape(-1),
                self.down[expert].reshape(-1),
            )
        )

    def packed_all(self) -> torch.Tensor:
        """``[E, 3*H*I]`` packed slots."""
        return torch.stack([self.packed(e) for e in range(self.router.shape[0])])


def config1_inputs(seed: int = 0, tokens: int = 32):
    """Configuration 1: one MoE block in fp32.

    ``torch.Generator().manual_seed(seed)``; draws, in this order,
    ``W_router[128,2048]``, ``W_gate_up[128,1536,2048]``, ``W_down[128,2048,768]``
    (all N(0,1)*0.02, fp32), then ``x[tokens,2048]`` N(0,1).
    """
    g = torch.Generator().manual_seed(seed)
    router = torch.randn(NUM_EXPERTS, HIDDEN, generator=g) * 0.02
    gate_up = torch.randn(NUM_EXPERTS, 2 * MOE_INTER, HIDDEN, generator=g) * 0.02
    down = torch.randn(NUM_EXPERTS, HIDDEN, MOE_INTER, generator=g) * 0.02
    x = torch.randn(tokens, HIDDEN, generator=g)
    return MoeLayerWeights(router, gate_up, down), x


def bf16_layer_inputs(seed: int, tokens: int, hidden: int = HIDDEN, experts: int = NUM_EXPERTS,
                      inter: int = MOE_INTER, x_scale: float = 1.0):
    """One bf16 MoE layer: N(0,0.02) weights and N(0,1)*x_scale inputs.

    Draw order: router, gate_up, down, x (each fp32 then cast to bf16)."""
    g = torch.Generator().manual_seed(seed)
    router = (torch.randn(experts, hidden, generator=g) * 0.02).to(torch.bfloat16)
    gate_up = (torch.randn(experts, 2 * inter, hidden, generator=g) * 0.02).to(torch.bfloat16)
    down = (torch.randn(experts, hidden, inter, generator=g) * 0.02).to(torch.bfloat16)
    x = (torch.randn(tokens, hidden, generator=g) * x_scale).to(torch.bfloat16)
    return MoeLayerWeights(router, gate_up, down), x


def zipf_routes(tokens: int, layer: int, seed: int, experts: int = NUM_EXPERTS,
                top_k: int = TOP_K, s: float = 1.1) -> np.ndarray:
    """Configurations 3 and 5: per-layer Zipf(s) routes.

    ``perm = randperm(experts)`` seeded by ``seed*1000+layer``; the expert of
    rank r (1-based) has weight r**-s; each token draws ``top_k`` distinct
    experts by Gumbel-top-k (sampling without replacement).  Returns
    ``int64[tokens, top_k]`` in draw order."""
    rng = np.random.default_rng(seed * 1000 + layer)
    perm = rng.permutation(experts)
    ranks = np.empty(experts, dtype=np.float64)
    ranks[perm] = np.arange(1, experts + 1)
    logw = -s * np.log(ranks)
    gumbel = rng.gumbel(size=(tokens, experts))
    keys = logw[None, :] + gumbel
    return np.argsort(-keys, axis=1, kind="stable")[:, :top_k].astype(np.int64)


def random_tree(num_nodes: int, max_depth: int, max_branch: int, seed: int, vocab: int = VOCAB):
    """Deterministic synthetic draft tree.

    Parents precede children (1-based ids, 0 = the pending seed), depth <=
    ``max_depth``, at most ``max_branch`` children per node, distinct sibling
    tokens: the invariants ``Eagle3DraftTree`` validates
    (``runtime/eagle3_types.py:336-400``).  Later nodes are preferred as
    parents so the tree reaches its depth.  Returns
    ``(token_ids, parent_ids, depths)``."""
    rng = np.random.default_rng(seed)
    parents: list = []
    depths: list = []
    tokens: list = []
    child_count = {0: 0}
    node_depth = {0: 0}
    sibling_tokens: dict = {0: set()}
    while len(parents) < num_nodes:
        candidates = [n for n in range(len(parents) + 1)
                      if node_depth[n] < max_depth and child_count[n] < max_branch]
        if not candidates:
            raise ValueError("tree shape cannot hold that many nodes")
        weights = np.array([1.0 + n for n in candidates], dtype=np.float64)
        parent = int(rng.choice(candidates, p=weights / weights.sum()))
        node = len(parents) + 1
        token = int(rng.integers(0, vocab))
        while token in sibling_tokens[parent]:
            token = int(rng.integers(0, vocab))
        sibling_tokens[parent].add(token)
        parents.append(parent)
        depths.append(node_depth[parent] + 1)
        tokens.append(token)
        child_count[parent] += 1
        child_count[node] = 0
        node_depth[node] = node_depth[parent] + 1
        sibling_tokens[node] = set()
    return tuple(tokens), tuple(parents), tuple(depths)


# Natural-cache coefficients of the reference's frozen A100 selection model
# (per node count 0..7, ns; and ns per distinct (layer, expert) in the
# verification footprint), used as realistic synthetic cost models.
SELECTION_INTERCEPT_NS = (142213640.2719444, 147532305.64501184, 150522238.9747455,
                          152268786.28951707, 152742629.59439692, 163203998.73306817,
                          155175323.9989069, 156067696.05019823)
SELECTION_EXPERT_NS = 210715.51267433458
# Mean pass time per node count of the same (natural, legacy) model.
SELECTION_SIZE_MEAN_NS = (223128397.1388889, 274429869.9444444, 306112232.25, 334490879.0833333,
                          357604933.5833333, 389313450.25, 394875926.0833333, 410155485.0833333)


@dataclass(frozen=True)
class SelectionCase:
    parents: tuple      # parent raw id of raw = 1..n (0 = the seed)
    depths: tuple
    cum_logp: tuple     # cumulative log-probability of raw = 1..n
    routes: np.ndarray  # int64 [n + 1, 48, 8]: top-8 experts of raw 0..n per layer
    resident: np.ndarray  # bool [48, 128]


def selection_case(seed: int, nodes: int, *, shared_routes: bool = False, level_prob=None,
                   resident_frac: float = 0.3) -> SelectionCase:
    """A top-2 draft pool like the reference's (2 nodes at depth 1, then 4 per
    level whose parents are 2 distinct nodes of the previous level), random
    conditional probabilities (or ``level_prob`` = (p_odd_raw, p_even_raw)),
    per-(raw, layer) top-8 routes of distinct experts (or experts 0..7 for
    every raw when ``shared_routes``), and a random resident set (at most 48
    experts per layer)."""
    rng = np.random.default_rng(seed)
    parents, depths = [0, 0], [1, 1]
    prev = [1, 2]
    while len(parents) < nodes:
        chosen = sorted(rng.choice(prev, size=2, replace=False).tolist())
        level = []
        for par in chosen:
            for _ in range(2):
                parents.append(int(par))
                depths.append(depths[par - 1] + 1)
                level.append(len(parents))
        prev = level
    parents, depths = parents[:nodes], depths[:nodes]
    cum = []
    for raw, par in enumerate(parents, start=1):
        if level_prob is None:
            cond = float(np.log(rng.uniform(0.05, 0.95)))
        else:
            cond = float(np.log(level_prob[0] if raw % 2 else level_prob[1]))
        cum.append((0.0 if par == 0 else cum[par - 1]) + cond)
    if shared_routes:
        routes = np.broadcast_to(np.arange(8), (nodes + 1, 48, 8)).copy()
    else:
        routes = np.stack([np.stack([rng.permutation(128)[:8] for _ in range(48)])
                           for _ in range(nodes + 1)])
    resident = np.zeros((48, 128), dtype=bool)
    for layer in range(48):
        count = int(min(48, rng.binomial(128, resident_frac)))
        resident[layer, rng.permutation(128)[:count]] = True
    return SelectionCase(tuple(parents), tuple(depths), tuple(cum), routes.astype(np.int64), resident)


def token_routes(tokens, layers: int = NUM_LAYERS, *, experts: int = NUM_EXPERTS, top_k: int = TOP_K,
                 s: float = 1.1, seed: int = 0):
    """Configuration 4: a token's route at every layer, Zipf(s) over experts
    under a per-layer permutation, ``top_k`` distinct experts drawn by
    Gumbel-top-k whose uniforms are a hash of (seed, layer, token, expert).
    The same token always takes the same route, so a drafted candidate's
    expert footprint is known before it is verified.  ``tokens``: int64
    tensor ``[n]`` on any device; returns int64 ``[n, layers, top_k]`` on
    that device."""
    dev = tokens.device
    t = tokens.to(torch.int64).reshape(-1, 1, 1)
    l = torch.arange(layers, device=dev, dtype=torch.int64).reshape(1, -1, 1)
    e = torch.arange(experts, device=dev, dtype=torch.int64).reshape(1, 1, -1)
    mask = (1 << 62) - 1
    x = ((seed * 1_000_003 + l) * 1_000_033 + t) * 131 + e
    # multiply-xorshift mixing kept below 2**62, so int64 never overflows
    for mult, shift in ((0x1CE4E5B9, 29), (0x133111EB, 31), (0x2545F491, 27)):
        x = (x * mult) & mask
        x = x ^ (x >> shift)
    u = ((x & ((1 << 52) - 1)).to(torch.float64) + 0.5) / float(1 << 52)
    gumbel = -torch.log(-torch.log(u))
    key = (layers, experts, float(s), seed, str(dev))
    logw = _ZIPF_LOGW.get(key)
    if logw is None:
        rng = np.random.default_rng(seed * 7919 + 17)
        perms = np.stack([rng.permutation(experts) for _ in range(layers)])
        ranks = np.empty((layers, experts), dtype=np.float64)
        for li in range(layers):
            ranks[li, perms[li]] = np.arange(1, experts + 1)
        logw = _ZIPF_LOGW[key] = torch.from_numpy(-s * np.log(ranks)).to(dev).unsqueeze(0)
    return torch.topk(logw + gumbel, top_k, dim=-1).indices


_ZIPF_LOGW: dict = {}  # (layers, experts, s, seed, device) -> per-layer Zipf log-weights
