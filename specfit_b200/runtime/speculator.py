"""End-to-end speculative decoding: draft, SpecFit selection, verify, commit.

The cycle of ``ShallowTreeSpeculator._generate``
(``src/specfit/runtime/eagle3_tree.py:963-1500``) with an explicit
candidate-pool selector, on the B200 path:

1. the drafter builds a candidate pool from the committed tokens, their
   target features (hidden states of the target's layers 1, 23, 44 captured
   during the previous verification) and the pending seed;
2. SpecFit exact selection (``sf_specfit_select``) picks the verification
   sub-tree from the pool's route footprints;
3. the target verifies seed + tree in one forward under the ancestor mask,
   over a ``ReservedCache``;
4. the accepted path is committed: the KV rows of the seed and the accepted
   nodes are compacted in place (``_compact_tree_cache``, :833-858), their
   target features appended, and the target's prediction after the last
   accepted node becomes the next pending seed.

Configuration 4 of the benchmark runs this with random weights, so two
parts are synthetic and explicit here: each token routes through the target
by a fixed per-token Zipf(1.1) route (``synthetic.token_routes``), which
both replaces the router output during verification and gives SpecFit its
exact route footprints; and acceptance is simulated — a node at depth d is
accepted with probability p_d, p_d ~ Beta(4, 2) drawn once per depth from a
seed — with the greedy path through accepted nodes in node order.

With ``graphs=True`` drafting runs as device work replayed from one CUDA
graph per number of new rows (``DeviceDraft``), and each verification tree
size (1 to 8 rows) gets one
CUDA graph of the target forward, captured once and replayed at any
committed length: the reserved cache runs in static mode (keys/values
written at a device-side offset, attention over every reserved row), and the
ids, positions, mask and route override live in static device buffers that
each cycle refills.  Every expert must be resident (no host synchronisation
in the MoE blocks).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import selection as sel
from .. import synthetic
from .kv_cache import ReservedCache, compact_tree_cache_
from .tree_attention import clear_mask_cache


class BernoulliAcceptance:
    """p_d ~ Beta(a, b) per depth (drawn once); each verified node at depth d
    is accepted with probability p_d, independently, in node order."""

    def __init__(self, seed: int, max_depth: int = 8, a: float = 4.0, b: float = 2.0) -> None:
        self.rng = np.random.default_rng(seed)
        self.p = self.rng.beta(a, b, size=max_depth)

    def path(self, tree) -> tuple:
        ok = [bool(self.rng.random() < self.p[d - 1]) for d in tree.depths]
        children: dict = {}
        for node, parent in enumerate(tree.parent_ids, start=1):
            children.setdefault(parent, []).append(node)
        out, cur = [], 0
        while True:
            nxt = next((c for c in children.get(cur, ()) if ok[c - 1]), None)
            if nxt is None:
                return tuple(out)
            out.append(nxt)
            cur = nxt


@dataclass
class CycleRecord:
    pool_nodes: int
    selected: int
    accepted: int
    draft_ms: float
    select_ms: float
    verify_ms: float
    commit_ms: float


@dataclass
class DecodeResult:
    tokens: list
    cycles: list = field(default_factory=list)
    decode_s: float = 0.0
    prefill_s: float = 0.0

    @property
    def committed(self) -> int:
        return len(self.tokens)


class B200TreeSpeculator:
    def __init__(self, loaded, drafter, *, cost_model, acceptance: BernoulliAcceptance,
                 route_seed: int = 0, top_k: int = 4, max_depth: int = 8, first_width: int = 4,
                 level_width: int = 8, max_nodes: int = sel.MAX_DRAFT_NODES,
                 graphs: bool = False, reserve_tokens: int = 0, lean: bool = False) -> None:
        self.loaded = loaded
        self.model = loaded.model
        if lean:
            from .lean_forward import LeanQwen3Forward

            self.fwd = LeanQwen3Forward(self.model)
        else:
            self.fwd = self.model
        self.drafter = drafter
        self.cost_model = cost_model
        self.acceptance = acceptance
        self.route_seed = route_seed
        self.top_k, self.max_depth = top_k, max_depth
        self.first_width, self.level_width = first_width, level_width
        self.max_nodes = max_nodes
        cfg = self.model.config
        self.layers, self.experts, self.route_k = (cfg.num_hidden_layers, cfg.num_experts,
                                                   cfg.num_experts_per_tok)
        self.graphs = graphs
        self.reserve_tokens = reserve_tokens  # KV capacity to reserve (graphs keep one cache)
        self._aux: dict = {}
        self._override = None  # [q, layers, K] routes of the verify rows
        self._graphs: dict = {}
        self._offset = None
        self._cache = None
        self._ddraft = None
        if graphs:
            from .eagle3_drafter import DeviceDraft

            self._ddraft = DeviceDraft(drafter, top_k=top_k, max_depth=max_depth,
                                       first_width=first_width, level_width=level_width,
                                       max_new=1 + max_depth)

    # ------------------------------------------------------------- hooks
    def _install(self):
        hooks = []
        for li in self.drafter.layer_indices:
            def cap(mod, args, out, li=li):
                self._aux[li] = out[0] if isinstance(out, tuple) else out
            hooks.append(self.model.model.layers[li].register_forward_hook(cap))
        for l, layer in enumerate(self.model.model.layers):
            def route(mod, args, out, l=l):
                if self._override is None:
                    return None
                return out[0], out[1], self._override[:, l, :]
            hooks.append(layer.mlp.gate.register_forward_hook(route))
        return hooks

    def _features(self) -> torch.Tensor:
        """Target features of the last forward's rows: ``[rows, 3H]``."""
        return torch.cat([self._aux[li].reshape(-1, self._aux[li].shape[-1])
                          for li in self.drafter.layer_indices], dim=-1)

    # ------------------------------------------------------------- graphs
    def _graph(self, q: int, cache):
        g = self._graphs.get(q)
        if g is not None:
            return g
        dev = self.model.model.embed_tokens.weight.device
        cap = cache.layers[0].capacity
        ids = torch.zeros(1, q, dtype=torch.long, device=dev)
        pos = torch.zeros(1, q, dtype=torch.long, device=dev)
        mask = torch.zeros(1, 1, q, cap, dtype=torch.bool, device=dev)
        routes = torch.zeros(q, self.layers, self.route_k, dtype=torch.long, device=dev)
        base = cache.get_seq_length()
        if base + q > cap:
            raise RuntimeError("the reserved cache cannot hold the verification rows")
        self._offset.fill_(base)  # warm-up writes land past the committed rows
        mask[..., :base] = True
        mask[..., base:base + q] = torch.tril(torch.ones(q, q, dtype=torch.bool, device=dev))
        cache.set_static(self._offset, cap - q)
        self._override = routes
        try:
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side), torch.no_grad():
                for _ in range(2):
                    self.fwd(input_ids=ids, attention_mask=mask, position_ids=pos,
                               past_key_values=cache, use_cache=True)
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            clear_mask_cache()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph), torch.no_grad():
                out = self.fwd(input_ids=ids, attention_mask=mask, position_ids=pos,
                                 past_key_values=cache, use_cache=True)
                argmax = out.logits[0].argmax(-1)
                feats = self._features()
            clear_mask_cache()
        finally:
            self._override = None
            cache.set_static(None)
            cache.set_length(base)
        g = dict(graph=graph, ids=ids, pos=pos, mask=mask, routes=routes, argmax=argmax, feats=feats)
        self._graphs[q] = g
        return g

    def _verify_graph(self, cache, tree, pending, routes_sel, base: int):
        q = 1 + tree.draft_node_count
        g = self._graph(q, cache)
        dev = g["ids"].device
        g["ids"].copy_(tree.verification_token_ids(pending))
        g["pos"].copy_(tree.verification_position_ids(base_kv_length=base, device="cpu")
                       .to(dev, non_blocking=True))
        m = g["mask"]
        m[..., : base + q].copy_(tree.verification_attention_mask(base_kv_length=base, device="cpu")
                                 .to(dev, non_blocking=True))
        m[..., base + q:] = False
        g["routes"].copy_(routes_sel)
        self._offset.fill_(base)
        g["graph"].replay()
        cache.set_length(base + q)
        return g["ids"], g["argmax"], g["feats"]

    def release_graphs(self) -> None:
        self._graphs.clear()
        if self._ddraft is not None:
            self._ddraft.release()

    def calibrate_cost_model(self, *, expert_ns: float, reps: int = 5, seed: int = 0):
        """A ``SelectionCostModel`` fitted to this GPU, the way the reference
        fits its own (``docs/results/selection-refinement-*.json``): for each
        tree size n = 0..max_nodes the verify graph of a chain of n random
        tokens is replayed ``reps`` times over the current cache (its rows go
        past the committed length and are dropped), and
        ``intercept[n] = median time - expert_ns * |footprint|``; the slope
        ``expert_ns`` (one distinct (layer, expert) of the footprint) is given,
        e.g. one packed expert's bytes over the measured HBM bandwidth.
        Needs ``graphs=True`` and a cache left by ``generate``."""
        from ..selection import SelectionCostModel
        from .eagle3_types import Eagle3DraftTree

        cache = self._cache
        if not self.graphs or cache is None or not cache.layers[0].is_initialized:
            raise RuntimeError("calibration needs the verify graphs and a prefilled cache")
        dev = self._offset.device
        base = cache.get_seq_length()
        rng = np.random.default_rng(seed)
        vocab = self.model.config.vocab_size
        hooks = self._install()
        intercepts, means = [], []
        try:
            for n in range(self.max_nodes + 1):
                toks = [int(t) for t in rng.integers(0, vocab, size=n + 1)]
                tree = Eagle3DraftTree(tuple(toks[1:]), tuple(range(n)), tuple(range(1, n + 1)),
                                       (0.5,) * n, tuple(np.log(0.5) * np.arange(1, n + 1)))
                routes = synthetic.token_routes(torch.tensor(toks, device=dev), self.layers,
                                                experts=self.experts, top_k=self.route_k,
                                                seed=self.route_seed)
                union = int(np.unpackbits(np.bitwise_or.reduce(
                    sel.footprints(routes.cpu().numpy(), self.experts), axis=0).view(np.uint8)).sum())
                pending = torch.tensor([[toks[0]]], device=dev)
                times = []
                for _ in range(reps + 1):
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record()
                    self._verify_graph(cache, tree, pending, routes, base)
                    e.record()
                    e.synchronize()
                    cache.set_length(base)
                    times.append(s.elapsed_time(e) * 1e6)
                t = float(np.median(times[1:]))
                means.append(t)
                intercepts.append(max(t - expert_ns * union, 0.0))
        finally:
            for h in hooks:
                h.remove()
        return SelectionCostModel(tuple(means), tuple(intercepts), float(expert_ns))

    # ------------------------------------------------------------ generate
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int, *, sync_timing: bool = False):
        if input_ids.ndim != 2 or input_ids.shape[0] != 1:
            raise ValueError("tree speculation currently requires batch size 1")
        if max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be positive")
        dev = input_ids.device
        ctx = input_ids.shape[1]
        q_max = 1 + self.max_nodes
        need = max(ctx + max_new_tokens + q_max + 1, self.reserve_tokens)
        if self.graphs:
            # The graphs hold the cache's buffers: one cache per speculator, reused.
            cache = self._cache
            if cache is None or cache.layers[0].capacity < need:
                self._graphs.clear()
                cache = self._cache = ReservedCache(config=self.model.config, capacity=need)
            elif cache.layers[0].is_initialized:
                cache.set_length(0)
            if self._offset is None:
                self._offset = torch.zeros((), dtype=torch.long, device=dev)
        else:
            cache = ReservedCache(config=self.model.config, capacity=need)
        self.drafter.begin_generation(ctx + max_new_tokens + 2 + self.first_width
                                      + self.level_width * self.max_depth)
        hooks = self._install()
        result = DecodeResult(tokens=[])
        tick = (lambda: torch.cuda.synchronize(dev)) if sync_timing else (lambda: None)
        try:
            t0 = time.perf_counter()
            with torch.no_grad():
                out = self.fwd(input_ids=input_ids, past_key_values=cache, use_cache=True,
                                 logits_to_keep=1)
            aux = self._features()
            pending = out.logits[:, -1:].argmax(-1)
            fed = input_ids
            if self.graphs:
                for q in range(1, q_max + 1):  # every tree size, captured once
                    self._graph(q, cache)
            torch.cuda.synchronize(dev)
            result.prefill_s = time.perf_counter() - t0
            t_start = time.perf_counter()
            while len(result.tokens) < max_new_tokens:
                remaining = max_new_tokens - len(result.tokens)
                if remaining == 1:
                    result.tokens.append(int(pending.reshape(-1)[0]))
                    break
                ta = time.perf_counter()
                n_new = fed.shape[1] + 1 - self.drafter._fed
                with torch.no_grad():
                    if (self._ddraft is not None and self.drafter._fed > 0 and remaining - 1 >= self.max_depth
                            and n_new <= self._ddraft.max_new):
                        pool = self._ddraft.pool(fed_ids=fed, aux_history=aux, pending_seed=pending)
                    else:
                        pool = self.drafter.build_candidate_pool(
                            fed_ids=fed, aux_history=aux, pending_seed=pending, top_k=self.top_k,
                            max_depth=min(self.max_depth, remaining - 1), first_width=self.first_width,
                            level_width=self.level_width)
                        if self._ddraft is not None and len(self._ddraft._graphs) < self._ddraft.max_new:
                            self._ddraft.prepare()  # every drafting graph, before the next cycle
                tick()
                tb = time.perf_counter()
                toks = torch.tensor((pool.seed_token_id,) + tuple(c.target_token_id for c in pool.candidates),
                                    device=dev)
                routes = synthetic.token_routes(toks, self.layers, experts=self.experts,
                                                top_k=self.route_k, seed=self.route_seed)
                ids = sel.search([c.parent_raw_id for c in pool.candidates],
                                 [c.cumulative_log_probability for c in pool.candidates],
                                 sel.footprints(routes.cpu().numpy(), self.experts), self.cost_model,
                                 None, max_nodes=min(self.max_nodes, remaining - 1))
                tree = pool.to_tree(tuple(ids))
                tc = time.perf_counter()
                base = cache.get_seq_length()
                routes_sel = routes[[0] + list(ids)]
                if self.graphs:
                    verify_ids, verifier, q_aux = self._verify_graph(cache, tree, pending, routes_sel, base)
                else:
                    verify_ids = tree.verification_token_ids(pending)
                    mask = tree.verification_attention_mask(base_kv_length=base, device=dev)
                    pos = tree.verification_position_ids(base_kv_length=base, device=dev)
                    self._override = routes_sel
                    try:
                        with torch.no_grad():
                            vout = self.fwd(input_ids=verify_ids, attention_mask=mask,
                                              position_ids=pos, past_key_values=cache, use_cache=True)
                    finally:
                        self._override = None
                    q_aux = self._features()
                    verifier = vout.logits[0].argmax(-1)
                tick()
                td = time.perf_counter()
                path = self.acceptance.path(tree)
                positions = (0,) + path
                compact_tree_cache_(cache, base_kv_length=base, verification_positions=positions,
                                    verification_node_count=verify_ids.shape[1])
                ptens = torch.tensor(positions, device=dev)
                committed = verify_ids[:, ptens]
                fed = torch.cat((fed, committed), dim=1)
                aux = torch.cat((aux, q_aux.index_select(0, ptens)), dim=0)
                pending = verifier[positions[-1]].reshape(1, 1).clone()
                result.tokens.extend(committed[0].tolist())
                te = time.perf_counter()
                result.cycles.append(CycleRecord(len(pool.candidates), len(ids), len(path),
                                                 (tb - ta) * 1e3, (tc - tb) * 1e3, (td - tc) * 1e3,
                                                 (te - td) * 1e3))
            torch.cuda.synchronize(dev)
            result.decode_s = time.perf_counter() - t_start
            result.tokens = result.tokens[:max_new_tokens]
        finally:
            for h in hooks:
                h.remove()
            self.drafter.end_generation()
        return result
