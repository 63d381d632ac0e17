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

from .. import ops
from .. import selection as sel
from .. import synthetic
from .eagle3_types import tree_from_arrays
from .kv_cache import ReservedCache, compact_tree_cache_
from .tree_attention import clear_mask_cache




def _verify_argmax(out):
    """The target's greedy token per verify row: the lean forward's fused
    lm_head argmax when it produced one (equal, bit for bit, to the argmax of
    the logits it returns), else the argmax of the logits."""
    fused = getattr(out, "argmax", None)
    return fused[0] if fused is not None else out.logits[0].argmax(-1)

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


def verify_input_rows(tree, base: int) -> list:
    """The verify graph's per-row inputs for ``tree`` at committed length
    ``base``: (pool row, position, ancestor set over the tree block) of the
    seed (row 0) and each node -- the positions of
    ``Eagle3DraftTree.verification_position_ids`` and, as bitsets, the rows
    of its ``verification_attention_mask`` past the committed columns
    (src/specfit/runtime/eagle3_types.py:429-473)."""
    rows = [(0, base, 1)]
    anc = [1]
    for i, (raw, par, dep) in enumerate(zip(tree.source_raw_ids, tree.parent_ids, tree.depths), 1):
        anc.append(anc[par] | (1 << i))
        rows.append((int(raw), base + int(dep), anc[i]))
    return rows


def visibility_from_ancestors(anc: torch.Tensor, offset: torch.Tensor, cap: int) -> torch.Tensor:
    """Boolean ``[q, cap]`` visibility over a whole reserved KV buffer: column
    c is visible to row r when c < offset (committed rows) or when
    0 <= c - offset < 64 and bit c - offset of ``anc[r]`` is set (graph-
    capturable torch ops; the bool-mask form of ``sf_tree_mask_words``)."""
    q = anc.shape[0]
    rel = torch.arange(cap, device=anc.device) - offset
    bit = (anc.view(q, 1) >> rel.clamp(0, 63).view(1, cap)) & 1
    return (rel < 0).view(1, cap) | ((rel < 64).view(1, cap) & bit.bool())


@dataclass
class CycleRecord:
    pool_nodes: int
    selected: int
    accepted: int
    draft_ms: float
    select_ms: float
    verify_ms: float
    commit_ms: float
    experts: int = 0  # distinct (layer, expert) pairs of the verified rows (the footprint)


@dataclass
class DecodeResult:
    tokens: list
    cycles: list = field(default_factory=list)
    decode_s: float = 0.0
    prefill_s: float = 0.0
    draft_split: list = field(default_factory=list)  # DeviceDraft.last_timing of each device-drafted cycle

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
        self.lean = lean
        self.reserve_tokens = reserve_tokens  # KV capacity to reserve (graphs keep one cache)
        self._aux: dict = {}
        self._override = None  # [layers, q, K] routes of the verify rows (each layer contiguous)
        self._graphs: dict = {}
        self._offset = None
        self._cache = None
        self._ddraft = None
        if graphs:
            from .eagle3_drafter import DeviceDraft

            self._ddraft = DeviceDraft(drafter, top_k=top_k, max_depth=max_depth,
                                       first_width=first_width, level_width=level_width,
                                       max_new=1 + max_depth)
            # The pool as device buffers (row 0 = the seed, row r = raw id r):
            # tokens, their synthetic routes and route footprints, written by
            # every drafting graph and read by every verify graph.
            dev = drafter.fc.weight.device
            rows = 1 + self._ddraft.n_cand
            words = (self.layers * self.experts + 63) // 64
            self._pool_tok = torch.zeros(rows, dtype=torch.long, device=dev)
            self._pool_routes = torch.zeros(rows, self.layers, self.route_k, dtype=torch.long, device=dev)
            self._pool_fp = torch.zeros(rows, words, dtype=torch.long, device=dev)
            self._ddraft.post = self._post_draft
        self._pos_host = torch.zeros(64, dtype=torch.long).pin_memory() if torch.cuda.is_available() else None

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
                return out[0], out[1], self._override[l]
            hooks.append(layer.mlp.gate.register_forward_hook(route))
        return hooks

    def _features(self) -> torch.Tensor:
        """Target features of the last forward's rows: ``[rows, 3H]``."""
        return torch.cat([self._aux[li].reshape(-1, self._aux[li].shape[-1])
                          for li in self.drafter.layer_indices], dim=-1)

    # ------------------------------------------------------------- graphs
    def _routes_into(self) -> None:
        """Routes and footprints of every pool row (device work)."""
        r = synthetic.token_routes(self._pool_tok, self.layers, experts=self.experts,
                                   top_k=self.route_k, seed=self.route_seed)
        self._pool_routes.copy_(r)
        sel.footprints_device(r, self.experts, out=self._pool_fp)

    def _post_draft(self, seed: torch.Tensor, out: torch.Tensor) -> None:
        """Appended to each drafting graph: the pool's tokens into the pool
        buffers, then their routes and footprints."""
        self._pool_tok[:1].copy_(seed)
        self._pool_tok[1:].copy_(out[:, 0])
        self._routes_into()

    def _graph(self, q: int, cache):
        """The verify graph of ``q`` rows.  Its inputs are one device int64
        block ``vin [3, q]`` (pool row of each verify row, position,
        ancestor set over the tree block) plus the pool buffers; token ids,
        the route override and the visibility words are built inside the
        graph."""
        g = self._graphs.get(q)
        if g is not None:
            return g
        dev = self.model.model.embed_tokens.weight.device
        cap = cache.layers[0].capacity
        base = cache.get_seq_length()
        if base + q > cap:
            raise RuntimeError("the reserved cache cannot hold the verification rows")
        vin = torch.zeros(3, q, dtype=torch.long, device=dev)
        ar = torch.arange(q, device=dev)
        vin[0] = ar
        vin[1] = base + ar
        vin[2] = (torch.ones_like(ar) << (ar + 1)) - 1  # a chain: warm-up and capture inputs
        routes = torch.zeros(self.layers, q, self.route_k, dtype=torch.long, device=dev)
        words = (cap + 31) // 32
        self._offset.fill_(base)  # warm-up writes land past the committed rows
        cache.set_static(self._offset, cap - q)
        self._override = routes

        def body():
            rows, pos, anc = vin[0], vin[1], vin[2]
            ids = self._pool_tok.index_select(0, rows).view(1, q)
            routes.copy_(self._pool_routes.index_select(0, rows).transpose(0, 1))
            if self.lean:
                w = ops.tree_mask_words(anc, self._offset, words)
                out = self.fwd(input_ids=ids, attention_words=w.view(1, q, words),
                               position_ids=pos.view(1, q), past_key_values=cache, use_cache=True)
            else:
                vis = visibility_from_ancestors(anc, self._offset, cap)
                out = self.fwd(input_ids=ids, attention_mask=vis.view(1, 1, q, cap),
                               position_ids=pos.view(1, q), past_key_values=cache, use_cache=True)
            return ids, _verify_argmax(out), self._features()

        try:
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side), torch.no_grad():
                for _ in range(2):
                    body()
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            clear_mask_cache()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph), torch.no_grad():
                ids, argmax, feats = body()
            clear_mask_cache()
        finally:
            self._override = None
            cache.set_static(None)
            cache.set_length(base)
        # Every buffer the graph reads or writes that was allocated outside
        # the capture stays referenced here (routes: the override buffer).
        g = dict(graph=graph, vin=vin, vin_host=torch.zeros(3, q, dtype=torch.long).pin_memory(),
                 routes=routes, ids=ids, argmax=argmax, feats=feats)
        self._graphs[q] = g
        return g

    def _verify_graph(self, cache, tree, base: int):
        """Replays the verify graph for ``tree`` over pool rows
        ``(0,) + tree.source_raw_ids`` at committed length ``base``: one
        host-to-device copy of the [3, q] input block."""
        q = 1 + tree.draft_node_count
        g = self._graph(q, cache)
        h = g["vin_host"].numpy()
        for i, (row, pos, anc) in enumerate(verify_input_rows(tree, base)):
            h[0, i], h[1, i], h[2, i] = row, pos, anc
        g["vin"].copy_(g["vin_host"], non_blocking=True)
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
                self._pool_tok[: n + 1].copy_(torch.tensor(toks))
                self._routes_into()
                fp = self._pool_fp[: n + 1].cpu().numpy().view(np.uint64)
                union = int(np.unpackbits(np.bitwise_or.reduce(fp, axis=0).view(np.uint8)).sum())
                times = []
                for _ in range(reps + 1):
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record()
                    self._verify_graph(cache, tree, base)
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

    def calibrate_cycle_cost_model(self, input_ids: torch.Tensor, *, expert_ns: float,
                                   tokens: int = 64):
        """A ``SelectionCostModel`` fitted the way the reference fits its
        own, on whole local cycles (``docs/results/selection-refinement-*.json``:
        "fixed-state local cycles"): for each tree size n = 0..max_nodes a
        generation of ``tokens`` tokens runs with the selection forced to
        size n (a cost model under which only size-n trees have a finite
        price), each cycle's wall time (draft, select, verify, commit) is
        taken, and ``intercept[n] = median(cycle time - expert_ns *
        |footprint|)`` over the cycles that verified n nodes (the first
        cycle, with the eager catch-up, excluded).  ``expert_ns`` is given,
        e.g. one packed expert's bytes over the measured HBM bandwidth."""
        from ..selection import SelectionCostModel

        keep = self.cost_model
        sizes = self.max_nodes + 1
        intercepts, means = [], []
        try:
            for n in range(sizes):
                price = tuple(1e6 if i == n else 1e15 for i in range(sizes))
                self.cost_model = SelectionCostModel(price, price, float(expert_ns))
                res = self.generate(input_ids, tokens)
                cyc = [c for c in res.cycles[1:] if c.selected == n]
                if not cyc:
                    raise RuntimeError(f"no cycle verified {n} nodes during calibration")
                total = [1e6 * (c.draft_ms + c.select_ms + c.verify_ms + c.commit_ms) for c in cyc]
                means.append(float(np.median(total)))
                intercepts.append(max(float(np.median([t - expert_ns * c.experts
                                                       for t, c in zip(total, cyc)])), 0.0))
        finally:
            self.cost_model = keep
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
            # Committed tokens and their target features live in preallocated
            # buffers; fed / aux are views of their filled rows.
            rows_max = ctx + max_new_tokens + q_max + 1
            feats0 = self._features()
            fed_buf = torch.empty(1, rows_max, dtype=input_ids.dtype, device=dev)
            aux_buf = torch.empty(rows_max, feats0.shape[1], dtype=feats0.dtype, device=dev)
            fed_buf[:, :ctx].copy_(input_ids)
            aux_buf[:ctx].copy_(feats0)
            L = ctx
            fed, aux = fed_buf[:, :L], aux_buf[:L]
            pending = out.logits[:, -1:].argmax(-1)
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
                n_new = L + 1 - self.drafter._fed
                max_nodes = min(self.max_nodes, remaining - 1)
                routes = None
                with torch.no_grad():
                    if (self._ddraft is not None and self.drafter._fed > 0 and remaining - 1 >= self.max_depth
                            and n_new <= self._ddraft.max_new):
                        # Device drafting: pool rows and footprints in one read-back.
                        arr, (fp,) = self._ddraft.pool_arrays(fed_ids=fed, aux_history=aux,
                                                              pending_seed=pending, extra=(self._pool_fp,))
                        tb = time.perf_counter()
                        result.draft_split.append(self._ddraft.last_timing)
                        tok = arr[:, 0].astype(np.int64)
                        par = arr[:, 1].astype(np.int64) + 1  # raw parent ids (0 = the seed)
                        cond = np.minimum(arr[:, 2], 0.0)     # log-probabilities
                        depth = arr[:, 4].astype(np.int64)
                        cum = arr[:, 3]                       # parent's cum + cond, in fp64
                        ids = sel.search(par, cum, fp[: 1 + len(tok)].view(np.uint64), self.cost_model,
                                         None, max_nodes=max_nodes)
                        tree = tree_from_arrays(tuple(ids), tok, par, depth, cond, cum)
                        n_pool = len(tok)
                    else:
                        pool = self.drafter.build_candidate_pool(
                            fed_ids=fed, aux_history=aux, pending_seed=pending, top_k=self.top_k,
                            max_depth=min(self.max_depth, remaining - 1), first_width=self.first_width,
                            level_width=self.level_width)
                        if self._ddraft is not None and len(self._ddraft._graphs) < self._ddraft.max_new:
                            self._ddraft.prepare()  # every drafting graph, before the next cycle
                        tb = time.perf_counter()
                        toks = torch.tensor((pool.seed_token_id,) + tuple(c.target_token_id for c in pool.candidates))
                        n_pool = len(pool.candidates)
                        if self.graphs:
                            self._pool_tok[: n_pool + 1].copy_(toks)
                            self._routes_into()
                            fp = self._pool_fp[: n_pool + 1].cpu().numpy().view(np.uint64)
                        else:
                            routes = synthetic.token_routes(toks.to(dev), self.layers, experts=self.experts,
                                                            top_k=self.route_k, seed=self.route_seed)
                            fp = sel.footprints(routes.cpu().numpy(), self.experts)
                        ids = sel.search([c.parent_raw_id for c in pool.candidates],
                                         [c.cumulative_log_probability for c in pool.candidates],
                                         fp, self.cost_model, None, max_nodes=max_nodes)
                        tree = pool.to_tree(tuple(ids))
                rows_fp = np.asarray(fp)[[0] + list(tree.source_raw_ids)].view(np.uint64)
                experts = int(np.bitwise_count(np.bitwise_or.reduce(rows_fp, axis=0)).sum())
                tick()
                tc = time.perf_counter()
                base = cache.get_seq_length()
                if self.graphs:
                    verify_ids, verifier, q_aux = self._verify_graph(cache, tree, base)
                else:
                    verify_ids = tree.verification_token_ids(pending)
                    mask = tree.verification_attention_mask(base_kv_length=base, device=dev)
                    pos = tree.verification_position_ids(base_kv_length=base, device=dev)
                    self._override = routes[[0] + list(tree.source_raw_ids)].transpose(0, 1).contiguous()
                    try:
                        with torch.no_grad():
                            vout = self.fwd(input_ids=verify_ids, attention_mask=mask,
                                            position_ids=pos, past_key_values=cache, use_cache=True)
                    finally:
                        self._override = None
                    q_aux = self._features()
                    verifier = _verify_argmax(vout)
                tick()
                td = time.perf_counter()
                path = self.acceptance.path(tree)
                positions = (0,) + path
                n = len(positions)
                compact_tree_cache_(cache, base_kv_length=base, verification_positions=positions,
                                    verification_node_count=verify_ids.shape[1])
                ph = self._pos_host[:n]
                ph.numpy()[:] = positions
                ptens = ph.to(dev, non_blocking=True)
                torch.index_select(verify_ids, 1, ptens, out=fed_buf[:, L:L + n])
                torch.index_select(q_aux, 0, ptens, out=aux_buf[L:L + n])
                pending = verifier[positions[-1]].reshape(1, 1).clone()
                result.tokens.extend(fed_buf[0, L:L + n].tolist())
                L += n
                fed, aux = fed_buf[:, :L], aux_buf[:L]
                te = time.perf_counter()
                result.cycles.append(CycleRecord(n_pool, len(ids), len(path),
                                                 (tb - ta) * 1e3, (tc - tb) * 1e3, (td - tc) * 1e3,
                                                 (te - td) * 1e3, experts))
            torch.cuda.synchronize(dev)
            result.decode_s = time.perf_counter() - t_start
            result.tokens = result.tokens[:max_new_tokens]
        finally:
            for h in hooks:
                h.remove()
            self.drafter.end_generation()
        return result
