"""EAGLE-3-shaped tree drafter stand-in on the B200 kernels.

The reference drafts with an EAGLE-3 model from ``speculators`` (absent here,
so drafter parity is unpinned); BASELINE configuration 4 specifies a
stand-in of the same shape with random weights: one decoder layer, hidden
2048, an ``fc`` fusing the target's hidden states of layers (1, 23, 44)
(``QWEN3_EAGLE3_LAYER_INDICES``, ``src/specfit/runtime/eagle3_chain.py:23``)
into 2048, the target's token embedding, and a 151,936-way lm_head.

Alignment (EAGLE): the drafter row of token ``x_p`` uses ``embed(x_p)`` and
the fused target feature of position ``p - 1``; a drafted node uses its
token's embedding and its parent's drafter output in place of the target
feature.  Rows of committed tokens stay in the drafter's own KV buffer; a
cycle's tree rows are appended after them and dropped after drafting, except
the pending seed's row, which is exactly the committed row it will become.

Random weights give a nearly flat softmax over 151,936 tokens (top-1 mass
~1e-5), which would make every drafted node worthless to SpecFit; the
stand-in therefore scales its logits by ``logit_scale`` (default 4.5, a
logit standard deviation near 4, top-1 mass ~0.2-0.8) so its confidences are
in the range of the simulated acceptance rates.

Drafting (``build_candidate_pool``) grows a candidate pool level by level:
level 1 holds the seed's ``first_width`` most likely children, and every
later level the ``level_width`` most likely children (by cumulative
log-probability) of the previous level's nodes, each node offering its
``top_k`` most likely tokens, up to ``max_depth`` levels.  Attention runs on
``sf_tree_attention`` (the committed rows as prefix, the tree rows under
their ancestor mask); projections are cuBLAS GEMMs.

``DeviceDraft`` runs the same drafting with no host round trip: the level
expansions (top-k per node, cumulative scores, the best ``level_width``
children) are tensor ops, rows are written at device-side offsets, each
row's visibility is a 64-bit ancestor set inside the tree block expanded
into a mask over the whole KV buffer (``sf_tree_mask_words``), and the pool
comes back in one copy.  Its layer runs on the fused kernels of the lean
target forward (``sf_add_rmsnorm``, ``sf_qk_norm_rope`` without head norms,
fused q|k|v and gate|up GEMMs).
Its fixed shapes let it be one CUDA graph per number of catch-up rows.
"""
from __future__ import annotations

import time

import torch
from torch import nn

import torch.nn.functional as F

from .. import _native as N
from .. import ops
from .eagle3_types import Eagle3DraftCandidate, Eagle3DraftCandidatePool

AUX_LAYERS = (1, 23, 44)


def _rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def _rope(x: torch.Tensor, pos: torch.Tensor, theta: float) -> torch.Tensor:
    """Rotary embedding (half-split convention) of ``x [heads, n, D]``."""
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d))
    ang = pos.float()[:, None] * inv[None, :]
    cos, sin = torch.cos(ang), torch.sin(ang)
    xf = x.float()
    a, b = xf[..., : d // 2], xf[..., d // 2:]
    return torch.cat((a * cos - b * sin, b * cos + a * sin), dim=-1).to(x.dtype)


def _bits(rows: list, device) -> torch.Tensor:
    """int32 words of per-row visibility bitsets (Python ints)."""
    width = max(1, max((r.bit_length() for r in rows), default=1))
    words = (width + 31) // 32
    data = []
    for r in rows:
        for w in range(words):
            word = (r >> (32 * w)) & 0xFFFFFFFF
            data.append(word - (1 << 32) if word >= (1 << 31) else word)
    return torch.tensor(data, dtype=torch.int32).view(len(rows), words).to(device)


class Eagle3DrafterStandIn(nn.Module):
    def __init__(self, *, hidden: int, heads: int, kv_heads: int, head_dim: int, inter: int,
                 vocab: int, embed: nn.Embedding, rope_theta: float, eps: float,
                 aux_layers=AUX_LAYERS, logit_scale: float = 4.5, device=None,
                 dtype=torch.bfloat16) -> None:
        super().__init__()
        self.hidden, self.heads, self.kv_heads, self.head_dim = hidden, heads, kv_heads, head_dim
        self.vocab, self.theta, self.eps = vocab, rope_theta, eps
        self.logit_scale = float(logit_scale)
        self.layer_indices = tuple(aux_layers)
        kw = dict(device=device, dtype=dtype)
        self.fc = nn.Linear(len(self.layer_indices) * hidden, hidden, bias=False, **kw)
        self.emb_norm = nn.Parameter(torch.ones(hidden, **kw))
        self.hid_norm = nn.Parameter(torch.ones(hidden, **kw))
        self.q_proj = nn.Linear(2 * hidden, heads * head_dim, bias=False, **kw)
        self.k_proj = nn.Linear(2 * hidden, kv_heads * head_dim, bias=False, **kw)
        self.v_proj = nn.Linear(2 * hidden, kv_heads * head_dim, bias=False, **kw)
        self.o_proj = nn.Linear(heads * head_dim, hidden, bias=False, **kw)
        self.post_norm = nn.Parameter(torch.ones(hidden, **kw))
        self.gate_proj = nn.Linear(hidden, inter, bias=False, **kw)
        self.up_proj = nn.Linear(hidden, inter, bias=False, **kw)
        self.down_proj = nn.Linear(inter, hidden, bias=False, **kw)
        self.final_norm = nn.Parameter(torch.ones(hidden, **kw))
        self.lm_head = nn.Linear(hidden, vocab, bias=False, **kw)
        self.embed = embed  # the target's token embedding (shared, not re-drawn)
        self._k = self._v = None
        self._len = 0  # rows of committed tokens (and the kept seed row) in the KV buffer
        self._fed = 0  # committed tokens those rows cover

    # ---------------------------------------------------------------- state
    def begin_generation(self, capacity: int) -> None:
        """Start a sequence; the KV buffer (``capacity`` rows, rounded up to
        a multiple of 32) is kept and reused while it is large enough, so
        graphs captured over it stay valid."""
        capacity = (capacity + 31) // 32 * 32
        if self._k is None or self._k.shape[1] < capacity:
            dev = self.fc.weight.device
            shape = (self.kv_heads, capacity, self.head_dim)
            self._k = torch.zeros(shape, dtype=self.fc.weight.dtype, device=dev)
            self._v = torch.zeros(shape, dtype=self.fc.weight.dtype, device=dev)
        self._len = self._fed = 0

    def end_generation(self) -> None:
        self._len = self._fed = 0

    def release(self) -> None:
        """Free the KV buffer."""
        self._k = self._v = None
        self._len = self._fed = 0

    # --------------------------------------------------------------- forward
    def _rows(self, tokens: torch.Tensor, feats: torch.Tensor, pos: torch.Tensor,
              bits: torch.Tensor | None, prefix: int) -> torch.Tensor:
        """Drafter layer over ``n`` rows appended at ``self._len``; returns
        the layer output ``[n, H]`` (rows stay in the buffer)."""
        n = tokens.shape[0]
        if self._len + n > self._k.shape[1]:
            raise RuntimeError("drafter KV buffer is full")
        x = torch.cat((_rms_norm(self.embed(tokens), self.emb_norm, self.eps),
                       _rms_norm(feats, self.hid_norm, self.eps)), dim=-1)
        q = self.q_proj(x).view(n, self.heads, self.head_dim).transpose(0, 1)
        k = self.k_proj(x).view(n, self.kv_heads, self.head_dim).transpose(0, 1)
        v = self.v_proj(x).view(n, self.kv_heads, self.head_dim).transpose(0, 1)
        q = _rope(q, pos, self.theta).contiguous()
        end = self._len + n
        self._k[:, self._len:end].copy_(_rope(k, pos, self.theta))
        self._v[:, self._len:end].copy_(v)
        self._len = end
        attn = ops.tree_attention(q, self._k[:, :end], self._v[:, :end], bits, prefix,
                                  scale=self.head_dim ** -0.5)
        h = feats + self.o_proj(attn.reshape(n, self.heads * self.head_dim))
        m = _rms_norm(h, self.post_norm, self.eps)
        return h + self.down_proj(torch.nn.functional.silu(self.gate_proj(m)) * self.up_proj(m))

    def _top(self, h: torch.Tensor, k: int):
        """The k most likely next tokens of each row: (log-probs, ids), one
        fused log-softmax + top-k launch over the lm_head logits."""
        logits = self.lm_head(_rms_norm(h, self.final_norm, self.eps))
        return ops.logsoftmax_topk(logits, k, self.logit_scale)

    # -------------------------------------------------------------- drafting
    def build_candidate_pool(self, *, fed_ids: torch.Tensor, aux_history: torch.Tensor,
                             pending_seed: torch.Tensor, top_k: int = 4, max_depth: int = 8,
                             first_width: int = 4, level_width: int = 8) -> Eagle3DraftCandidatePool:
        """``fed_ids [1, L]`` committed tokens, ``aux_history [L, 3H]`` their
        target features (layers ``layer_indices`` concatenated), the pending
        seed ``[1, 1]``.  Returns the candidate pool in generation order."""
        dev = self.fc.weight.device
        L = fed_ids.shape[1]
        if aux_history.shape[0] != L:
            raise ValueError("aux history must cover every fed token")
        # Rows of the newly committed tokens (catch-up) and the seed row: token
        # p uses the target feature of position p - 1 (zero for p = 0).
        start = self._fed
        feats = self.fc(aux_history[max(start - 1, 0):L])
        if start == 0:
            feats = torch.cat((torch.zeros_like(feats[:1]), feats), dim=0)
        toks = torch.cat((fed_ids[0, start:L], pending_seed.reshape(1)))
        n_new = toks.shape[0]
        pos = torch.arange(start, L + 1, device=dev)
        chain = [(1 << (i + 1)) - 1 for i in range(n_new)]  # causal among the new rows
        h = self._rows(toks, feats, pos, _bits(chain, dev), self._len)
        committed_rows = self._len - 1  # the tree block starts at the seed row
        seed_hidden = h[-1]
        vals, idx = (t[0] for t in self._top(h[-1:], min(top_k, first_width)))
        cands: list = []
        vis = {0: 1}  # raw id -> visibility bitset inside the tree block (seed = bit 0)
        rows_in_block = 1
        hidden_of = {0: seed_hidden}
        frontier = []
        for v, t in zip(vals.tolist(), idx.tolist()):
            raw = len(cands) + 1
            cands.append(Eagle3DraftCandidate(raw, 0, 1, int(t), float(v), float(v), raw - 1, (int(t),)))
            frontier.append(raw)
        steps = 1
        for depth in range(1, max_depth):
            rows = []
            for j, raw in enumerate(frontier):
                vis[raw] = vis[cands[raw - 1].parent_raw_id] | (1 << (rows_in_block + j))
                rows.append(vis[raw])
            rows_in_block += len(frontier)
            tok = torch.tensor([cands[r - 1].target_token_id for r in frontier], device=dev)
            parent_feats = torch.stack([hidden_of[cands[r - 1].parent_raw_id] for r in frontier])
            lvl_pos = torch.full((len(frontier),), L + depth, device=dev)
            hl = self._rows(tok, parent_feats, lvl_pos, _bits(rows, dev), committed_rows)
            steps += 1
            for j, raw in enumerate(frontier):
                hidden_of[raw] = hl[j]
            v, t = self._top(hl, top_k)
            options = []
            for j, raw in enumerate(frontier):
                base = cands[raw - 1].cumulative_log_probability
                for vv, tt in zip(v[j].tolist(), t[j].tolist()):
                    options.append((base + vv, raw, int(tt), float(vv)))
            options.sort(key=lambda o: (-o[0], o[1], o[2]))
            frontier = []
            for _, parent, tok_id, cond in options[:level_width]:
                p = cands[parent - 1]
                raw = len(cands) + 1
                cands.append(Eagle3DraftCandidate(raw, parent, depth + 1, tok_id, cond,
                                                  p.cumulative_log_probability + cond, raw - 1,
                                                  p.path + (tok_id,)))
                frontier.append(raw)
        # Keep the committed rows and the seed row; drop the tree rows.
        self._len = committed_rows + 1
        self._fed = L + 1
        return Eagle3DraftCandidatePool(int(pending_seed.reshape(-1)[0]), top_k, max_depth,
                                        tuple(cands), path_score_calls=steps,
                                        draft_transformer_steps=steps, draft_forward_calls=steps,
                                        draft_query_tokens=n_new + rows_in_block - 1)


def build_random_drafter(target, *, seed: int = 0, std: float = 0.02, inter: int = 6144,
                         aux_layers=AUX_LAYERS, logit_scale: float = 4.5) -> Eagle3DrafterStandIn:
    """Random-init stand-in shaped for ``target`` (a Qwen3-MoE HF model),
    sharing its token embedding; weights N(0, std) from ``seed``."""
    cfg = target.config
    dev = target.model.embed_tokens.weight.device
    d = Eagle3DrafterStandIn(hidden=cfg.hidden_size, heads=cfg.num_attention_heads,
                             kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim, inter=inter,
                             vocab=cfg.vocab_size, embed=target.model.embed_tokens,
                             rope_theta=cfg.rope_parameters["rope_theta"], eps=cfg.rms_norm_eps,
                             aux_layers=aux_layers, logit_scale=logit_scale, device=dev,
                             dtype=target.model.embed_tokens.weight.dtype)
    g = torch.Generator(device=dev).manual_seed(seed)
    with torch.no_grad():
        for name, p in sorted(d.named_parameters(), key=lambda kv: kv[0]):
            if name.startswith("embed."):
                continue
            if p.ndim == 1:
                p.fill_(1.0)
            else:
                p.normal_(0.0, std, generator=g)
    d.eval()
    return d


class DeviceDraft:
    """Graph-capturable drafting for one drafter and fixed widths.

    The drafter's KV buffer must have been started with ``begin_generation``
    and its committed rows filled by one eager ``build_candidate_pool`` (the
    prefill catch-up).  ``pool`` then drafts a full ``max_depth`` pool from up
    to ``max_new`` new rows (the newly committed tokens and the pending seed),
    replaying a CUDA graph captured per row count."""

    def __init__(self, drafter: Eagle3DrafterStandIn, *, top_k: int = 4, max_depth: int = 8,
                 first_width: int = 4, level_width: int = 8, max_new: int = 8) -> None:
        self.last_timing: dict = {}
        d = drafter
        self.d = d
        self.top_k, self.max_depth = top_k, max_depth
        self.first_width, self.level_width, self.max_new = first_width, level_width, max_new
        self.widths = [first_width] + [level_width] * (max_depth - 1)
        self.n_cand = sum(self.widths)
        rows_block = 1 + sum(self.widths[:-1])
        if rows_block > 64:
            raise ValueError("the tree block must fit a 64-bit ancestor set")
        dev = d.fc.weight.device
        self.dev = dev
        z = lambda *shape, dt=torch.long: torch.zeros(*shape, dtype=dt, device=dev)
        self.tokens = z(max_new)                      # new rows: committed tokens, then the seed
        self.aux = z(max_new, d.fc.in_features, dt=d.fc.weight.dtype)  # their features' sources
        self.start = z(())                            # committed rows before this cycle
        self.out = torch.zeros(self.n_cand, 5, dtype=torch.float64, device=dev)
        # Frontier buffers, two sets used alternately by the levels: tokens,
        # cumulative scores, ancestor sets, positions and parent hidden rows.
        wmax = max(self.widths)
        self._lv = [dict(tok=z(wmax), cum=z(wmax, dt=torch.float64), vis=z(wmax), pos=z(wmax),
                         hid=z(wmax, d.hidden, dt=d.fc.weight.dtype)) for _ in range(2)]
        self._seed_cum = z(1, dt=torch.float64)
        self._seed_vis = torch.ones(1, dtype=torch.long, device=dev)
        self._seed_pos = z(())                      # block row of the seed (= its position)
        self._host_out = torch.empty(self.n_cand, 5, dtype=torch.float64).pin_memory()
        self._host_extra: dict = {}
        # Optional device work appended to every drafting graph: called as
        # post(seed [1] int64, out [n_cand, 5] float64) after the pool is built.
        self.post = None
        self._graphs: dict = {}
        with torch.no_grad():
            self.wqkv = torch.cat((d.q_proj.weight, d.k_proj.weight, d.v_proj.weight), 0).contiguous()
            self.wgu = torch.cat((d.gate_proj.weight, d.up_proj.weight), 0).contiguous()
        self.inter = d.gate_proj.weight.shape[0]
        self.inv_freq = 1.0 / (d.theta ** (torch.arange(0, d.head_dim, 2, device=dev, dtype=torch.float32)
                                           / d.head_dim))

    def _norm(self, x, res_in, res_out, w, out):
        N.check(N.lib.sf_add_rmsnorm(x.data_ptr(), None if res_in is None else res_in.data_ptr(),
                                     None if res_out is None else res_out.data_ptr(), w.data_ptr(),
                                     float(self.d.eps), x.shape[0], x.shape[1], out.data_ptr(),
                                     torch.cuda.current_stream(self.dev).cuda_stream),
                "sf_add_rmsnorm")
        ops._launched(1)

    def _rows(self, tokens, feats, pos, vis, block_start, write_at):
        """The drafter layer over ``n`` rows written at device row
        ``write_at``; returns (layer output, its final-norm rows)."""
        d = self.d
        n = tokens.shape[0]
        H, D = d.hidden, d.head_dim
        cap = d._k.shape[1]
        stream = torch.cuda.current_stream(self.dev).cuda_stream
        e_n = torch.empty(n, H, dtype=feats.dtype, device=self.dev)
        f_n = torch.empty_like(e_n)
        self._norm(d.embed(tokens), None, None, d.emb_norm, e_n)
        self._norm(feats.contiguous(), None, None, d.hid_norm, f_n)
        qkv = ops.linear(torch.cat((e_n, f_n), dim=-1), self.wqkv)
        cos = torch.empty(n, D, dtype=feats.dtype, device=self.dev)
        sin = torch.empty_like(cos)
        N.check(N.lib.sf_rope_rows(pos.data_ptr(), n, self.inv_freq.data_ptr(), D, cos.data_ptr(),
                                   sin.data_ptr(), stream), "sf_rope_rows")
        q = torch.empty(d.heads, n, D, dtype=feats.dtype, device=self.dev)
        N.check(N.lib.sf_qk_norm_rope(qkv.data_ptr(), 1, n, d.heads, d.kv_heads, D, None, None,
                                      cos.data_ptr(), sin.data_ptr(), float(d.eps), q.data_ptr(),
                                      d._k.data_ptr(), d._v.data_ptr(), d.kv_heads * cap * D, cap * D,
                                      0, write_at.data_ptr(), stream), "sf_qk_norm_rope")
        words = torch.empty(n, cap // 32, dtype=torch.int32, device=self.dev)
        N.check(N.lib.sf_tree_mask_words(vis.data_ptr(), n, block_start.data_ptr(), cap // 32,
                                         words.data_ptr(), stream), "sf_tree_mask_words")
        ops._launched(3)
        attn = ops.tree_attention(q, d._k, d._v, words, 0, scale=D ** -0.5)
        o = ops.linear(attn.reshape(n, d.heads * D), d.o_proj.weight)
        h = torch.empty_like(e_n)
        m = torch.empty_like(e_n)
        self._norm(o, feats.contiguous(), h, d.post_norm, m)
        gu = ops.linear(m, self.wgu)
        dn = ops.linear(F.silu(gu[:, : self.inter]) * gu[:, self.inter:], d.down_proj.weight)
        out = torch.empty_like(e_n)
        hn = torch.empty_like(e_n)
        self._norm(dn, h, out, d.final_norm, hn)
        return out, hn

    def _top(self, hn, k):
        return ops.logsoftmax_topk(ops.linear(hn, self.d.lm_head.weight), k, self.d.logit_scale)

    def _draft(self, n_new: int) -> None:
        """The whole drafting of one cycle as device work (captured)."""
        d = self.d
        dev = self.dev
        toks = self.tokens[:n_new]
        feats = ops.linear(self.aux[:n_new], d.fc.weight)
        torch.add(self.start, n_new - 1, out=self._seed_pos)  # the seed's position = committed tokens
        pos = self.start + torch.arange(n_new, device=dev)
        chain = (torch.ones((), dtype=torch.int64, device=dev) << torch.arange(1, n_new + 1, device=dev)) - 1
        # Catch-up rows are causal among themselves after the committed rows;
        # the seed row (last) opens the tree block at row seed_pos.
        h, hn = self._rows(toks, feats, pos, chain, self.start, self.start)
        block = self._seed_pos
        stream = torch.cuda.current_stream(dev).cuda_stream
        H = d.hidden

        def level(v, t, rows, k, cum, vis, hidden, width, first, depth, row_base, nxt, out_at):
            N.check(N.lib.sf_draft_level(v.data_ptr(), t.data_ptr(), rows, k, cum.data_ptr(),
                                         vis.data_ptr(), hidden.data_ptr(), H, width, first, depth,
                                         row_base, self._seed_pos.data_ptr(), nxt["tok"].data_ptr(),
                                         nxt["cum"].data_ptr(), nxt["vis"].data_ptr(),
                                         nxt["pos"].data_ptr(), nxt["hid"].data_ptr(),
                                         self.out[out_at].data_ptr(), stream), "sf_draft_level")
            ops._launched(1)

        # Level 1: the seed row's best first_width tokens (parent -1 = the seed,
        # block row 0); their rows go at block rows 1.. .
        v0, t0 = self._top(hn[-1:], self.widths[0])
        level(v0, t0, 1, self.widths[0], self._seed_cum, self._seed_vis, h[-1:].contiguous(),
              self.widths[0], -1, 0, 1, self._lv[0], 0)
        first = 0                      # candidate index of the frontier's first node
        row_next = 1                   # block row of the frontier's first node
        w = self.widths[0]
        for depth in range(1, self.max_depth):
            cur, nxt = self._lv[(depth - 1) % 2], self._lv[depth % 2]
            hl, hln = self._rows(cur["tok"][:w], cur["hid"][:w], cur["pos"][:w], cur["vis"][:w], block,
                                 block + row_next)
            v, t = self._top(hln, self.top_k)                                # [w, k]
            level(v, t, w, self.top_k, cur["cum"], cur["vis"], hl, self.widths[depth], first, depth,
                  row_next + w, nxt, first + w)
            first += w
            row_next += w
            w = self.widths[depth]

        if self.post is not None:
            self.post(self.tokens[n_new - 1: n_new], self.out)

    def _graph(self, n_new: int):
        if getattr(self, "_kptr", None) != self.d._k.data_ptr():
            self._graphs.clear()  # a new KV buffer: earlier graphs point at the old one
            self._kptr = self.d._k.data_ptr()
        g = self._graphs.get(n_new)
        if g is not None:
            return g
        side = torch.cuda.Stream(device=self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(2):
                self._draft(n_new)
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph), torch.no_grad():
            self._draft(n_new)
        self._graphs[n_new] = graph
        return graph

    def prepare(self) -> None:
        """Capture the graph of every row count 1..max_new now (their warm-up
        writes land past the committed rows and are overwritten later), so no
        capture happens between cycles."""
        d = self.d
        if d._fed == 0:
            raise RuntimeError("prepare after the eager catch-up of a sequence")
        self.start.fill_(d._len)
        for n in range(1, self.max_new + 1):
            self._graph(n)

    def pool_arrays(self, *, fed_ids: torch.Tensor, aux_history: torch.Tensor,
                    pending_seed: torch.Tensor, extra: tuple = ()):
        """Drafts one pool (graph replay) and reads back, with one host
        synchronisation, the pool rows ``[n_cand, 5]`` (token, parent index or
        -1, conditional and cumulative log-probability, depth; generation
        order) as a numpy array, plus each device tensor in ``extra``."""
        d = self.d
        t0 = time.perf_counter()
        L = fed_ids.shape[1]
        start = d._fed
        n_new = L + 1 - start
        if start == 0 or not 1 <= n_new <= self.max_new:
            raise ValueError("device drafting needs 1..max_new new rows after an eager catch-up")
        self.tokens[: n_new - 1].copy_(fed_ids[0, start:L])
        self.tokens[n_new - 1].copy_(pending_seed.reshape(()))
        self.aux[:n_new].copy_(aux_history[start - 1:L])
        self.start.fill_(d._len)
        t1 = time.perf_counter()
        self._graph(n_new).replay()
        t2 = time.perf_counter()
        self._host_out.copy_(self.out, non_blocking=True)
        hosts = []
        for t in extra:
            h = self._host_extra.get(t.data_ptr())
            if h is None or h.shape != t.shape or h.dtype != t.dtype:
                h = self._host_extra[t.data_ptr()] = torch.empty(t.shape, dtype=t.dtype).pin_memory()
            h.copy_(t, non_blocking=True)
            hosts.append(h.numpy())
        t3 = time.perf_counter()
        torch.cuda.current_stream(self.dev).synchronize()
        t4 = time.perf_counter()
        d._len += n_new       # committed rows + the seed row stay; tree rows are dropped
        d._fed = L + 1
        # Host-side split of the last call (ms): input copies, graph launch,
        # read-back launch, wait for the GPU.
        self.last_timing = {"inputs": (t1 - t0) * 1e3, "launch": (t2 - t1) * 1e3,
                            "readback": (t3 - t2) * 1e3, "wait": (t4 - t3) * 1e3}
        return self._host_out.numpy(), hosts

    def pool(self, *, fed_ids: torch.Tensor, aux_history: torch.Tensor,
             pending_seed: torch.Tensor) -> Eagle3DraftCandidatePool:
        n_new = fed_ids.shape[1] + 1 - self.d._fed
        arr, _ = self.pool_arrays(fed_ids=fed_ids, aux_history=aux_history, pending_seed=pending_seed)
        rows = arr.tolist()
        cands = []
        for i, (t, par, cond, _, depth) in enumerate(rows):
            par = int(par)
            pc = 0.0 if par < 0 else cands[par].cumulative_log_probability
            pp = () if par < 0 else cands[par].path
            cands.append(Eagle3DraftCandidate(i + 1, par + 1, int(depth), int(t), min(float(cond), 0.0),
                                              pc + min(float(cond), 0.0), i, pp + (int(t),)))
        steps = self.max_depth
        return Eagle3DraftCandidatePool(int(pending_seed.reshape(-1)[0]), self.top_k, self.max_depth,
                                        tuple(cands), path_score_calls=steps,
                                        draft_transformer_steps=steps, draft_forward_calls=steps,
                                        draft_query_tokens=n_new + sum(self.widths[:-1]))

    def release(self) -> None:
        self._graphs.clear()
