"""Verification trees.

``Eagle3DraftTree`` mirrors ``src/specfit/runtime/eagle3_types.py:302-502``:
the same fields, validation rules and error messages, and the same
verification inputs — token ids (seed first, :429-433), position ids (seed at
``base``, node at ``base + depth``, :435-448), the ancestor attention mask
(:450-473) and the greedy accepted path (:475-502).  New here:
``verification_tree_bits`` gives the packed ancestor bitmask the tree
attention kernel consumes, built on the host in O(nodes * words) instead of a
per-element mask walk.
"""
from __future__ import annotations

from dataclasses import dataclass
from math import isclose, isfinite, log

import numpy as np
import torch


def _is_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


@dataclass(frozen=True, slots=True)
class Eagle3DraftTree:
    token_ids: tuple
    parent_ids: tuple
    depths: tuple
    conditional_probabilities: tuple
    cumulative_log_probabilities: tuple
    source_raw_ids: tuple = ()

    def __post_init__(self) -> None:
        n = len(self.token_ids)
        if not self.source_raw_ids and n:
            object.__setattr__(self, "source_raw_ids", tuple(range(1, n + 1)))
        fields = (self.parent_ids, self.depths, self.conditional_probabilities,
                  self.cumulative_log_probabilities, self.source_raw_ids)
        if any(len(f) != n for f in fields):
            raise ValueError("draft tree fields must have equal lengths")
        if any(not _is_int(r) or r <= 0 for r in self.source_raw_ids):
            raise ValueError("source raw IDs must be positive integers")
        if len(set(self.source_raw_ids)) != n:
            raise ValueError("source raw IDs must be unique")
        siblings: dict = {}
        cumulative = {0: 0.0}
        for node, (tok, par, dep, p, cum) in enumerate(zip(
                self.token_ids, self.parent_ids, self.depths, self.conditional_probabilities,
                self.cumulative_log_probabilities), start=1):
            if not _is_int(tok) or tok < 0:
                raise ValueError("tree token IDs must be non-negative integers")
            if not _is_int(par) or not 0 <= par < node:
                raise ValueError("tree parents must precede their children")
            if not _is_int(dep):
                raise ValueError("tree depths must contain integers")
            parent_depth = 0 if par == 0 else self.depths[par - 1]
            if dep != parent_depth + 1:
                raise ValueError("tree node depth differs from its parent")
            if not isfinite(p) or not 0.0 < p <= 1.0:
                raise ValueError("conditional probabilities must be in (0, 1]")
            if not isfinite(cum):
                raise ValueError("cumulative log probabilities must be finite")
            if not isclose(cum, cumulative[par] + log(p), rel_tol=1e-5, abs_tol=1e-6):
                raise ValueError("cumulative score differs from its parent and conditional probability")
            kids = siblings.setdefault(par, set())
            if tok in kids:
                raise ValueError("siblings must use distinct token IDs")
            kids.add(tok)
            cumulative[node] = cum

    @property
    def draft_node_count(self) -> int:
        return len(self.token_ids)

    @property
    def verification_raw_ids(self) -> tuple:
        return (0,) + self.source_raw_ids

    def raw_ids_for_verification_positions(self, positions: tuple) -> tuple:
        if any(not _is_int(p) or not 0 <= p <= self.draft_node_count for p in positions):
            raise ValueError("verification positions are outside the draft tree")
        raw = self.verification_raw_ids
        return tuple(raw[p] for p in positions)

    def verification_token_ids(self, pending_seed: torch.Tensor) -> torch.Tensor:
        if pending_seed.shape != (1, 1):
            raise ValueError("pending_seed must have shape [1, 1]")
        drafts = pending_seed.new_tensor(self.token_ids).unsqueeze(0)
        return torch.cat((pending_seed, drafts), dim=1)

    def verification_position_ids(self, *, base_kv_length: int, device) -> torch.Tensor:
        if base_kv_length < 0:
            raise ValueError("base_kv_length must be non-negative")
        pos = (base_kv_length,) + tuple(base_kv_length + d for d in self.depths)
        return torch.tensor(pos, dtype=torch.long, device=device).unsqueeze(0)

    def _ancestor_rows(self) -> list:
        rows = [1]  # python-int bitsets over verification positions
        for node, parent in enumerate(self.parent_ids, start=1):
            rows.append(rows[parent] | (1 << node))
        return rows

    def verification_attention_mask(self, *, base_kv_length: int, device) -> torch.Tensor:
        if base_kv_length < 0:
            raise ValueError("base_kv_length must be non-negative")
        q = 1 + self.draft_node_count
        rows = self._ancestor_rows()
        tree = torch.tensor([[(r >> j) & 1 for j in range(q)] for r in rows], dtype=torch.bool)
        mask = torch.ones(1, 1, q, base_kv_length + q, dtype=torch.bool)
        mask[0, 0, :, base_kv_length:] = tree
        return mask.to(device)

    def verification_tree_bits(self, device) -> torch.Tensor:
        """``int32[1+n, ceil((1+n)/32)]``: bit j of row i set when verification
        position j is i or one of its ancestors."""
        q = 1 + self.draft_node_count
        words = (q + 31) // 32
        data = []
        for r in self._ancestor_rows():
            for w in range(words):
                v = (r >> (32 * w)) & 0xFFFFFFFF
                data.append(v - (1 << 32) if v >= (1 << 31) else v)
        return torch.tensor(data, dtype=torch.int32).view(q, words).to(device)

    def accepted_path(self, verifier_token_ids: torch.Tensor) -> tuple:
        if verifier_token_ids.shape != (1, 1 + self.draft_node_count):
            raise ValueError("verifier tokens do not match the draft tree")
        verifier = [int(v) for v in verifier_token_ids[0].tolist()]
        children: dict = {}
        for node, parent in enumerate(self.parent_ids, start=1):
            children.setdefault(parent, []).append(node)
        accepted = []
        parent = 0
        while True:
            want = verifier[parent]
            match = [n for n in children.get(parent, ()) if self.token_ids[n - 1] == want]
            if not match:
                break
            if len(match) != 1:
                raise RuntimeError("target token matches multiple sibling nodes")
            parent = match[0]
            accepted.append(parent)
        return tuple(accepted)


def _check_nonneg_int(value, message: str) -> None:
    if not _is_int(value) or value < 0:
        raise ValueError(message)


@dataclass(frozen=True, slots=True)
class Eagle3DraftCandidate:
    """One drafted candidate (``src/specfit/runtime/eagle3_types.py:86-143``):
    raw ids count from 1 in generation order, parents precede children."""

    raw_id: int
    parent_raw_id: int
    depth: int
    target_token_id: int
    conditional_log_probability: float
    cumulative_log_probability: float
    generation_ordinal: int
    path: tuple

    def __post_init__(self) -> None:
        if not _is_int(self.raw_id) or self.raw_id <= 0:
            raise ValueError("candidate raw IDs must be positive integers")
        if not _is_int(self.parent_raw_id) or not 0 <= self.parent_raw_id < self.raw_id:
            raise ValueError("candidate parents must precede their children")
        if not _is_int(self.depth) or self.depth <= 0:
            raise ValueError("candidate depths must be positive integers")
        _check_nonneg_int(self.target_token_id, "candidate token IDs must be non-negative integers")
        if not isfinite(self.conditional_log_probability) or self.conditional_log_probability > 0.0:
            raise ValueError("conditional log probabilities must be finite and <= 0")
        if not isfinite(self.cumulative_log_probability):
            raise ValueError("cumulative log probabilities must be finite")
        _check_nonneg_int(self.generation_ordinal, "generation ordinals must be non-negative integers")
        if not isinstance(self.path, tuple):
            raise ValueError("candidate paths must be immutable tuples")
        if len(self.path) != self.depth or self.path[-1] != self.target_token_id:
            raise ValueError("candidate path must end at the candidate token")

    @property
    def conditional_probability(self) -> float:
        from math import exp

        return exp(self.conditional_log_probability)


@dataclass(frozen=True, slots=True)
class Eagle3DraftCandidatePool:
    """A drafted candidate pool (``eagle3_types.py:146-300``) and its
    ancestor-closed sub-trees (``to_tree``)."""

    seed_token_id: int
    top_k: int
    max_depth: int
    candidates: tuple
    path_score_calls: int
    draft_transformer_steps: int
    draft_forward_calls: int = 0
    draft_query_tokens: int = 0

    def __post_init__(self) -> None:
        _check_nonneg_int(self.seed_token_id, "candidate-pool seed must be a non-negative token ID")
        if not _is_int(self.top_k) or self.top_k <= 0:
            raise ValueError("candidate-pool top_k must be a positive integer")
        if not _is_int(self.max_depth) or self.max_depth <= 0:
            raise ValueError("candidate-pool depth must be a positive integer")
        if not isinstance(self.candidates, tuple) or not self.candidates:
            raise ValueError("candidate pool must contain at least one node")
        if not _is_int(self.path_score_calls) or self.path_score_calls <= 0:
            raise ValueError("path_score_calls must be a positive integer")
        if not _is_int(self.draft_transformer_steps) or self.draft_transformer_steps < self.path_score_calls:
            raise ValueError("draft_transformer_steps must cover every path score call")
        for name in ("draft_forward_calls", "draft_query_tokens"):
            _check_nonneg_int(getattr(self, name), f"{name} must be a non-negative integer")
        seen: dict = {}
        sibling_tokens: dict = {}
        for expected, c in enumerate(self.candidates, start=1):
            if c.raw_id != expected:
                raise ValueError("candidate raw IDs must be consecutive")
            if c.generation_ordinal != expected - 1:
                raise ValueError("candidate ordinals must follow generation order")
            if c.depth > self.max_depth:
                raise ValueError("candidate depth exceeds the pool depth")
            if c.parent_raw_id == 0:
                pdepth, ppath, pscore = 0, (), 0.0
            else:
                parent = seen.get(c.parent_raw_id)
                if parent is None:
                    raise ValueError("candidate parent is absent from the pool")
                pdepth, ppath, pscore = parent.depth, parent.path, parent.cumulative_log_probability
            if c.depth != pdepth + 1:
                raise ValueError("candidate depth differs from its parent")
            if c.path != ppath + (c.target_token_id,):
                raise ValueError("candidate path differs from its parent path")
            if not isclose(c.cumulative_log_probability, pscore + c.conditional_log_probability,
                           rel_tol=1e-5, abs_tol=1e-6):
                raise ValueError("candidate cumulative score is inconsistent")
            toks = sibling_tokens.setdefault(c.parent_raw_id, set())
            if c.target_token_id in toks:
                raise ValueError("candidate siblings must use distinct token IDs")
            toks.add(c.target_token_id)
            seen[c.raw_id] = c

    @property
    def nodes(self) -> tuple:
        """The candidates, under the name the selection code reads."""
        return self.candidates

    @property
    def raw_candidate_count(self) -> int:
        return len(self.candidates)

    @property
    def actual_depth(self) -> int:
        return max(c.depth for c in self.candidates)

    def to_tree(self, selected_raw_ids: tuple) -> Eagle3DraftTree:
        if not isinstance(selected_raw_ids, tuple):
            raise ValueError("selected raw IDs must be an immutable tuple")
        if any(not _is_int(r) or r <= 0 for r in selected_raw_ids):
            raise ValueError("selected raw IDs must be positive integers")
        if len(set(selected_raw_ids)) != len(selected_raw_ids):
            raise ValueError("selected raw IDs must be unique")
        by_raw = {c.raw_id: c for c in self.candidates}
        try:
            chosen = [by_raw[r] for r in selected_raw_ids]
        except KeyError as error:
            raise ValueError("selected raw ID is absent from the pool") from error
        keep = set(selected_raw_ids)
        if any(c.parent_raw_id != 0 and c.parent_raw_id not in keep for c in chosen):
            raise ValueError("selected candidates must be ancestor-closed")
        chosen.sort(key=lambda c: c.generation_ordinal)
        node_of = {c.raw_id: i for i, c in enumerate(chosen, start=1)}
        return Eagle3DraftTree(
            token_ids=tuple(c.target_token_id for c in chosen),
            parent_ids=tuple(0 if c.parent_raw_id == 0 else node_of[c.parent_raw_id] for c in chosen),
            depths=tuple(c.depth for c in chosen),
            conditional_probabilities=tuple(c.conditional_probability for c in chosen),
            cumulative_log_probabilities=tuple(c.cumulative_log_probability for c in chosen),
            source_raw_ids=tuple(c.raw_id for c in chosen),
        )


def tree_from_arrays(selected_raw_ids: tuple, token_ids, parent_raw_ids, depths, conditional_log_probs,
                     cumulative_log_probs) -> Eagle3DraftTree:
    """``Eagle3DraftCandidatePool.to_tree`` for a pool held as arrays indexed
    by raw id - 1 (parent raw id 0 = the seed; generation order = raw id
    order), for callers that never build the candidate objects.  Same checks
    on the selection; the tree validates itself."""
    from math import exp

    n = len(token_ids)
    if not isinstance(selected_raw_ids, tuple):
        raise ValueError("selected raw IDs must be an immutable tuple")
    if any(not _is_int(r) or r <= 0 for r in selected_raw_ids):
        raise ValueError("selected raw IDs must be positive integers")
    if len(set(selected_raw_ids)) != len(selected_raw_ids):
        raise ValueError("selected raw IDs must be unique")
    if any(r > n for r in selected_raw_ids):
        raise ValueError("selected raw ID is absent from the pool")
    keep = set(selected_raw_ids)
    chosen = sorted(int(r) for r in selected_raw_ids)
    if any(int(parent_raw_ids[r - 1]) != 0 and int(parent_raw_ids[r - 1]) not in keep for r in chosen):
        raise ValueError("selected candidates must be ancestor-closed")
    node_of = {r: i for i, r in enumerate(chosen, start=1)}
    rows = [r - 1 for r in chosen]
    # One gather per field (numpy arrays or sequences), then plain Python values.
    tok, par, dep, cond, cum = (np.asarray(f)[rows].tolist() for f in (
        token_ids, parent_raw_ids, depths, conditional_log_probs, cumulative_log_probs))
    return Eagle3DraftTree(
        token_ids=tuple(int(t) for t in tok),
        parent_ids=tuple(0 if int(p) == 0 else node_of[int(p)] for p in par),
        depths=tuple(int(d) for d in dep),
        conditional_probabilities=tuple(exp(float(c)) for c in cond),
        cumulative_log_probabilities=tuple(float(c) for c in cum),
        source_raw_ids=tuple(chosen),
    )
