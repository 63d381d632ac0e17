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
