"""The sparse-MoE block of a Qwen3-MoE decoder layer on the B200 kernels.

``Qwen3B200TopKRouter`` replaces ``Qwen3MoeTopKRouter`` (transformers/models/
qwen3_moe/modeling_qwen3_moe.py:254-272) and ``Qwen3B200SparseMoeBlock``
replaces ``Qwen3MoeSparseMoeBlock`` (:275-287) at ``layer.mlp``.  The block
keeps a ``gate`` child whose forward returns ``(probs, weights, indices)`` so
route-capture hooks on ``layer.mlp.gate`` read ``output[2]`` exactly as the
reference's runner does (scripts/run_specfit_main_comparison.py:536-566), and
an ``experts`` child with the ``Qwen3OffloadedExperts`` interface.
"""
from __future__ import annotations

import torch
from torch import nn

from .. import ops


class Qwen3B200TopKRouter(nn.Module):
    def __init__(self, num_experts: int, hidden_size: int, top_k: int, norm_topk_prob: bool = True,
                 *, device=None, dtype=None) -> None:
        super().__init__()
        self.top_k = top_k
        self.num_experts = num_experts
        self.norm_topk_prob = norm_topk_prob
        self.hidden_dim = hidden_size
        self.weight = nn.Parameter(torch.zeros(num_experts, hidden_size, device=device, dtype=dtype),
                                   requires_grad=False)

    def forward(self, hidden_states: torch.Tensor):
        h = hidden_states.reshape(-1, self.hidden_dim)
        return ops.router_topk(h, self.weight, self.top_k, self.norm_topk_prob)


class Qwen3B200SparseMoeBlock(nn.Module):
    def __init__(self, gate: Qwen3B200TopKRouter, experts: nn.Module) -> None:
        super().__init__()
        self.gate = gate
        self.experts = experts

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        shape = hidden_states.shape
        flat = hidden_states.reshape(-1, shape[-1])
        _, routing_weights, selected = self.gate(flat)
        out = self.experts(flat, selected, routing_weights)
        return out.reshape(shape)
