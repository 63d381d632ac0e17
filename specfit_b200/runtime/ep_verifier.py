"""A Qwen3-MoE target whose MoE blocks run expert-parallel over a process group.

Each rank holds the non-expert weights (replicated) and the experts
``[r*E/N, (r+1)*E/N)`` of every layer, resident in HBM (16 per layer at
N = 8: 48 x 16 x 9.44 MB = 7.2 GB).  Attention is data-parallel: every rank
runs its own requests through the model, and each layer's MoE block
exchanges routed rows with the other ranks (``ExpertParallelMoE``).  Every
rank must therefore call ``forward`` the same number of times, in step.

The weights equal ``build_random_offloaded_qwen3``'s for the same seed (the
experts are drawn from the same per-layer generators and sliced), so a
one-rank group reproduces the single-GPU model, and the expert-parallel
block keeps the single-GPU block's results bit for bit.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

from .. import synthetic
from .expert_parallel import ExpertParallelMoE
from .moe_block import Qwen3B200SparseMoeBlock, Qwen3B200TopKRouter
from .qwen3_verifier import materialize_random_, qwen3_moe_config
from .tree_attention import install as install_tree_attention


class ExpertParallelExperts(nn.Module):
    """``experts`` child of the sparse-MoE block with the
    ``Qwen3OffloadedExperts`` call signature (hidden, top_k_index,
    top_k_weights), backed by this rank's share of the layer's experts."""

    def __init__(self, layer_id: int, moe: ExpertParallelMoE) -> None:
        super().__init__()
        self.layer_id = layer_id
        self.moe = moe
        self.num_experts = moe.num_experts

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                top_k_weights: torch.Tensor) -> torch.Tensor:
        return self.moe.forward(hidden_states, top_k_index, top_k_weights)


def local_expert_block(layer: int, seed: int, experts: int, elems: int, rank: int, world: int,
                       device, std: float = 0.02, dtype=torch.bfloat16) -> torch.Tensor:
    """Rank ``rank``'s experts of one layer, drawn exactly as
    ``ExpertHostPool.fill_random`` draws the whole layer."""
    g = torch.Generator(device=device).manual_seed(seed + layer)
    full = torch.randn(experts, elems, generator=g, device=device, dtype=torch.float32).mul_(std)
    per = experts // world
    out = full[rank * per:(rank + 1) * per].to(dtype)
    del full
    return out


@dataclass
class LoadedEpQwen3:
    model: nn.Module
    rank: int
    world: int
    peer: object = None  # PeerExchange shared by every layer, once attached

    def moes(self) -> list:
        return [layer.mlp.experts.moe for layer in self.model.model.layers]

    def attach_peer_exchange(self, max_tokens: int, group=None, **kw):
        """Allocate and map the peer regions (collective over the group) and
        give every layer the same exchange (layers run one after another)."""
        from .ep_peer import PeerExchange

        m = self.moes()[0]
        self.peer = PeerExchange(rank=self.rank, world=self.world, max_tokens=max_tokens,
                                 hidden_size=m.hidden, top_k=m.top_k, local_experts=m.local_experts,
                                 device=m.storage.device, dtype=m.storage.dtype, group=group, **kw)
        for moe in self.moes():
            moe.peer = self.peer
        return self.peer

    def use_peer(self, on: bool) -> None:
        for moe in self.moes():
            moe.use_peer = bool(on)

    def close(self) -> None:
        torch.cuda.synchronize()
        if self.peer is not None:
            self.peer.close()
            self.peer = None


def build_random_ep_qwen3(*, device, rank: int, world: int, group=None,
                          num_layers: int = synthetic.NUM_LAYERS, seed: int = 0,
                          dtype=torch.bfloat16, config=None, std: float = 0.02) -> LoadedEpQwen3:
    from transformers import Qwen3MoeForCausalLM

    device = torch.device(device)
    cfg = config if config is not None else qwen3_moe_config(num_layers)
    cfg._attn_implementation = "sdpa"
    hidden, inter = cfg.hidden_size, cfg.moe_intermediate_size
    if cfg.num_experts % world:
        raise ValueError("the experts must shard evenly over the ranks")
    blocks = [local_expert_block(l, seed, cfg.num_experts, 3 * hidden * inter, rank, world, device,
                                 std, dtype) for l in range(cfg.num_hidden_layers)]
    with torch.device("meta"):
        model = Qwen3MoeForCausalLM(cfg)
    for l, layer in enumerate(model.model.layers):
        gate = Qwen3B200TopKRouter(cfg.num_experts, hidden, cfg.num_experts_per_tok,
                                   cfg.norm_topk_prob, device="meta")
        layer.mlp = Qwen3B200SparseMoeBlock(gate, nn.Identity())
    materialize_random_(model, cfg, device, seed, std, dtype)
    for l, layer in enumerate(model.model.layers):
        moe = ExpertParallelMoE(num_experts=cfg.num_experts, top_k=cfg.num_experts_per_tok,
                                hidden_size=hidden, intermediate_size=inter, local_storage=blocks[l],
                                rank=rank, world=world, group=group)
        layer.mlp.experts = ExpertParallelExperts(l, moe)
    install_tree_attention(model)
    return LoadedEpQwen3(model, rank, world)
