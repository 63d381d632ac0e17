"""Expert-parallel MoE block over several GPUs of one node.

The reference runs on one GPU (it refuses ``device_count() != 1``,
scripts/run_specfit_main_comparison.py:465); sharding the 128 experts over
2/4/8 B200s is new.  Rank r owns the contiguous expert range
``[r*E/N, (r+1)*E/N)`` with its weights resident in HBM; every rank routes
its own tokens (attention stays data-parallel).  Per layer:

1. ``send``: the source packs one row per (token, destination rank) — the
   hidden state plus the token's local expert ids and routing weights on that
   rank (``sf_ep_send_pack``), so a token crosses NVLink at most once per
   rank;
2. the (pairs, routes) counts and then the rows are exchanged
   (``all_to_all_single``);
3. ``compute``: the destination groups the received routes by local expert
   (sources in rank order, tokens in order: the single-GPU groups), runs the
   grouped SwiGLU and packs one weighted output row per received route;
4. the rows travel back, and ``combine`` reduces every token's routes with
   the single-GPU combine (ascending expert id, bf16 rounding per add).

Two exchanges implement steps 2 and 4: NCCL ``all_to_all_single`` (one host
synchronisation per layer for the split sizes), and, when a ``PeerExchange``
is attached and ``use_peer`` is set, stores straight into the other ranks'
memory with device-side arrival counters (no host synchronisation, so a
verify pass can be captured in a CUDA graph).  Both give the same result.

So the block's output is the one-GPU output bit for bit.  The exchange goes
through NCCL over NVLink / NVSwitch; the phases are plain functions so a
test can also drive several ranks' phases on one device.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import ops


@dataclass
class RecvPlan:
    send_pairs: list
    send_routes: list
    recv_pairs: list
    recv_routes: list


def plan_from_counts(send_counts, recv_counts) -> RecvPlan:
    """Split sizes of both exchanges from the (pairs, routes) count tables
    ``[world, 2]`` sent and received (host values)."""
    s = [[int(a), int(b)] for a, b in send_counts]
    r = [[int(a), int(b)] for a, b in recv_counts]
    return RecvPlan([a for a, _ in s], [b for _, b in s], [a for a, _ in r], [b for _, b in r])


def all_to_all_rows(tensor: torch.Tensor, send_splits: list, recv_splits: list, group=None):
    out = torch.empty((sum(recv_splits), *tensor.shape[1:]), dtype=tensor.dtype, device=tensor.device)
    dist.all_to_all_single(out, tensor[: sum(send_splits)], output_split_sizes=recv_splits,
                           input_split_sizes=send_splits, group=group)
    return out


class ExpertParallelMoE:
    """One layer's experts on this rank of an expert-parallel group.

    ``local_storage``: ``[E/N, >= 3*H*I]`` packed expert slots
    (``[gate | up | down]``) of this rank's experts in ascending order,
    resident in HBM."""

    def __init__(self, *, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int,
                 local_storage: torch.Tensor, rank: int, world: int, group=None) -> None:
        if world < 1 or num_experts % world:
            raise ValueError("num_experts must be divisible by the world size")
        self.num_experts = num_experts
        self.top_k = top_k
        self.world = world
        self.rank = rank
        self.group = group
        self.local_experts = num_experts // world
        if local_storage.shape[0] != self.local_experts:
            raise ValueError("local_storage must hold exactly this rank's experts")
        self.hidden = hidden_size
        self.inter = intermediate_size
        self.storage = local_storage
        self.slot = torch.arange(self.local_experts, dtype=torch.int32, device=local_storage.device)
        self.last_plan: RecvPlan | None = None  # split sizes of the latest forward (host ints)
        self.peer = None  # PeerExchange shared by the layers of this rank, if any
        self.use_peer = False

    @classmethod
    def from_process_group(cls, group=None, **kw) -> "ExpertParallelMoE":
        return cls(rank=dist.get_rank(group), world=dist.get_world_size(group), group=group, **kw)

    # -- phases --------------------------------------------------------------

    def send(self, hidden: torch.Tensor, top_k_index: torch.Tensor,
             top_k_weights: torch.Tensor) -> ops.EpSend:
        return ops.ep_send_pack(hidden, top_k_index, top_k_weights, self.num_experts, self.world)

    def compute(self, recv_rows: torch.Tensor, pairs: int, routes: int, dtype: torch.dtype):
        """Weighted expert outputs for the received routes, one row each in
        (pair, slot) order."""
        if pairs == 0:
            return torch.empty(0, self.hidden, dtype=dtype, device=self.storage.device)
        d, return_src = ops.ep_recv_group(recv_rows, pairs, self.hidden, self.top_k,
                                          self.local_experts, dtype)
        xs, ws = ops.ep_recv_gather(recv_rows, d, self.hidden, dtype, routes)
        ys = ops.grouped_swiglu(xs, ws, d, self.slot, self.storage, self.hidden, self.inter)
        return ops.ep_return_pack(ys, return_src, routes)

    def combine(self, returned: torch.Tensor, send: ops.EpSend, top_k_index: torch.Tensor):
        return ops.ep_combine(returned, send, top_k_index)

    # -- one layer over the process group -------------------------------------

    def forward(self, hidden: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor):
        if self.use_peer:
            if self.peer is None:
                raise RuntimeError("use_peer is set but no PeerExchange is attached")
            return self.peer.layer(self, hidden, top_k_index, top_k_weights)
        send = self.send(hidden, top_k_index, top_k_weights)
        if self.world == 1:  # the exchange with oneself is the identity
            counts = send.counts.cpu()
            plan = self.last_plan = plan_from_counts(counts, counts)
            out_rows = self.compute(send.rows, plan.send_pairs[0], plan.send_routes[0], hidden.dtype)
            return self.combine(out_rows, send, top_k_index)
        recv_counts = torch.empty_like(send.counts)
        dist.all_to_all_single(recv_counts, send.counts, group=self.group)
        both = torch.stack((send.counts, recv_counts)).cpu()  # the one host sync per layer
        plan = self.last_plan = plan_from_counts(both[0], both[1])
        recv_rows = all_to_all_rows(send.rows, plan.send_pairs, plan.recv_pairs, self.group)
        out_rows = self.compute(recv_rows, sum(plan.recv_pairs), sum(plan.recv_routes), hidden.dtype)
        returned = all_to_all_rows(out_rows, plan.recv_routes, plan.send_routes, self.group)
        return self.combine(returned, send, top_k_index)

