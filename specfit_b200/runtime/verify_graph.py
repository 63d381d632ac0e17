"""One verify pass captured as a CUDA graph.

When every layer's expert cache holds all of its experts, or the caches are
device-managed (misses planned and filled on the device), the verify forward
(``eagle3_tree.py:1243-1250`` in the reference: the target over the seed +
tree tokens under the ancestor mask) needs no host synchronisation: routing,
grouping, fills, the grouped SwiGLU launches and the combine all run from
device state.  ``VerifyGraph`` captures that forward once for a fixed tree size and
committed length and replays it, removing the per-op host launch cost of the
eager Hugging Face forward.

The KV cache's committed prefix is not modified by a replay.  With a
``ReservedCache`` the captured forward writes the tree's keys/values into
the reserved rows after the prefix (the same rows on every replay) and the
rollback is ``crop``.  With a plain ``DynamicCache`` the captured forward
concatenates the prefix with the tree's keys/values into graph-owned
buffers, exactly as an eager ``update`` followed by a rollback would; the
prefix tensors are then kept alive for the graph's lifetime, and the cache
object is left holding them after capture.
"""
from __future__ import annotations

import torch

from .kv_cache import ReservedLayer
from .tree_attention import clear_mask_cache


class VerifyGraph:
    """``batch`` requests (the cache's batch) verify trees of ``q_len`` rows
    each; ``replay`` returns the argmax ``[q_len]`` (batch 1) or
    ``[batch, q_len]``."""

    def __init__(self, model, kv_cache, *, q_len: int, device, batch: int = 1, forward=None) -> None:
        self.model = model
        self.forward = forward if forward is not None else model  # e.g. a LeanQwen3Forward
        self.cache = kv_cache
        self.device = torch.device(device)
        self.prefix_len = kv_cache.get_seq_length()
        self.q_len = q_len
        self.batch = batch
        self.ids = torch.zeros(batch, q_len, dtype=torch.long, device=self.device)
        self.mask = torch.zeros(batch, 1, q_len, self.prefix_len + q_len, dtype=torch.bool,
                                device=self.device)
        self.pos = torch.zeros(batch, q_len, dtype=torch.long, device=self.device)
        self._prefix = [(layer.keys, layer.values) for layer in kv_cache.layers]
        self.graph = None
        self.logits = None
        self.argmax = None

    def _restore_prefix(self) -> None:
        for layer, (k, v) in zip(self.cache.layers, self._prefix):
            if isinstance(layer, ReservedLayer):
                layer.crop(self.prefix_len)
            else:
                layer.keys, layer.values = k, v

    def _forward(self):
        with torch.no_grad():
            out = self.forward(input_ids=self.ids, attention_mask=self.mask, position_ids=self.pos,
                               past_key_values=self.cache, use_cache=True)
            fused = getattr(out, "argmax", None)  # the lean forward's lm_head + argmax kernel
            if fused is not None:
                am = fused[0] if self.batch == 1 else fused
            else:
                am = out.logits[0].argmax(-1) if self.batch == 1 else out.logits.argmax(-1)
            return out.logits, am

    def _require_resident(self) -> None:
        for layer in self.model.model.layers:
            experts = layer.mlp.experts
            moe = getattr(experts, "moe", None)
            if moe is not None:  # expert-parallel layer: only the peer exchange is sync-free
                if not moe.use_peer:
                    raise RuntimeError("VerifyGraph needs the expert-parallel layers in peer mode")
                continue
            if experts.cache.device_managed:  # misses are planned and filled on the device
                continue
            if experts.cache.device_slot_table(experts._keys) is None:
                raise RuntimeError("VerifyGraph needs every expert of every layer resident "
                                   "(slots >= experts, caches warmed) or device-managed caches")

    def load(self, ids, mask, pos) -> None:
        """Copy one tree's inputs into the graph's static buffers (async)."""
        self.ids.copy_(ids, non_blocking=True)
        self.mask.copy_(mask, non_blocking=True)
        self.pos.copy_(pos, non_blocking=True)

    def capture(self, ids, mask, pos, warmup: int = 2) -> None:
        self._require_resident()
        for layer in self.cache.layers:
            if isinstance(layer, ReservedLayer) and layer.capacity < self.prefix_len + self.q_len:
                raise RuntimeError("the reserved KV cache must hold the prefix plus the tree")
        self.load(ids, mask, pos)
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._forward()
                self._restore_prefix()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        clear_mask_cache()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits, self.argmax = self._forward()
        clear_mask_cache()
        self._restore_prefix()

    def replay(self) -> torch.Tensor:
        """Runs the captured pass on the loaded inputs; returns the device
        argmax over the vocabulary per verification position."""
        self.graph.replay()
        return self.argmax
