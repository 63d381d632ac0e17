"""One verify pass captured as a CUDA graph.

When every layer's expert cache holds all of its experts, the verify forward
(``eagle3_tree.py:1243-1250`` in the reference: the target over the seed +
tree tokens under the ancestor mask) needs no host synchronisation: routing,
grouping, the grouped SwiGLU launches and the combine all run from device
state.  ``VerifyGraph`` captures that forward once for a fixed tree size and
committed length and replays it, removing the per-op host launch cost of the
eager Hugging Face forward.

The KV cache's committed prefix is not modified by a replay: the captured
forward concatenates the prefix with the tree's keys/values into graph-owned
buffers, exactly as an eager ``DynamicCache.update`` followed by a rollback to
the prefix would.  The prefix tensors are kept alive for the graph's
lifetime, and the cache object is left holding them after capture.
"""
from __future__ import annotations

import torch

from .tree_attention import clear_mask_cache


class VerifyGraph:
    def __init__(self, model, kv_cache, *, q_len: int, device) -> None:
        self.model = model
        self.cache = kv_cache
        self.device = torch.device(device)
        self.prefix_len = kv_cache.get_seq_length()
        self.q_len = q_len
        self.ids = torch.zeros(1, q_len, dtype=torch.long, device=self.device)
        self.mask = torch.zeros(1, 1, q_len, self.prefix_len + q_len, dtype=torch.bool, device=self.device)
        self.pos = torch.zeros(1, q_len, dtype=torch.long, device=self.device)
        self._prefix = [(layer.keys, layer.values) for layer in kv_cache.layers]
        self.graph = None
        self.logits = None
        self.argmax = None

    def _restore_prefix(self) -> None:
        for layer, (k, v) in zip(self.cache.layers, self._prefix):
            layer.keys, layer.values = k, v

    def _forward(self):
        with torch.no_grad():
            out = self.model(input_ids=self.ids, attention_mask=self.mask, position_ids=self.pos,
                             past_key_values=self.cache, use_cache=True)
            return out.logits, out.logits[0].argmax(-1)

    def _require_resident(self) -> None:
        for layer in self.model.model.layers:
            experts = layer.mlp.experts
            if experts.cache.device_slot_table(experts._keys) is None:
                raise RuntimeError("VerifyGraph needs every expert of every layer resident "
                                   "(slots >= experts, caches warmed)")

    def load(self, ids, mask, pos) -> None:
        """Copy one tree's inputs into the graph's static buffers (async)."""
        self.ids.copy_(ids, non_blocking=True)
        self.mask.copy_(mask, non_blocking=True)
        self.pos.copy_(pos, non_blocking=True)

    def capture(self, ids, mask, pos, warmup: int = 2) -> None:
        self._require_resident()
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
