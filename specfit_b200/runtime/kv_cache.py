"""KV cache with reserved capacity: the verify pass writes in place.

The reference keeps a Hugging Face ``DynamicCache`` and rolls it back to the
committed prefix after every verify pass (``crop``,
src/specfit/runtime/eagle3_tree.py:1496-1500).  ``DynamicLayer.update``
concatenates, so every layer of every verify pass copies the whole cache
(for 8 requests x 4096 tokens that is 67 MB read + written per layer).
``ReservedCache`` is a ``DynamicCache`` whose layers reserve room for
``capacity`` tokens up front: ``update`` writes the new keys/values into the
reserved rows and returns views of the filled part, and ``crop`` only moves
the length.  Keys/values returned to attention are ``[B, Hkv, T, D]`` views
with row stride D and head stride capacity*D.

Because the buffers never move, a CUDA graph captured over a verify pass
writes the same rows on every replay, and rolling back is ``crop``.
"""
from __future__ import annotations

import torch
from transformers.cache_utils import DynamicCache, DynamicLayer


class ReservedLayer(DynamicLayer):
    def __init__(self, capacity: int) -> None:
        super().__init__()
        if capacity <= 0:
            raise ValueError("capacity must be positive")
        self.capacity = capacity
        self.length = 0
        self._kbuf = None
        self._vbuf = None

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.dtype, self.device = key_states.dtype, key_states.device
        b, h, n, d = key_states.shape
        cap = max(self.capacity, n)
        self._kbuf = torch.empty(b, h, cap, d, dtype=self.dtype, device=self.device)
        self._vbuf = torch.empty(b, h, cap, value_states.shape[-1], dtype=self.dtype, device=self.device)
        self.capacity = cap
        self.length = 0
        self._publish()
        self.is_initialized = True

    def _publish(self) -> None:
        self.keys = self._kbuf[..., : self.length, :]
        self.values = self._vbuf[..., : self.length, :]

    def _grow(self, need: int) -> None:
        cap = max(need, 2 * self.capacity)
        k = torch.empty(*self._kbuf.shape[:2], cap, self._kbuf.shape[3], dtype=self.dtype, device=self.device)
        v = torch.empty(*self._vbuf.shape[:2], cap, self._vbuf.shape[3], dtype=self.dtype, device=self.device)
        k[..., : self.length, :].copy_(self._kbuf[..., : self.length, :])
        v[..., : self.length, :].copy_(self._vbuf[..., : self.length, :])
        self._kbuf, self._vbuf, self.capacity = k, v, cap

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        if key_states.shape[:2] != self._kbuf.shape[:2]:
            raise ValueError("batch or head count differs from the reserved cache")
        end = self.length + key_states.shape[-2]
        if end > self.capacity:
            self._grow(end)
        self._kbuf[..., self.length:end, :].copy_(key_states)
        self._vbuf[..., self.length:end, :].copy_(value_states)
        self.length = end
        self._publish()
        return self.keys, self.values

    def get_seq_length(self) -> int:
        return self.length if self.is_initialized else 0

    def crop(self, max_length: int) -> None:
        if max_length < 0:
            max_length = self.get_seq_length() - abs(max_length)
        if self.get_seq_length() <= max_length:
            return
        self.length = max_length
        self._publish()

    def batch_repeat_interleave(self, repeats: int) -> None:
        if self.get_seq_length() > 0:
            self._kbuf = self._kbuf.repeat_interleave(repeats, dim=0)
            self._vbuf = self._vbuf.repeat_interleave(repeats, dim=0)
            self._publish()

    def batch_select_indices(self, indices: torch.Tensor) -> None:
        if self.get_seq_length() > 0:
            self._kbuf = self._kbuf[indices, ...]
            self._vbuf = self._vbuf[indices, ...]
            self._publish()


class ReservedCache(DynamicCache):
    """``DynamicCache`` with every full-attention layer reserving
    ``capacity`` tokens (context + the largest verification tree)."""

    def __init__(self, *, config, capacity: int) -> None:
        super().__init__(config=config)
        self.layers = [ReservedLayer(capacity) if type(layer) is DynamicLayer else layer
                       for layer in self.layers]
