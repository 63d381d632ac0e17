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

Static mode (``ReservedCache.set_static``) serves graphs that must work at
any committed length: ``update`` writes at the device-side offset and returns
the whole reserved buffer, and the attention mask (over all reserved rows)
decides what is visible.  Buffers start zeroed, so rows never written hold
finite values that a zero attention weight cancels.
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
        self.static_offset = None  # device int64 scalar: write position in static mode
        self.static_length = 0     # sequence length reported in static mode
        self._arange = None

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.dtype, self.device = key_states.dtype, key_states.device
        b, h, n, d = key_states.shape
        cap = max(self.capacity, n)
        self._kbuf = torch.zeros(b, h, cap, d, dtype=self.dtype, device=self.device)
        self._vbuf = torch.zeros(b, h, cap, value_states.shape[-1], dtype=self.dtype, device=self.device)
        self.capacity = cap
        self.length = 0
        self._publish()
        self.is_initialized = True

    def _publish(self) -> None:
        self.keys = self._kbuf[..., : self.length, :]
        self.values = self._vbuf[..., : self.length, :]

    def _grow(self, need: int) -> None:
        cap = max(need, 2 * self.capacity)
        k = torch.zeros(*self._kbuf.shape[:2], cap, self._kbuf.shape[3], dtype=self.dtype, device=self.device)
        v = torch.zeros(*self._vbuf.shape[:2], cap, self._vbuf.shape[3], dtype=self.dtype, device=self.device)
        k[..., : self.length, :].copy_(self._kbuf[..., : self.length, :])
        v[..., : self.length, :].copy_(self._vbuf[..., : self.length, :])
        self._kbuf, self._vbuf, self.capacity = k, v, cap

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        if key_states.shape[:2] != self._kbuf.shape[:2]:
            raise ValueError("batch or head count differs from the reserved cache")
        if self.static_offset is not None:
            n = key_states.shape[-2]
            if self._arange is None or self._arange.numel() < n:
                self._arange = torch.arange(max(n, 16), device=self.device)
            rows = self.static_offset + self._arange[:n]
            self._kbuf.index_copy_(-2, rows, key_states)
            self._vbuf.index_copy_(-2, rows, value_states)
            return self._kbuf, self._vbuf
        end = self.length + key_states.shape[-2]
        if end > self.capacity:
            self._grow(end)
        self._kbuf[..., self.length:end, :].copy_(key_states)
        self._vbuf[..., self.length:end, :].copy_(value_states)
        self.length = end
        self._publish()
        return self.keys, self.values

    def get_seq_length(self) -> int:
        if self.static_offset is not None:
            return self.static_length
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

    def set_static(self, offset: torch.Tensor | None, reported_length: int = 0) -> None:
        """Enter static mode (writes at the device scalar ``offset``, whole
        buffers returned, ``reported_length`` as the sequence length) or, with
        ``None``, leave it."""
        for layer in self.layers:
            if isinstance(layer, ReservedLayer):
                if offset is not None and not layer.is_initialized:
                    raise RuntimeError("static mode needs initialised layers (run a prefill first)")
                layer.static_offset = offset
                layer.static_length = reported_length

    def set_length(self, length: int) -> None:
        """Host-side length of every reserved layer (after a static pass)."""
        for layer in self.layers:
            if isinstance(layer, ReservedLayer):
                if length > layer.capacity:
                    raise ValueError("length exceeds the reserved capacity")
                layer.length = length
                layer._publish()


def compact_tree_cache_(cache, *, base_kv_length: int, verification_positions: tuple,
                        verification_node_count: int) -> None:
    """Keep the accepted verification rows: rows ``base + p`` for ``p`` in
    ``verification_positions`` move to ``base, base + 1, ...`` and the cache
    is cropped after them (``_compact_tree_cache``,
    src/specfit/runtime/eagle3_tree.py:833-858).  Works on any cache whose
    layers expose ``keys`` / ``values``; reserved layers move rows inside
    their buffers."""
    expected = base_kv_length + verification_node_count
    n = len(verification_positions)
    layers = cache.layers
    if (layers and all(isinstance(l, ReservedLayer) and l.is_initialized for l in layers)
            and layers[0]._kbuf.is_cuda and layers[0]._kbuf.shape[0] == 1
            and layers[0]._kbuf.dtype == torch.bfloat16):
        if any(l.get_seq_length() != expected for l in layers):
            raise RuntimeError("target cache layer has an unexpected length")
        _compact_native(cache, base_kv_length, verification_positions)
        cache.crop(base_kv_length + n)
        return
    src = None
    for layer in layers:
        if layer.get_seq_length() != expected:
            raise RuntimeError("target cache layer has an unexpected length")
        if src is None or src.device != layer.keys.device:
            src = torch.tensor([base_kv_length + p for p in verification_positions], dtype=torch.long,
                               device=layer.keys.device)
        k = layer.keys.index_select(-2, src)  # owns its result: overlapping moves are safe
        v = layer.values.index_select(-2, src)
        layer.keys[..., base_kv_length:base_kv_length + n, :].copy_(k)
        layer.values[..., base_kv_length:base_kv_length + n, :].copy_(v)
    cache.crop(base_kv_length + n)


def _compact_native(cache, base: int, positions: tuple) -> None:
    """All layers' accepted rows moved in two launches (``sf_kv_compact``)."""
    from .. import _native as N
    from .. import ops

    layers = cache.layers
    l0 = layers[0]
    dev = l0._kbuf.device
    ptrs = tuple(p for l in layers for p in (l._kbuf.data_ptr(), l._vbuf.data_ptr()))
    table = getattr(cache, "_compact_table", None)
    if table is None or table[0] != ptrs:
        heads, cap, d = l0._kbuf.shape[1], l0.capacity, l0._kbuf.shape[3]
        if any(l._kbuf.shape[1:] != l0._kbuf.shape[1:] or l.capacity != cap for l in layers):
            raise ValueError("every layer must share one reserved shape")
        dev_ptrs = torch.tensor(ptrs, dtype=torch.int64, device=dev)
        stage = torch.empty(2 * len(layers) * 16 * heads * d, dtype=torch.bfloat16, device=dev)
        table = cache._compact_table = (ptrs, dev_ptrs, stage, heads, cap, d)
    _, dev_ptrs, stage, heads, cap, d = table
    n = len(positions)
    if n > 16:
        raise ValueError("at most 16 kept rows per compaction")
    src = torch.tensor(positions, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
    N.check(N.lib.sf_kv_compact(dev_ptrs.data_ptr(), len(layers), heads, d, cap * d, base,
                                src.data_ptr(), n, stage.data_ptr(),
                                torch.cuda.current_stream(dev).cuda_stream), "sf_kv_compact")
    ops._launched(2)
