"""StreamingLLM sink + ring-window KV-cache oracle.  Test infrastructure only.

Restates the index math of the reference's ring buffer, which exists twice in
the reference with identical rules:

* C++: ``RingBufferKVCache::append`` (``csrc/kv_cache/ring_buffer.cu:109-141``),
  ``get_kv`` (``:143-200``), ``get_valid_length`` (``:203-209``);
* Python fallback: ``QExtractKVCache._get_write_pos`` (``qextract/kv_cache.py:114-119``),
  ``_build_indices`` (``:121-142``), ``valid_length`` (``:144-152``).

``count`` (``write_count`` in the reference) is the number of tokens written;
it advances only when the last layer is appended (``kv_cache.py:92-93``,
``ring_buffer.cu:138-140``), so every layer of one step writes the same slot.
"""

from __future__ import annotations

import numpy as np

__all__ = ["RingIndexOracle", "RingCacheOracle"]


class RingIndexOracle:
    """Pure index math for a ring of ``sink`` permanent slots followed by a
    ``window``-slot circular region."""

    def __init__(self, sink: int, window: int):
        assert sink >= 0 and window >= 1
        self.sink = sink
        self.window = window

    @property
    def capacity(self) -> int:
        return self.sink + self.window

    def write_pos(self, count: int) -> int:
        """Slot of the ``count``-th token (``kv_cache.py:114-119``)."""
        if count < self.sink:
            return count
        return self.sink + (count - self.sink) % self.window

    def valid_length(self, count: int) -> int:
        """``kv_cache.py:144-152``."""
        if count <= self.sink:
            return count
        return self.sink + min(count - self.sink, self.window)

    def indices(self, count: int) -> np.ndarray:
        """Slots in logical (oldest-first) order: sinks, then the ring starting
        at the oldest surviving token (``kv_cache.py:121-142``)."""
        idx = list(range(min(count, self.sink)))
        if count > self.sink:
            filled = min(count - self.sink, self.window)
            if count - self.sink <= self.window:
                start = 0
            else:
                start = (count - self.sink) % self.window
            idx.extend(self.sink + (start + i) % self.window for i in range(filled))
        return np.asarray(idx, dtype=np.int32)

    def positions(self, count: int) -> np.ndarray:
        """Absolute token position held by each slot of ``indices(count)``
        (sinks hold tokens ``0..sink-1``; the ring holds the newest
        ``filled`` tokens in order).  Derived from the same rules."""
        ns = min(count, self.sink)
        pos = list(range(ns))
        if count > self.sink:
            filled = min(count - self.sink, self.window)
            pos.extend(range(count - filled, count))
        return np.asarray(pos, dtype=np.int64)

    def slot_positions(self, count: int) -> np.ndarray:
        """Per physical slot, the absolute position stored there, or -1 if the
        slot is empty.  Length ``capacity``."""
        out = np.full(self.capacity, -1, dtype=np.int64)
        for t in range(count):
            out[self.write_pos(t)] = t
        return out


class RingCacheOracle:
    """Sequential, token-by-token restatement of the reference cache
    (``qextract/kv_cache.py:63-112`` fallback), extended with a batch axis.
    Storage per layer: ``[batch, sink + window, kv_heads, head_dim]``."""

    def __init__(self, num_layers, num_kv_heads, head_dim, sink_size=4,
                 window_size=4092, batch=1, dtype=np.float16):
        self.L, self.H, self.D = num_layers, num_kv_heads, head_dim
        self.B = batch
        self.idx = RingIndexOracle(sink_size, window_size)
        shape = (num_layers, batch, self.idx.capacity, num_kv_heads, head_dim)
        self.k = np.zeros(shape, dtype=dtype)
        self.v = np.zeros(shape, dtype=dtype)
        self.count = 0

    def append(self, new_k, new_v, layer_idx: int):
        """``new_k``: ``[H, D]`` (single token, batch 1, reference form),
        ``[T, H, D]`` (batch 1) or ``[B, T, H, D]``."""
        k = np.asarray(new_k)
        v = np.asarray(new_v)
        if k.ndim == 2:
            k, v = k[None, None], v[None, None]
        elif k.ndim == 3:
            k, v = k[None], v[None]
        assert k.shape[0] == self.B
        T = k.shape[1]
        for j in range(T):
            pos = self.idx.write_pos(self.count + j)
            self.k[layer_idx, :, pos] = k[:, j]
            self.v[layer_idx, :, pos] = v[:, j]
        if layer_idx == self.L - 1:
            self.count += T

    def get_kv(self, layer_idx: int, b: int = 0):
        ind = self.idx.indices(self.count)
        return self.k[layer_idx, b][ind], self.v[layer_idx, b][ind]

    @property
    def valid_length(self) -> int:
        return self.idx.valid_length(self.count)

    def memory_usage_bytes(self) -> int:
        """``qextract/kv_cache.py:159-163`` (fp16, K and V)."""
        return self.L * self.idx.capacity * self.H * self.D * 2 * 2 * self.B

    def reset(self):
        self.count = 0
        self.k[:] = 0
        self.v[:] = 0
