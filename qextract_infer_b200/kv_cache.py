"""``QExtractKVCache``: the reference's Python cache wrapper
(``qextract/kv_cache.py:10-186``) over the native ring cache.

Same constructor, ``append`` / ``get_kv`` / ``valid_length`` /
``max_capacity`` / ``memory_usage_bytes`` / ``reset`` / ``repr``.  Unlike the
reference there is no pure-PyTorch fallback: without the native library the
constructor raises.  Additions: ``batch``, multi-token ``append`` and
``decode_attention``.
"""

from __future__ import annotations

import torch


class QExtractKVCache:
    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, sink_size: int = 4,
                 window_size: int = 4092, device: str = "cuda", dtype: torch.dtype = torch.float16,
                 batch: int = 1):
        if dtype != torch.float16:
            raise RuntimeError("QExtractKVCache stores float16 K/V")
        try:
            from ._C import RingBufferKVCache
        except ImportError as e:  # no silent fallback
            raise RuntimeError("QExtractKVCache needs the native library "
                               "(python -m qextract_infer_b200.build)") from e
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.sink_size = sink_size
        self.window_size = window_size
        self.total_size = sink_size + window_size
        self.device = device
        self.dtype = dtype
        self.batch = batch
        self._backend = RingBufferKVCache(num_layers, num_kv_heads, head_dim, sink_size,
                                          window_size, batch=batch, device=device)

    @property
    def write_count(self) -> int:
        return self._backend.get_total_written()

    def append(self, new_k: torch.Tensor, new_v: torch.Tensor, layer_idx: int) -> None:
        """Append one token (``[H, D]``) or a chunk (``[T, H, D]`` / ``[B, T, H, D]``)
        to ``layer_idx``; the token count advances after the last layer."""
        self._backend.append(new_k, new_v, layer_idx)

    def get_kv(self, layer_idx: int):
        """(k, v) in logical order, each ``[valid_len, H, D]`` (batch 1)."""
        return self._backend.get_kv(layer_idx)

    def decode_attention(self, q: torch.Tensor, layer_idx: int, softmax_scale=None):
        return self._backend.decode_attention(q, layer_idx, softmax_scale)

    @property
    def k_cache(self) -> torch.Tensor:
        return self._backend.k

    @property
    def v_cache(self) -> torch.Tensor:
        return self._backend.v

    @property
    def valid_length(self) -> int:
        return self._backend.get_valid_length()

    @property
    def max_capacity(self) -> int:
        return self.total_size

    def memory_usage_bytes(self) -> int:
        """``L * (S + W) * H * D * 2 bytes * 2 (K, V)`` per sequence
        (``qextract/kv_cache.py:159-163``)."""
        return self.num_layers * self.total_size * self.num_kv_heads * self.head_dim * 2 * 2 * self.batch

    def reset(self) -> None:
        self._backend.reset()

    def __repr__(self):
        mem_mb = self.memory_usage_bytes() / (1024 * 1024)
        return (f"QExtractKVCache(layers={self.num_layers}, kv_heads={self.num_kv_heads}, "
                f"head_dim={self.head_dim}, sink={self.sink_size}, window={self.window_size}, "
                f"valid={self.valid_length}/{self.total_size}, mem={mem_mb:.1f}MB)")
