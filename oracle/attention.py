"""GQA decode-attention oracle over the sink + ring window.  Test infrastructure only.

Parity unpinned: the reference has no attention kernel.  The semantics are
the reference cache's logical slot order (``qextract/kv_cache.py:121-142``,
``csrc/kv_cache/ring_buffer.cu:143-200``) combined with HF transformers'
Qwen3 eager attention (third-party: transformers 5.5.0,
``models/qwen3/modeling_qwen3.py:184-219`` -- ``repeat_kv`` maps query head
``h`` to KV head ``h // (Hq / Hkv)``; scores ``q k^T / sqrt(D)``; softmax in
fp32).  Keys are stored post-RoPE, so no rotation happens here.  All math is
fp32 with one fp16 rounding of the output.
"""

from __future__ import annotations

import numpy as np

__all__ = ["gqa_decode_attention_ref"]


def gqa_decode_attention_ref(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                             scale: float | None = None,
                             return_f32: bool = False) -> np.ndarray:
    """``q``: ``[Hq, D]``; ``k``, ``v``: ``[S, Hkv, D]`` (gathered in logical
    order; any order gives the same result up to fp32 rounding).
    Returns ``[Hq, D]``."""
    hq, d = q.shape
    s, hkv, d2 = k.shape
    assert d == d2 and hq % hkv == 0
    rep = hq // hkv
    if scale is None:
        scale = 1.0 / np.sqrt(d)
    qf = q.astype(np.float32)
    kf = np.repeat(k.astype(np.float32), rep, axis=1)  # [S, Hq, D]
    vf = np.repeat(v.astype(np.float32), rep, axis=1)
    scores = np.einsum("hd,shd->hs", qf, kf) * np.float32(scale)  # [Hq, S]
    m = scores.max(axis=1, keepdims=True)
    p = np.exp(scores - m)
    p /= p.sum(axis=1, keepdims=True)
    out = np.einsum("hs,shd->hd", p, vf)
    return out if return_f32 else out.astype(np.float16)
