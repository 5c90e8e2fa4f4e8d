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

__all__ = ["gqa_decode_attention_ref", "prefill_attention_ref", "ring_positions"]


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


def ring_positions(count: int, sink: int, window: int) -> tuple[np.ndarray, np.ndarray]:
    """(slots, positions) of the ring's valid tokens after ``count`` writes, in
    logical order: the sinks, then the window from its oldest surviving token
    (``kv_cache.py:121-142``); slot of position p >= sink is
    ``sink + (p - sink) % window`` (``kv_cache.py:114-119``)."""
    pos = list(range(min(count, sink)))
    if count > sink:
        filled = min(count - sink, window)
        pos += list(range(count - filled, count))
    pos = np.asarray(pos, dtype=np.int64)
    slots = np.where(pos < sink, pos, sink + (pos - sink) % window)
    return slots, pos


def prefill_attention_ref(q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray,
                          k_cache: np.ndarray, v_cache: np.ndarray, count: int, sink: int,
                          window: int, scale: float | None = None) -> np.ndarray:
    """One sequence: ``q`` ``[n, Hq, D]`` at positions ``count ..``; ``k_new``,
    ``v_new`` ``[n, Hkv, D]``; the ring ``k_cache``/``v_cache`` ``[S+W, Hkv, D]``
    after ``count`` tokens.  Key kp is visible to query p iff kp <= p and
    (kp < sink or kp > p - window): HF's causal mask with the StreamingLLM
    sink + window eviction, the chunk attended before its append.  fp32, one
    fp16 rounding.  Returns ``[n, Hq, D]``."""
    n, hq, d = q.shape
    hkv = k_new.shape[1]
    rep = hq // hkv
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    slots, cpos = ring_positions(count, sink, window)
    kk = np.concatenate([k_cache[slots], k_new]).astype(np.float32)  # [L, Hkv, D]
    vv = np.concatenate([v_cache[slots], v_new]).astype(np.float32)
    kpos = np.concatenate([cpos, count + np.arange(n)])
    qpos = count + np.arange(n)
    vis = (kpos[None, :] <= qpos[:, None]) & ((kpos[None, :] < sink) |
                                              (kpos[None, :] > qpos[:, None] - window))
    kf = np.repeat(kk, rep, axis=1)
    vf = np.repeat(vv, rep, axis=1)
    sc = np.einsum("nhd,lhd->hnl", q.astype(np.float32), kf) * np.float32(scale)
    sc = np.where(vis[None], sc, -np.inf)
    sc -= sc.max(axis=2, keepdims=True)
    pr = np.exp(sc)
    pr /= pr.sum(axis=2, keepdims=True)
    return np.einsum("hnl,lhd->nhd", pr, vf).astype(np.float16)
