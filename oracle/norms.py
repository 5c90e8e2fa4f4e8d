"""RMSNorm and SwiGLU oracles in numpy.  Test infrastructure only."""

from __future__ import annotations

import numpy as np

__all__ = ["rmsnorm_ref", "swiglu_ref", "swiglu_ref_single_round"]


def rmsnorm_ref(x: np.ndarray, weight: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """``fp16((x * rsqrt(mean(x^2) + eps)) * w)`` in fp32
    (``tests/test_rmsnorm.py:12-18``; kernel math ``csrc/kernels/rmsnorm.cu:134,153``).
    ``x`` is ``[..., H]`` fp16, ``weight`` ``[H]`` fp16."""
    xf = x.astype(np.float32)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    r = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    return ((xf * r) * weight.astype(np.float32)).astype(np.float16)


def _silu_f32(g: np.ndarray) -> np.ndarray:
    gf = g.astype(np.float32)
    with np.errstate(over="ignore"):
        return gf / (np.float32(1.0) + np.exp(-gf))


def swiglu_ref(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """``fp16(silu(g.float())) * up`` -- the reference test's two-rounding form
    (``tests/test_swiglu.py:11-13``): silu in fp32 rounded to fp16, then an
    fp16 multiply (one more rounding)."""
    s = _silu_f32(gate).astype(np.float16)
    return (s.astype(np.float32) * up.astype(np.float32)).astype(np.float16)


def swiglu_ref_single_round(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """``fp16(silu(g) * u)`` with fp32 math and one rounding -- the reference
    kernel's math (``csrc/kernels/swiglu.cu:65-68``) and the fp32 bench
    reference (``benchmarks/bench_kernels.py:68-69``)."""
    return (_silu_f32(gate) * up.astype(np.float32)).astype(np.float16)
