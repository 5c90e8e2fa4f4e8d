"""Operator module with the names, arguments and error behaviour of the
reference's ``qextract._C`` (pybind11 module, ``csrc/binding.cpp:32-74``),
implemented over the C ABI of ``libqx_b200.so`` (``include/qx_b200.h``).

Differences from the reference, all widening what it accepts:

* ``w4a16_gemv`` / ``w4a16_lora_gemv`` take ``input`` of shape ``[K]`` or
  ``[..., K]`` and return ``[N]`` / ``[..., N]`` (the reference reads
  ``input.size(0)`` as K, ``csrc/kernels/w4a16_lora_gemv.cu:285``, so 2-D
  inputs silently computed nothing);
* ``zeros`` may be the reference's fp16 ``[G, N]`` or GPTQ-packed
  ``qzeros`` int32 ``[G, N/8]`` (``zero_offset=1`` for the GPTQ-v1 "+1"
  storage);
* ``RingBufferKVCache.append`` also takes ``[T, H, D]`` and ``[B, T, H, D]``
  chunks, and the cache adds ``decode_attention``.

Every op runs on the current torch CUDA stream and raises if the native
library is missing or the inputs are not CUDA tensors: there is no CPU path.
"""

from __future__ import annotations

import functools
import math

import numpy as np
import torch

from . import _lib, _workspace

__all__ = ["fused_rmsnorm", "fused_swiglu", "w4a16_gemv", "w4a16_lora_gemv",
           "RingBufferKVCache", "decode_attention", "ring_slot_indices"]

_LIB = _lib.load()  # fail at import time if the native library is absent
_SUPPORTED_RANKS = (8, 16, 32, 48, 64, 128)


def _check_input(t: torch.Tensor, name: str):
    # same conditions as CHECK_CUDA_INPUT (csrc/include/common.h:20-28)
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_fp16(t: torch.Tensor, name: str):
    if t.dtype != torch.float16:
        raise RuntimeError(f"{name} must be float16, got {t.dtype}")


def _stream(device: torch.device):
    return torch.cuda.current_stream(device)


_raw_stream_of = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _raw_stream(device: torch.device) -> int:
    """cudaStream_t of the current torch stream of ``device`` (no Stream object)."""
    if _raw_stream_of is not None:
        return _raw_stream_of(device.index)
    return torch.cuda.current_stream(device).cuda_stream


@functools.lru_cache(maxsize=256)
def _lora_scale(lora_alpha: float, r: int) -> float:
    return float(np.float32(lora_alpha) / np.float32(r))  # fp32 division, as w4a16_lora_gemv.cu:221


def _ptr(t):
    return None if t is None else t.data_ptr()


DEVERR_MBAR_TIMEOUT, DEVERR_PEER_TIMEOUT = 1, 2


def device_error(reset: bool = True) -> int:
    """The sticky device-side error bits of the current device (a bounded
    wait inside a kernel that ran out: 1 = an mbarrier phase, 2 = a peer
    rank's flag); synchronises with the device.  ``reset`` clears them."""
    import ctypes
    code = ctypes.c_uint(0)
    _lib.check(_LIB.qx_get_device_error(ctypes.byref(code), 1 if reset else 0), "get_device_error")
    return int(code.value)


def check_device_error(what: str = "device") -> None:
    """Raise if a kernel's bounded wait ran out since the last check (its
    output was undefined); clears the bits."""
    code = device_error(reset=True)
    if code:
        names = [n for b, n in ((DEVERR_MBAR_TIMEOUT, "mbarrier wait timed out"),
                                (DEVERR_PEER_TIMEOUT, "peer rank did not arrive")) if code & b]
        raise RuntimeError(f"{what}: device-side error 0x{code:x} ({', '.join(names)})")


# ------------------------------------------------------------------ norms --
def fused_rmsnorm(input: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``fp16((x * rsqrt(mean(x^2) + eps)) * w)`` over the last dim
    (reference: ``csrc/kernels/rmsnorm.cu:162-210``)."""
    _check_input(input, "input")
    _check_input(weight, "weight")
    _check_fp16(input, "input")
    _check_fp16(weight, "weight")
    hidden = input.size(-1)
    if weight.numel() != hidden:
        raise RuntimeError(f"weight size mismatch: {weight.numel()} vs {hidden}")
    out = torch.empty_like(input)
    rows = input.numel() // hidden if hidden else 0
    st = _stream(input.device)
    _lib.check(_LIB.qx_fused_rmsnorm(input.data_ptr(), weight.data_ptr(), out.data_ptr(), rows,
                                     hidden, float(eps), st.cuda_stream), "fused_rmsnorm")
    return out


def fused_swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``fp16(silu(gate) * up)`` elementwise (reference: ``csrc/kernels/swiglu.cu:94-135``)."""
    _check_input(gate, "gate")
    _check_input(up, "up")
    _check_fp16(gate, "gate")
    if gate.shape != up.shape:
        raise RuntimeError("gate and up must have same shape")
    _check_fp16(up, "up")
    out = torch.empty_like(gate)
    st = _stream(gate.device)
    _lib.check(_LIB.qx_fused_swiglu(gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel(),
                                    st.cuda_stream), "fused_swiglu")
    return out


# ------------------------------------------------------ fused decode step --
def add_rmsnorm(x: torch.Tensor, delta: torch.Tensor, weight: torch.Tensor,
                eps: float = 1e-6) -> torch.Tensor:
    """Residual add and RMSNorm in one pass: ``x += delta`` (in place, fp16
    rounding) and returns ``fused_rmsnorm(x, weight, eps)`` (new component:
    the reference's patched layer runs the add and the norm separately)."""
    for t, n in ((x, "x"), (delta, "delta"), (weight, "weight")):
        _check_input(t, n)
        _check_fp16(t, n)
    if x.shape != delta.shape or weight.dim() != 1 or weight.numel() != x.size(-1):
        raise RuntimeError("add_rmsnorm: x and delta must match, weight must be [hidden]")
    out = torch.empty_like(x)
    st = _stream(x.device)
    _lib.check(_LIB.qx_add_rmsnorm(x.data_ptr(), delta.data_ptr(), weight.data_ptr(), out.data_ptr(),
                                   x.numel() // x.size(-1), x.size(-1), float(eps), st.cuda_stream),
               "add_rmsnorm")
    return out


def qk_norm_rope_append(qkv: torch.Tensor, q_heads: int, kv_heads: int, q_norm: torch.Tensor,
                        k_norm: torch.Tensor, eps: float, cos_row: torch.Tensor,
                        sin_row: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                        sink: int, window: int, pos: int) -> torch.Tensor:
    """One decode position: ``qkv`` fp16 ``[B, (q_heads + 2 kv_heads) * D]``;
    returns q ``[B, q_heads, D]`` (head-normed, rotated) and writes the
    head-normed, rotated k and the v heads into ring slot ``pos`` of
    ``k_cache`` / ``v_cache`` ``[B, sink + window, kv_heads, D]``."""
    for t, n in ((qkv, "qkv"), (q_norm, "q_norm"), (k_norm, "k_norm"), (k_cache, "k_cache"),
                 (v_cache, "v_cache")):
        _check_input(t, n)
        _check_fp16(t, n)
    D = q_norm.numel()
    B = qkv.size(0)
    if qkv.numel() != B * (q_heads + 2 * kv_heads) * D or k_norm.numel() != D:
        raise RuntimeError("qk_norm_rope_append: qkv must be [B, (q_heads + 2 kv_heads) * head_dim]")
    if tuple(k_cache.shape) != (B, sink + window, kv_heads, D) or v_cache.shape != k_cache.shape:
        raise RuntimeError("qk_norm_rope_append: cache must be [B, sink + window, kv_heads, head_dim]")
    for t, n in ((cos_row, "cos_row"), (sin_row, "sin_row")):
        _check_input(t, n)
        if t.dtype != torch.float32 or t.numel() != D:
            raise RuntimeError(f"{n} must be float32 [{D}]")
    q = torch.empty(B, q_heads, D, dtype=torch.float16, device=qkv.device)
    st = _stream(qkv.device)
    _lib.check(_LIB.qx_qk_norm_rope_append(
        qkv.data_ptr(), B, q_heads, kv_heads, D, q_norm.data_ptr(), k_norm.data_ptr(), float(eps),
        cos_row.data_ptr(), sin_row.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        int(sink), int(window), int(pos), st.cuda_stream), "qk_norm_rope_append")
    return q


def swiglu_packed(gate_up: torch.Tensor) -> torch.Tensor:
    """``gate_up`` fp16 ``[..., 2 I]`` (gate columns then up) ->
    ``fp16(silu(gate) * up)`` ``[..., I]`` (the formula of ``fused_swiglu``)."""
    _check_input(gate_up, "gate_up")
    _check_fp16(gate_up, "gate_up")
    inter = gate_up.size(-1) // 2
    out = torch.empty(*gate_up.shape[:-1], inter, dtype=torch.float16, device=gate_up.device)
    st = _stream(gate_up.device)
    _lib.check(_LIB.qx_swiglu_packed(gate_up.data_ptr(), out.data_ptr(), gate_up.numel() // (2 * inter),
                                     inter, st.cuda_stream), "swiglu_packed")
    return out


# ------------------------------------------------------------------- GEMV --
def _prepare_lora(lora_A, lora_B):
    """Pad rank up to a supported value with zero rows/columns (exact: the
    padding contributes 0 to x.A and to (x.A).B)."""
    r = lora_A.size(1)
    if r in _SUPPORTED_RANKS:
        return lora_A, lora_B, r
    rp = next((s for s in _SUPPORTED_RANKS if s >= r), None)
    if rp is None:
        raise RuntimeError(f"LoRA rank {r} > 128 is not supported")
    A = torch.zeros(lora_A.size(0), rp, dtype=lora_A.dtype, device=lora_A.device)
    B = torch.zeros(rp, lora_B.size(1), dtype=lora_B.dtype, device=lora_B.device)
    A[:, :r] = lora_A
    B[:r] = lora_B
    return A, B, rp


# rows from which w4a16(_lora)_gemv runs on the tensor-core GEMM instead of the decode GEMV
GEMM_MIN_ROWS = 128


class _Weights:
    """Validated description of one (qweight, scales, zeros, lora_A, lora_B,
    group_size, zero_offset) set, kept so that a decode loop calling the same
    weights again only checks that the tensors are still the same ones."""

    __slots__ = ("refs", "ptrs", "qw_shape", "K", "N", "packed", "rank", "A", "B", "dev",
                 "group", "zero_offset", "args")


_WCACHE: dict = {}
_WCACHE_MAX = 4096


def _validate_weights(qweight, scales, zeros, lora_A, lora_B, group_size, zero_offset) -> _Weights:
    for t, n in ((qweight, "qweight"), (scales, "scales"), (zeros, "zeros")):
        _check_input(t, n)
    _check_fp16(scales, "scales")
    if qweight.dtype != torch.int32 or qweight.dim() != 2:
        raise RuntimeError("qweight must be int32 [K/8, N]")
    K = qweight.size(0) * 8
    N = qweight.size(1)
    G = K // group_size if group_size > 0 else 0
    if scales.dim() != 2 or scales.size(0) != G or scales.size(1) != N:
        raise RuntimeError(f"scales must be [{G}, {N}], got {list(scales.shape)}")
    if zeros.dtype == torch.int32:
        packed = 1
        if tuple(zeros.shape) != (G, N // 8):
            raise RuntimeError(f"packed qzeros must be int32 [{G}, {N // 8}], got {list(zeros.shape)}")
    elif zeros.dtype == torch.float16:
        packed = 0
        if tuple(zeros.shape) != (G, N):
            raise RuntimeError(f"zeros must be fp16 [{G}, {N}], got {list(zeros.shape)}")
    else:
        raise RuntimeError(f"zeros must be float16 [G, N] or int32 qzeros [G, N/8], got {zeros.dtype}")
    rank = 0
    if lora_A is not None:
        _check_input(lora_A, "lora_A")
        _check_input(lora_B, "lora_B")
        _check_fp16(lora_A, "lora_A")
        _check_fp16(lora_B, "lora_B")
        if lora_A.dim() != 2 or lora_A.size(0) != K or lora_B.dim() != 2 or \
                lora_B.size(0) != lora_A.size(1) or lora_B.size(1) != N:
            raise RuntimeError(f"lora_A must be [{K}, r] and lora_B [r, {N}]")
        lora_A, lora_B, rank = _prepare_lora(lora_A, lora_B)
    devs = {t.get_device() for t in (qweight, scales, zeros, lora_A, lora_B) if t is not None}
    if len(devs) != 1:
        raise RuntimeError("qweight, scales, zeros and the LoRA factors must be on one device")
    w = _Weights()
    w.qw_shape = qweight.shape
    w.K, w.N, w.packed, w.rank = K, N, packed, rank
    w.A, w.B = lora_A, lora_B  # the (possibly padded) factors stay alive with the entry
    w.dev = devs.pop()
    w.group, w.zero_offset = int(group_size), int(zero_offset)
    w.args = (qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(), packed, w.zero_offset,
              _ptr(lora_A), _ptr(lora_B))
    return w


def _weights(qweight, scales, zeros, lora_A, lora_B, group_size, zero_offset) -> _Weights:
    import weakref
    key = (id(qweight), id(scales), id(zeros), id(lora_A), id(lora_B), group_size, zero_offset)
    w = _WCACHE.get(key)
    if w is not None:
        r = w.refs
        if (r[0]() is qweight and r[1]() is scales and r[2]() is zeros
                and (lora_A is None or (r[3]() is lora_A and r[4]() is lora_B))
                and qweight.data_ptr() == w.ptrs[0] and scales.data_ptr() == w.ptrs[1]
                and zeros.data_ptr() == w.ptrs[2] and qweight.shape == w.qw_shape
                and (lora_A is None or (lora_A.data_ptr() == w.ptrs[3]
                                        and lora_B.data_ptr() == w.ptrs[4]))):
            return w
    w = _validate_weights(qweight, scales, zeros, lora_A, lora_B, group_size, zero_offset)
    w.refs = tuple(weakref.ref(t) if t is not None else (lambda: None)
                   for t in (qweight, scales, zeros, lora_A, lora_B))
    w.ptrs = tuple(t.data_ptr() if t is not None else 0 for t in (qweight, scales, zeros, lora_A, lora_B))
    if len(_WCACHE) >= _WCACHE_MAX:
        _WCACHE.clear()
    _WCACHE[key] = w
    return w


def _w4a16(input, qweight, scales, zeros, lora_A, lora_B, group_size, lora_scale, zero_offset,
           path: str | None = None, out: torch.Tensor | None = None):
    """``path`` (tests and benchmarks): "gemm" forces the tensor-core GEMM;
    None routes by shape (GEMM for >= GEMM_MIN_ROWS rows, else the GEMV).
    ``out``: optional preallocated fp16 output ``[..., N]`` (written, returned)."""
    w = _weights(qweight, scales, zeros, lora_A, lora_B, group_size, zero_offset)
    if not (isinstance(input, torch.Tensor) and input.is_cuda and input.dtype == torch.float16
            and input.is_contiguous()):
        _check_input(input, "input")
        _check_fp16(input, "input")
    K, N = w.K, w.N
    if input.size(-1) != K:
        raise RuntimeError(f"qweight has {K // 8} packed rows; input K={input.size(-1)} needs "
                           f"{input.size(-1) // 8}")
    di = input.get_device()
    if di != w.dev:
        raise RuntimeError(f"input is on cuda:{di} but the weights are on cuda:{w.dev}")
    lead = input.shape[:-1]
    M = input.numel() // K
    if out is None:
        out = torch.empty(lead + (N,), dtype=torch.float16, device=input.device)
    elif not (out.is_cuda and out.dtype == torch.float16 and out.is_contiguous()
              and out.shape == lead + (N,) and out.get_device() == di):
        raise RuntimeError(f"out must be a contiguous fp16 CUDA tensor of shape {list(lead) + [N]} "
                           f"on cuda:{di}")
    rank = w.rank
    if path == "gemm" or (path is None and M >= GEMM_MIN_ROWS and N % 256 == 0 and K % 64 == 0
                          and rank <= 64):
        # prefill: the tcgen05 tensor-core GEMM
        dev = input.device
        st = _stream(dev)
        with torch.cuda.device(dev):
            need = _LIB.qx_w4a16_lora_gemm_sm100_workspace_size(M, rank)
            ws = _workspace.get(dev, st, need, "w4a16_gemm") if need else None
            _lib.check(_LIB.qx_w4a16_lora_gemm_sm100(
                input.data_ptr(), *w.args, out.data_ptr(), M, K, N, rank, w.group, float(lora_scale),
                _ptr(ws), int(need), st.cuda_stream), "w4a16_gemm")
        return out
    if di == torch.cuda.current_device():  # the decode hot path: no device switch
        rc = _LIB.qx_w4a16_lora_gemv(input.data_ptr(), *w.args, out.data_ptr(), M, K, N, rank, w.group,
                                     lora_scale, _raw_stream_of(di) if _raw_stream_of else
                                     torch.cuda.current_stream(di).cuda_stream)
        if rc < 0:
            _lib.check(rc, "w4a16_gemv")
    else:
        with torch.cuda.device(di):
            _lib.check(_LIB.qx_w4a16_lora_gemv(input.data_ptr(), *w.args, out.data_ptr(), M, K, N, rank,
                                               w.group, lora_scale, _raw_stream(input.device)),
                       "w4a16_gemv")
    return out


def interleave_gate_up(t: torch.Tensor, inter: int, packed: bool = False) -> torch.Tensor:
    """Reorders the columns of a gate|up operand ``[..., 2 I]`` (gate columns,
    then up; ``[..., 2 I / 8]`` int32 words of 8 columns when ``packed``: GPTQ
    qzeros) into blocks of 16 columns: the 8 gate columns of outputs
    8b..8b+7, then their 8 up columns (the layout of
    ``w4a16_lora_gemv_swiglu``).  Apply it to qweight, scales, qzeros and
    LoRA B alike."""
    if packed:
        nb = inter // 8
        idx = torch.stack([torch.arange(nb), torch.arange(nb) + nb], 1).reshape(-1)
    else:
        if inter % 8:
            raise RuntimeError(f"interleave_gate_up: I={inter} must be a multiple of 8")
        b = torch.arange(inter // 8)[:, None] * 8 + torch.arange(8)[None, :]  # [I/8, 8]
        idx = torch.stack([b, b + inter], 1).reshape(-1)
    return t.index_select(-1, idx.to(t.device)).contiguous()


def _w4a16_swiglu(input, qweight, scales, zeros, lora_A, lora_B, group_size, lora_scale, zero_offset):
    """SwiGLU of the gate|up projection whose operands ``interleave_gate_up``
    laid out: ``[..., N / 2]``.  Decode rows run the GEMV with the SwiGLU
    epilogue (one launch); prefill rows the tensor-core GEMM, then SwiGLU on
    the gathered gate and up columns."""
    w = _weights(qweight, scales, zeros, lora_A, lora_B, group_size, zero_offset)
    if not (isinstance(input, torch.Tensor) and input.is_cuda and input.dtype == torch.float16
            and input.is_contiguous()):
        _check_input(input, "input")
        _check_fp16(input, "input")
    K, N = w.K, w.N
    if input.size(-1) != K or N % 16:
        raise RuntimeError(f"w4a16_lora_gemv_swiglu: input K={input.size(-1)} (weights K={K}), "
                           f"N={N} must be a multiple of 16")
    di = input.get_device()
    if di != w.dev:
        raise RuntimeError(f"input is on cuda:{di} but the weights are on cuda:{w.dev}")
    lead = input.shape[:-1]
    M = input.numel() // K
    if M >= GEMM_MIN_ROWS and N % 256 == 0 and K % 64 == 0 and w.rank <= 64:
        y = _w4a16(input, qweight, scales, zeros, lora_A, lora_B, group_size, lora_scale, zero_offset)
        y = y.view(M, N // 16, 2, 8)
        return fused_swiglu(y[:, :, 0].reshape(M, N // 2), y[:, :, 1].reshape(M, N // 2)).view(
            lead + (N // 2,))
    out = torch.empty(lead + (N // 2,), dtype=torch.float16, device=input.device)
    with torch.cuda.device(di):
        _lib.check(_LIB.qx_w4a16_lora_gemv_swiglu(input.data_ptr(), *w.args, out.data_ptr(), M, K, N,
                                                  w.rank, w.group, lora_scale, _raw_stream(input.device)),
                   "w4a16_gemv_swiglu")
    return out


def _w4a16_addnorm(residual, delta, norm_weight, eps, residual_out, qweight, scales, zeros, lora_A, lora_B,
                   group_size, lora_scale, zero_offset, swiglu: bool = False):
    """The decode step's residual add + RMSNorm fused into the projection that
    follows (``qx_w4a16_lora_gemv_addnorm``): ``residual_out = fp16(residual +
    delta)``, ``x = rmsnorm(residual_out) * norm_weight`` and returns the
    W4A16-LoRA projection of x (``swiglu``: the SwiGLU form over interleaved
    gate|up operands, ``[M, N / 2]``).  Up to 8 rows; ``residual_out`` is a
    separate buffer (callers alternate two)."""
    w = _weights(qweight, scales, zeros, lora_A, lora_B, group_size, zero_offset)
    for t, n in ((residual, "residual"), (delta, "delta"), (norm_weight, "norm_weight"),
                 (residual_out, "residual_out")):
        _check_input(t, n)
        _check_fp16(t, n)
    K, N = w.K, w.N
    if residual.size(-1) != K or residual.shape != delta.shape or residual.shape != residual_out.shape \
            or norm_weight.numel() != K:
        raise RuntimeError(f"w4a16_lora_gemv_addnorm: residual, delta and residual_out must be [M, {K}], "
                           f"norm_weight [{K}]")
    di = residual.get_device()
    if di != w.dev:
        raise RuntimeError(f"residual is on cuda:{di} but the weights are on cuda:{w.dev}")
    lead = residual.shape[:-1]
    M = residual.numel() // K
    out = torch.empty(lead + ((N // 2) if swiglu else N,), dtype=torch.float16, device=residual.device)
    rc = _LIB.qx_w4a16_lora_gemv_addnorm(residual.data_ptr(), delta.data_ptr(), norm_weight.data_ptr(),
                                         float(eps), residual_out.data_ptr(), *w.args, out.data_ptr(), M, K, N,
                                         w.rank, w.group, lora_scale, 1 if swiglu else 0,
                                         _raw_stream(residual.device))
    if rc < 0:
        _lib.check(rc, "w4a16_gemv_addnorm")
    return out


def w4a16_lora_gemv_swiglu(input, qweight, scales, zeros, lora_A, lora_B, group_size: int = 128,
                           lora_alpha: float = 16.0, *, zero_offset: int = 0):
    """``fused_swiglu(gate, up)`` of one W4A16-LoRA gate|up projection whose
    operands ``interleave_gate_up`` reordered (new component: the reference
    runs the two projections and ``fused_swiglu`` separately,
    ``qextract/patch.py:94-113``)."""
    scale = _lora_scale(float(lora_alpha), lora_A.size(1))
    return _w4a16_swiglu(input, qweight, scales, zeros, lora_A, lora_B, group_size, scale, zero_offset)


def w4a16_gemv(input, qweight, scales, zeros, group_size: int = 128, *, zero_offset: int = 0,
               out: torch.Tensor | None = None):
    """``fp16(x . W)`` with ``W = s (q - z)`` from GPTQ int4 packing
    (reference: ``csrc/kernels/w4a16_lora_gemv.cu:233-265``).  ``out``: an
    optional preallocated output (an addition to the reference signature)."""
    return _w4a16(input, qweight, scales, zeros, None, None, group_size, 0.0, zero_offset, out=out)


def w4a16_lora_gemv(input, qweight, scales, zeros, lora_A, lora_B, group_size: int = 128,
                    lora_alpha: float = 16.0, *, zero_offset: int = 0,
                    out: torch.Tensor | None = None):
    """``fp16(x . W + (alpha / r) (x . A) . B)``; ``r = lora_A.size(1)``
    (reference: ``csrc/kernels/w4a16_lora_gemv.cu:268-323``).  ``out``: an
    optional preallocated output (an addition to the reference signature)."""
    scale = _lora_scale(float(lora_alpha), lora_A.size(1))
    return _w4a16(input, qweight, scales, zeros, lora_A, lora_B, group_size, scale, zero_offset, out=out)


# ------------------------------------------------------------- ring cache --
def ring_slot_indices(count: int, sink: int, window: int, device) -> torch.Tensor:
    """Logical-order slot list for ``count`` written tokens (int32, on device)."""
    dev = torch.device(device)
    valid = count if count <= sink else sink + min(count - sink, window)
    out = torch.empty(max(valid, 1), dtype=torch.int32, device=dev)
    st = _stream(dev)
    n = _lib.check(_LIB.qx_ring_slot_indices(out.data_ptr(), sink, window, count, st.cuda_stream),
                   "ring_slot_indices")
    assert n == valid
    return out[:valid]


def decode_attention(q, k_cache, v_cache, count: int, sink: int, window: int,
                     softmax_scale: float | None = None, *, after_append: bool = False):
    """GQA decode attention over the ring's valid slots, read in place.
    ``q`` fp16 ``[B, Hq, D]``; ``k_cache``/``v_cache`` fp16 ``[B, S+W, Hkv, D]``.
    ``after_append``: the kernel just before on the stream wrote only ``q``
    and position ``count - 1`` of the cache (``qk_norm_rope_append``); the
    attention then starts loading the other slots while it finishes."""
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _check_input(t, n)
        _check_fp16(t, n)
    B, Hq, D = q.shape
    if k_cache.dim() != 4 or k_cache.size(0) != B or k_cache.size(1) != sink + window or \
            k_cache.size(3) != D or v_cache.shape != k_cache.shape:
        raise RuntimeError("cache must be [B, sink + window, Hkv, D]")
    Hkv = k_cache.size(2)
    out = torch.empty_like(q)
    dev = q.device
    st = _stream(dev)
    with torch.cuda.device(dev):
        need = _LIB.qx_decode_attention_workspace_size(B, Hq, Hkv, D, sink, window)
        ws = _workspace.get(dev, st, need, "decode_attention")
        _lib.check(_LIB.qx_decode_attention_ex(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), B, Hq, Hkv, D,
            sink, window, int(count), float(softmax_scale or 0.0), ws.data_ptr(), ws.numel(),
            1 if after_append else 0, st.cuda_stream), "decode_attention")
    return out


def decode_attention_qkv(qkv: torch.Tensor, q_heads: int, kv_heads: int, q_norm: torch.Tensor,
                         k_norm: torch.Tensor, eps: float, cos_row: torch.Tensor, sin_row: torch.Tensor,
                         k_cache: torch.Tensor, v_cache: torch.Tensor, sink: int, window: int, pos: int,
                         softmax_scale: float | None = None) -> torch.Tensor:
    """``qk_norm_rope_append`` then ``decode_attention`` (count ``pos + 1``) in
    one kernel: ``qkv`` fp16 ``[B, (q_heads + 2 kv_heads) * D]``; writes the new
    token's k and v into ring slot ``pos``; returns ``[B, q_heads, D]``."""
    for t, n in ((qkv, "qkv"), (q_norm, "q_norm"), (k_norm, "k_norm"), (k_cache, "k_cache"),
                 (v_cache, "v_cache")):
        _check_input(t, n)
        _check_fp16(t, n)
    D = q_norm.numel()
    B = qkv.size(0)
    if qkv.numel() != B * (q_heads + 2 * kv_heads) * D or k_norm.numel() != D:
        raise RuntimeError("decode_attention_qkv: qkv must be [B, (q_heads + 2 kv_heads) * head_dim]")
    if tuple(k_cache.shape) != (B, sink + window, kv_heads, D) or v_cache.shape != k_cache.shape:
        raise RuntimeError("decode_attention_qkv: cache must be [B, sink + window, kv_heads, head_dim]")
    for t, n in ((cos_row, "cos_row"), (sin_row, "sin_row")):
        _check_input(t, n)
        if t.dtype != torch.float32 or t.numel() != D:
            raise RuntimeError(f"{n} must be float32 [{D}]")
    out = torch.empty(B, q_heads, D, dtype=torch.float16, device=qkv.device)
    dev = qkv.device
    st = _stream(dev)
    with torch.cuda.device(dev):
        need = _LIB.qx_decode_attention_workspace_size(B, q_heads, kv_heads, D, sink, window)
        ws = _workspace.get(dev, st, need, "decode_attention")
        _lib.check(_LIB.qx_decode_attention_qkv(
            qkv.data_ptr(), q_norm.data_ptr(), k_norm.data_ptr(), float(eps), cos_row.data_ptr(),
            sin_row.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), B, q_heads,
            kv_heads, D, int(sink), int(window), int(pos), float(softmax_scale or 0.0), ws.data_ptr(),
            ws.numel(), st.cuda_stream), "decode_attention_qkv")
    return out


def lm_head_argmax(h: torch.Tensor, weight: torch.Tensor, vocab_offset: int = 0):
    """Greedy head: ``h`` fp16 ``[B, H]`` (B <= 32), ``weight`` fp16 ``[H, V]``
    (a vocabulary slice).  Returns (max logit fp32 ``[B]``, index int64 ``[B]``
    + ``vocab_offset``) of the fp16 logits ``h @ weight``; ties go to the
    smallest index."""
    for t, n in ((h, "h"), (weight, "weight")):
        _check_input(t, n)
        _check_fp16(t, n)
    B, H = h.shape
    if weight.dim() != 2 or weight.size(0) != H:
        raise RuntimeError("lm_head_argmax: weight must be [H, V]")
    V = weight.size(1)
    dev = h.device
    val = torch.empty(B, dtype=torch.float32, device=dev)
    idx = torch.empty(B, dtype=torch.int64, device=dev)
    st = _stream(dev)
    with torch.cuda.device(dev):
        need = _LIB.qx_lm_head_argmax_workspace_size(V)
        ws = _workspace.get(dev, st, need, "lm_head_argmax")
        _lib.check(_LIB.qx_lm_head_argmax(h.data_ptr(), weight.data_ptr(), B, H, V, int(vocab_offset),
                                          val.data_ptr(), idx.data_ptr(), ws.data_ptr(), ws.numel(),
                                          st.cuda_stream), "lm_head_argmax")
    return val, idx


def prefill_attention(q, k_new, v_new, k_cache, v_cache, count: int, sink: int, window: int,
                      softmax_scale: float | None = None):
    """Attention of a prompt chunk before its append: ``q`` fp16 ``[B, n, Hq, D]``
    at positions ``count ..``, ``k_new``/``v_new`` fp16 ``[B, n, Hkv, D]``, the
    ring ``k_cache``/``v_cache`` ``[B, S+W, Hkv, D]`` after ``count`` tokens (read
    in place).  Returns ``[B, n, Hq, D]``: causal, sinks + the last ``window``
    positions visible (new component: the reference gathers the cache,
    ``qextract/kv_cache.py:96-112``, and attends over the copy)."""
    for t, nm in ((q, "q"), (k_new, "k_new"), (v_new, "v_new"), (k_cache, "k_cache"),
                  (v_cache, "v_cache")):
        _check_input(t, nm)
        _check_fp16(t, nm)
    B, n, Hq, D = q.shape
    Hkv = k_new.size(2)
    if tuple(k_new.shape) != (B, n, Hkv, D) or v_new.shape != k_new.shape:
        raise RuntimeError("k_new / v_new must be [B, n, Hkv, D] like q")
    if tuple(k_cache.shape) != (B, sink + window, Hkv, D) or v_cache.shape != k_cache.shape:
        raise RuntimeError("cache must be [B, sink + window, Hkv, D]")
    out = torch.empty_like(q)
    st = _stream(q.device)
    with torch.cuda.device(q.device):
        _lib.check(_LIB.qx_prefill_attention(
            q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
            out.data_ptr(), B, n, Hq, Hkv, D, sink, window, int(count), float(softmax_scale or 0.0),
            st.cuda_stream), "prefill_attention")
    return out


class RingBufferKVCache:
    """StreamingLLM sink + ring-window KV cache (reference:
    ``csrc/include/ring_buffer.h:32-77``, ``csrc/kv_cache/ring_buffer.cu``).

    Storage: ``k``/``v`` fp16 ``[num_layers, batch, sink + window, kv_heads, head_dim]``
    owned by this object.  ``write_count`` advances when the last layer is
    appended (``ring_buffer.cu:138-140``).
    """

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, sink_size: int = 4,
                 window_size: int = 4092, batch: int = 1, device=None):
        if window_size < 1 or sink_size < 0:
            raise RuntimeError("sink_size must be >= 0 and window_size >= 1")
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.sink_size, self.window_size = sink_size, window_size
        self.total_size = sink_size + window_size
        self.batch = batch
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda":
            raise RuntimeError("RingBufferKVCache lives on a CUDA device")
        self.device = dev
        shape = (num_layers, batch, self.total_size, num_kv_heads, head_dim)
        self.k = torch.zeros(shape, dtype=torch.float16, device=dev)
        self.v = torch.zeros(shape, dtype=torch.float16, device=dev)
        self._write_count = 0

    # --- reference methods (binding.cpp:67-74) ---
    def append(self, new_k: torch.Tensor, new_v: torch.Tensor, layer_idx: int) -> None:
        """``new_k``/``new_v``: ``[H, D]`` (one token, batch 1), ``[T, H, D]``
        (batch 1) or ``[B, T, H, D]``."""
        _check_input(new_k, "new_k")
        _check_input(new_v, "new_v")
        _check_fp16(new_k, "new_k")
        _check_fp16(new_v, "new_v")
        if new_k.shape != new_v.shape:
            raise RuntimeError("new_k and new_v must have the same shape")
        if not 0 <= layer_idx < self.num_layers:
            raise RuntimeError(f"layer_idx {layer_idx} out of range")
        if new_k.dim() == 2:
            B, T = 1, 1
        elif new_k.dim() == 3:
            B, T = 1, new_k.size(0)
        elif new_k.dim() == 4:
            B, T = new_k.size(0), new_k.size(1)
        else:
            raise RuntimeError("new_k must be [H, D], [T, H, D] or [B, T, H, D]")
        if B != self.batch or tuple(new_k.shape[-2:]) != (self.num_kv_heads, self.head_dim):
            raise RuntimeError(f"new_k shape {list(new_k.shape)} does not match the cache "
                               f"(batch={self.batch}, heads={self.num_kv_heads}, dim={self.head_dim})")
        st = _stream(self.device)
        _lib.check(_LIB.qx_ring_append(
            self.k[layer_idx].data_ptr(), self.v[layer_idx].data_ptr(), new_k.data_ptr(),
            new_v.data_ptr(), B, T, self.num_kv_heads, self.head_dim, self.sink_size,
            self.window_size, self._write_count, st.cuda_stream), "ring_append")
        if layer_idx == self.num_layers - 1:
            self._write_count += T

    def advance(self, tokens: int) -> None:
        """Count ``tokens`` positions that a fused decode kernel
        (``qk_norm_rope_append``) wrote into every layer."""
        self._write_count += int(tokens)

    def get_kv(self, layer_idx: int):
        """(K, V) in logical order: ``[valid, H, D]`` for batch 1, else
        ``[B, valid, H, D]`` (reference ``get_kv``, ``ring_buffer.cu:143-200``)."""
        valid = self.get_valid_length()
        shape = (self.batch, valid, self.num_kv_heads, self.head_dim)
        ko = torch.empty(shape, dtype=torch.float16, device=self.device)
        vo = torch.empty(shape, dtype=torch.float16, device=self.device)
        st = _stream(self.device)
        _lib.check(_LIB.qx_ring_gather(
            self.k[layer_idx].data_ptr(), self.v[layer_idx].data_ptr(), ko.data_ptr(), vo.data_ptr(),
            self.batch, self.num_kv_heads, self.head_dim, self.sink_size, self.window_size,
            self._write_count, st.cuda_stream), "ring_gather")
        if self.batch == 1:
            return ko[0], vo[0]
        return ko, vo

    def get_valid_length(self) -> int:
        c = self._write_count
        if c <= self.sink_size:
            return c
        return self.sink_size + min(c - self.sink_size, self.window_size)

    def get_total_written(self) -> int:
        return self._write_count

    def reset(self) -> None:
        self._write_count = 0

    # --- additions ---
    def slot_indices(self) -> torch.Tensor:
        return ring_slot_indices(self._write_count, self.sink_size, self.window_size, self.device)

    def decode_attention(self, q: torch.Tensor, layer_idx: int,
                         softmax_scale: float | None = None) -> torch.Tensor:
        """Attention of ``q`` (``[B, Hq, D]`` or ``[Hq, D]``) over this layer's
        valid slots, read in place."""
        squeeze = q.dim() == 2
        if squeeze:
            q = q.unsqueeze(0)
        out = decode_attention(q, self.k[layer_idx], self.v[layer_idx], self._write_count,
                               self.sink_size, self.window_size, softmax_scale)
        return out[0] if squeeze else out
