"""GPTQ int4 (W4A16) + LoRA oracle in numpy.  Test infrastructure only.

Restates the reference's PyTorch reference path for the W4A16(-LoRA) GEMV:

* packing contract: ``csrc/include/quantize_utils.h:5-8`` -- nibble ``i``
  (bits ``4i..4i+3``) of ``qweight[pr, n]`` is ``W_q[8*pr + i, n]``;
  the same rule is used by the kernel (``csrc/kernels/w4a16_lora_gemv.cu:179-189``)
  and by the test packer (``tests/test_w4a16_gemv.py:58-59``);
* group of row ``k`` is ``k // group_size`` (no act-order / g_idx):
  ``csrc/kernels/w4a16_lora_gemv.cu:181``;
* dequantisation ``fp16((q - z) * s)`` computed in fp32 and rounded once to
  fp16: ``tests/test_w4a16_gemv.py:68-90``;
* base + LoRA in fp32, one fp16 rounding at the end, LoRA scaling
  ``alpha / rank`` with ``rank = A.shape[1]``:
  ``tests/test_w4a16_gemv.py:178-186`` and
  ``csrc/kernels/w4a16_lora_gemv.cu:214-225``.

The reference kernel only accepts *unpacked* fp16 zeros ``[G, N]``
(``csrc/kernels/w4a16_lora_gemv.cu:310``); GPTQ checkpoints carry packed
``qzeros int32 [G, N/8]`` (nibble ``n % 8`` of ``qzeros[g, n // 8]``).
``unpack_qzeros`` turns the packed form into the unpacked one, with an
optional ``+1`` for the GPTQ-v1 storage convention.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "unpack_int4_rows",
    "pack_int4_rows",
    "unpack_qzeros",
    "pack_qzeros",
    "dequantize_gptq",
    "w4a16_gemv_ref",
    "w4a16_lora_gemv_ref",
    "simulate_gptq_quantize",
    "make_gemv_inputs",
]


def unpack_int4_rows(qweight: np.ndarray) -> np.ndarray:
    """int32 ``[K/8, N]`` -> uint8 ``[K, N]`` (values 0..15).

    ``out[8*pr + i, n] = (qweight[pr, n] >> 4*i) & 0xF``
    (``csrc/include/quantize_utils.h:5-8``; ``w4a16_lora_gemv.cu:187-189``).
    """
    q = np.ascontiguousarray(qweight).view(np.uint32)
    pr, n = q.shape
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, :, None]
    nib = (q[:, None, :] >> shifts) & np.uint32(0xF)
    return nib.reshape(pr * 8, n).astype(np.uint8)


def pack_int4_rows(wq: np.ndarray) -> np.ndarray:
    """uint8 ``[K, N]`` (0..15) -> int32 ``[K/8, N]``; inverse of ``unpack_int4_rows``
    (``tests/test_w4a16_gemv.py:55-59``)."""
    k, n = wq.shape
    assert k % 8 == 0
    w = wq.astype(np.uint32).reshape(k // 8, 8, n)
    out = np.zeros((k // 8, n), dtype=np.uint32)
    for i in range(8):
        out |= (w[:, i, :] & np.uint32(0xF)) << np.uint32(4 * i)
    return out.view(np.int32)


def unpack_qzeros(qzeros: np.ndarray, n: int, zero_offset: int = 0) -> np.ndarray:
    """GPTQ packed zeros int32 ``[G, N/8]`` -> float32 ``[G, N]``.

    ``z[g, n] = ((qzeros[g, n // 8] >> 4*(n % 8)) & 0xF) + zero_offset``.
    ``zero_offset = 1`` is the GPTQ-v1 storage convention.
    """
    q = np.ascontiguousarray(qzeros).view(np.uint32)
    g, n8 = q.shape
    assert n8 * 8 == n, (q.shape, n)
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    nib = (q[:, :, None] >> shifts) & np.uint32(0xF)
    return nib.reshape(g, n).astype(np.float32) + np.float32(zero_offset)


def pack_qzeros(z: np.ndarray) -> np.ndarray:
    """uint8 ``[G, N]`` (0..15) -> int32 ``[G, N/8]`` (nibble ``n % 8``)."""
    g, n = z.shape
    assert n % 8 == 0
    zz = z.astype(np.uint32).reshape(g, n // 8, 8)
    out = np.zeros((g, n // 8), dtype=np.uint32)
    for i in range(8):
        out |= (zz[:, :, i] & np.uint32(0xF)) << np.uint32(4 * i)
    return out.view(np.int32)


def _zeros_f32(zeros: np.ndarray, n: int, zero_offset: int) -> np.ndarray:
    if zeros.dtype == np.int32:
        return unpack_qzeros(zeros, n, zero_offset)
    assert zeros.dtype == np.float16, zeros.dtype
    return zeros.astype(np.float32)


def dequantize_gptq(qweight, scales, zeros, group_size: int = 128,
                    zero_offset: int = 0) -> np.ndarray:
    """fp16 ``[K, N]``: ``fp16((q - z) * s)`` in fp32 with one rounding
    (``tests/test_w4a16_gemv.py:68-90``).  ``zeros`` is fp16 ``[G, N]``
    (reference format) or GPTQ-packed int32 ``[G, N/8]``."""
    q = unpack_int4_rows(qweight).astype(np.float32)
    k, n = q.shape
    g = np.arange(k) // group_size
    s = scales.astype(np.float32)[g]
    z = _zeros_f32(zeros, n, zero_offset)[g]
    return ((q - z) * s).astype(np.float16)


def _as2d(x):
    x = np.asarray(x)
    lead = x.shape[:-1]
    return x.reshape(-1, x.shape[-1]), lead


def w4a16_gemv_ref(x, qweight, scales, zeros, group_size: int = 128,
                   zero_offset: int = 0, return_f32: bool = False):
    """``fp16(x.float() @ W.float())`` (``tests/test_w4a16_gemv.py:133-134``).

    ``x`` is ``[K]`` or ``[..., K]``; the result has the same leading dims and
    last dim ``N``."""
    w = dequantize_gptq(qweight, scales, zeros, group_size, zero_offset)
    x2, lead = _as2d(x)
    y = x2.astype(np.float32) @ w.astype(np.float32)
    y = y.reshape(*lead, w.shape[1])
    return y if return_f32 else y.astype(np.float16)


def w4a16_lora_gemv_ref(x, qweight, scales, zeros, lora_A, lora_B,
                        group_size: int = 128, lora_alpha: float = 16.0,
                        zero_offset: int = 0, return_f32: bool = False):
    """``fp16(x W + (alpha/r) (x A) B)`` with fp32 math
    (``tests/test_w4a16_gemv.py:178-186``; scaling ``alpha / rank`` as in
    ``csrc/kernels/w4a16_lora_gemv.cu:221``)."""
    w = dequantize_gptq(qweight, scales, zeros, group_size, zero_offset)
    x2, lead = _as2d(x)
    xf = x2.astype(np.float32)
    base = xf @ w.astype(np.float32)
    rank = lora_A.shape[1]
    lora = (xf @ lora_A.astype(np.float32)) @ lora_B.astype(np.float32)
    y = base + np.float32(lora_alpha / rank) * lora
    y = y.reshape(*lead, w.shape[1])
    return y if return_f32 else y.astype(np.float16)


def simulate_gptq_quantize(w: np.ndarray, group_size: int = 128):
    """Min/max asymmetric 4-bit quantisation into GPTQ packing
    (``tests/test_w4a16_gemv.py:14-65``).  Returns qweight int32 ``[K/8, N]``,
    scales fp16 ``[G, N]`` and unpacked fp16 zeros ``[G, N]`` (the reference
    test's format)."""
    wf = w.astype(np.float16)
    k, n = wf.shape
    assert k % group_size == 0
    gcount = k // group_size
    wg = wf.reshape(gcount, group_size, n)
    wmin = wg.min(axis=1)
    wmax = wg.max(axis=1)
    scales = ((wmax - wmin) / np.float16(15.0)).astype(np.float16)
    scales = np.maximum(scales, np.float16(1e-6)).astype(np.float16)
    zeros = (-wmin / scales).astype(np.float16)
    s32 = np.repeat(scales.astype(np.float32), group_size, axis=0)
    z32 = np.repeat(zeros.astype(np.float32), group_size, axis=0)
    q = np.clip(np.round(wf.astype(np.float32) / s32 + z32), 0, 15).astype(np.uint8)
    return pack_int4_rows(q), scales, zeros


def make_gemv_inputs(M: int, K: int, N: int, rank: int, group_size: int = 128,
                     seed: int = 0, packed_zeros: bool = True, zero_nibble: int = 8,
                     lora_std: float = 0.02):
    """Seeded synthetic W4A16-LoRA inputs with the decode-GEMV value
    distributions: x ~ N(0,1) fp16; qweight nibbles uniform 0..15; scales
    U(0.005, 0.02); qzeros nibbles all ``zero_nibble`` (0x88888888 for 8);
    A, B ~ N(0, lora_std).  ``M == 0`` gives a 1-D ``x`` of shape ``[K]``."""
    rng = np.random.Generator(np.random.PCG64(seed))
    G = K // group_size
    xs = (K,) if M == 0 else (M, K)
    x = rng.standard_normal(xs, dtype=np.float32).astype(np.float16)
    qweight = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.uint64)
    qweight = qweight.astype(np.uint32).view(np.int32)
    scales = rng.uniform(0.005, 0.02, size=(G, N)).astype(np.float16)
    if packed_zeros:
        nib = np.uint32(zero_nibble & 0xF)
        word = np.uint32(0)
        for i in range(8):
            word |= nib << np.uint32(4 * i)
        zeros = np.full((G, N // 8), word, dtype=np.uint32).view(np.int32)
    else:
        zeros = np.full((G, N), zero_nibble, dtype=np.float16)
    A = (rng.standard_normal((K, rank), dtype=np.float32) * lora_std).astype(np.float16)
    B = (rng.standard_normal((rank, N), dtype=np.float32) * lora_std).astype(np.float16)
    return dict(x=x, qweight=qweight, scales=scales, zeros=zeros, lora_A=A, lora_B=B)
