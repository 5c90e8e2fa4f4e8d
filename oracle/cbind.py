"""Build recipe and ctypes binding for ``qx_oracle.c``.  Test infrastructure only.

``build()`` compiles ``qx_oracle.c`` with gcc + OpenMP into
``oracle/_build/libqx_oracle.so``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "qx_oracle.c")
_OUT_DIR = os.path.join(_HERE, "_build")
_LIB_PATH = os.path.join(_OUT_DIR, "libqx_oracle.so")
_lib = None


def build(force: bool = False) -> str:
    os.makedirs(_OUT_DIR, exist_ok=True)
    if (not force and os.path.exists(_LIB_PATH)
            and os.path.getmtime(_LIB_PATH) >= os.path.getmtime(_SRC)):
        return _LIB_PATH
    tmp = _LIB_PATH + f".tmp{os.getpid()}"
    subprocess.check_call(["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC",
                           "-shared", "-std=c11", _SRC, "-o", tmp])
    os.replace(tmp, _LIB_PATH)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        path = build()
        L = ctypes.CDLL(path)
        L.qxo_h2f.restype = ctypes.c_float
        L.qxo_h2f.argtypes = [ctypes.c_uint16]
        L.qxo_f2h.restype = ctypes.c_uint16
        L.qxo_f2h.argtypes = [ctypes.c_float]
        p = ctypes.c_void_p
        L.qxo_w4a16_lora_gemv.restype = ctypes.c_int
        L.qxo_w4a16_lora_gemv.argtypes = [p, p, p, p, ctypes.c_int, ctypes.c_int, p, p, p, p,
                                          ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                          ctypes.c_int]
        L.qxo_dequantize.restype = ctypes.c_int
        L.qxo_dequantize.argtypes = [p, p, p, ctypes.c_int, ctypes.c_int, p, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.qxo_ring_write_pos.restype = ctypes.c_int64
        L.qxo_ring_write_pos.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int]
        L.qxo_ring_valid_length.restype = ctypes.c_int64
        L.qxo_ring_valid_length.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int]
        L.qxo_ring_indices.restype = ctypes.c_int64
        L.qxo_ring_indices.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int, p]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def c_w4a16_lora_gemv(x, qweight, scales, zeros, lora_A=None, lora_B=None,
                      group_size=128, lora_alpha=16.0, zero_offset=0, nthreads=0,
                      return_f32=False):
    """C oracle: same contract as ``oracle.gptq.w4a16_lora_gemv_ref``."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    lead = x.shape[:-1]
    K = x.shape[-1]
    M = int(np.prod(lead)) if lead else 1
    qweight = np.ascontiguousarray(qweight, dtype=np.int32)
    N = qweight.shape[1]
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    packed = 1 if zeros.dtype == np.int32 else 0
    zeros = np.ascontiguousarray(zeros)
    rank = 0
    if lora_A is not None:
        lora_A = np.ascontiguousarray(lora_A, dtype=np.float16)
        lora_B = np.ascontiguousarray(lora_B, dtype=np.float16)
        rank = lora_A.shape[1]
    y = np.empty((M, N), dtype=np.float16)
    yf = np.empty((M, N), dtype=np.float32) if return_f32 else None
    rc = lib().qxo_w4a16_lora_gemv(_ptr(x), _ptr(qweight), _ptr(scales), _ptr(zeros), packed,
                                   zero_offset, _ptr(lora_A), _ptr(lora_B), _ptr(y), _ptr(yf),
                                   M, K, N, rank, group_size, float(lora_alpha), int(nthreads))
    if rc != 0:
        raise ValueError("qxo_w4a16_lora_gemv: bad shapes")
    out = yf if return_f32 else y
    return out.reshape(*lead, N)


def c_dequantize(qweight, scales, zeros, group_size=128, zero_offset=0, nthreads=0):
    """C oracle: same contract as ``oracle.gptq.dequantize_gptq`` (fp16 ``[K, N]``)."""
    qweight = np.ascontiguousarray(qweight, dtype=np.int32)
    K, N = qweight.shape[0] * 8, qweight.shape[1]
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    packed = 1 if zeros.dtype == np.int32 else 0
    zeros = np.ascontiguousarray(zeros)
    W = np.empty((K, N), dtype=np.float16)
    rc = lib().qxo_dequantize(_ptr(qweight), _ptr(scales), _ptr(zeros), packed, zero_offset,
                              _ptr(W), K, N, group_size, int(nthreads))
    if rc != 0:
        raise ValueError("qxo_dequantize: bad shapes")
    return W


def c_ring_indices(count: int, sink: int, window: int) -> np.ndarray:
    L = lib()
    n = L.qxo_ring_valid_length(count, sink, window)
    out = np.empty(max(n, 1), dtype=np.int32)
    got = L.qxo_ring_indices(count, sink, window, _ptr(out))
    assert got == n
    return out[:n]
