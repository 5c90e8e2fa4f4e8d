"""C-ABI library: loads without a GPU, exports every declared symbol, and its
host-side argument validation rejects bad calls before touching a device.

CPU-only (no kernel is launched).
"""

import ctypes
import os
import re

import pytest

from qextract_infer_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qx_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qx_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 11, syms
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/qx_b200.h but not exported"
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature in _lib.SIGNATURES"
    assert set(_lib.SIGNATURES) == set(syms)
    assert b"sm_100a" in lib.qx_version()


def _gemv(lib, **kw):
    a = dict(x=16, qw=16, scales=16, zeros=16, packed=1, zoff=0, A=16, B=16, y=16, M=1, K=256,
             N=128, rank=16, group=128, scale=2.0, stream=None)
    a.update(kw)
    return lib.qx_w4a16_lora_gemv(a["x"], a["qw"], a["scales"], a["zeros"], a["packed"], a["zoff"],
                                  a["A"], a["B"], a["y"], a["M"], a["K"], a["N"], a["rank"],
                                  a["group"], a["scale"], a["stream"])


@pytest.mark.parametrize("kw,msg", [
    (dict(K=33), "multiple of 32"),
    (dict(group=48), "group_size"),
    (dict(N=12), "multiple of 8"),
    (dict(rank=12), "rank"),
    (dict(x=None), "null"),
    (dict(A=None), "lora_A"),
    (dict(x=24), "aligned"),
    (dict(packed=2), "zeros_packed"),
    (dict(scales=18), "aligned"),
])
def test_gemv_validation_errors(kw, msg):
    lib = _lib.load()
    rc = _gemv(lib, **kw)
    assert rc < 0
    assert msg in _lib.last_error(), _lib.last_error()


def test_gemv_empty_batch_is_a_noop():
    lib = _lib.load()
    assert _gemv(lib, M=0) == 0


def test_workspace_sizes_are_positive_and_monotone():
    lib = _lib.load()
    a = lib.qx_decode_attention_workspace_size(1, 32, 8, 128, 4, 4092)
    b = lib.qx_decode_attention_workspace_size(32, 32, 8, 128, 4, 4092)
    assert a > 0 and b > 0
    assert lib.qx_decode_attention_workspace_size(1, 30, 8, 128, 4, 4092) == 0


@pytest.mark.parametrize("call,msg", [
    (lambda L: L.qx_fused_rmsnorm(16, 16, 16, 4, 0, ctypes.c_float(1e-6), None), "bad sizes"),
    (lambda L: L.qx_fused_swiglu(None, 16, 16, 8, None), "null"),
    (lambda L: L.qx_ring_append(16, 16, 16, 16, 1, 1, 8, 128, 4, 0, 0, None), "window"),
    (lambda L: L.qx_ring_append(16, 16, 16, 16, 1, 1, 8, 128, 4, 8, -1, None), "negative"),
    (lambda L: L.qx_decode_attention(16, 16, 16, 16, 1, 32, 8, 64, 4, 8, 5, 0.0, 256, 1 << 20,
                                     None), "head_dim"),
    (lambda L: L.qx_decode_attention(16, 16, 16, 16, 1, 32, 8, 128, 4, 8, 0, 0.0, 256, 1 << 20,
                                     None), "empty cache"),
    (lambda L: L.qx_decode_attention(16, 16, 16, 16, 1, 30, 8, 128, 4, 8, 5, 0.0, 256, 1 << 20,
                                     None), "bad heads"),
])
def test_other_validation_errors(call, msg):
    lib = _lib.load()
    assert call(lib) < 0
    assert msg in _lib.last_error(), _lib.last_error()


def test_zero_size_calls_are_noops():
    lib = _lib.load()
    assert lib.qx_fused_rmsnorm(None, None, None, 0, 128, ctypes.c_float(1e-6), None) == 0
    assert lib.qx_fused_swiglu(None, None, None, 0, None) == 0
    assert lib.qx_ring_append(None, None, None, None, 1, 0, 8, 128, 4, 8, 0, None) == 0
    assert lib.qx_ring_slot_indices(None, 4, 8, 0, None) == 0


def test_ops_reject_cpu_tensors():
    import torch
    from qextract_infer_b200 import _C
    x = torch.zeros(4, 128, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        _C.fused_rmsnorm(x, torch.ones(128, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        _C.fused_swiglu(x, x)


def test_trace_entry_point_is_closed_in_the_product_library():
    """The product library carries no trace code: qx_trace_launches answers
    QX_ERR_UNSUPPORTED (only libqx_b200_trace.so records), and it validates the
    kernel family first."""
    lib = _lib.load()
    assert lib.qx_trace_launches(0, ctypes.c_void_p(16), 4) == -4
    assert "without tracing" in _lib.last_error()
    assert lib.qx_trace_launches(7, None, 0) == -1
    assert "unknown kernel" in _lib.last_error()


def test_addnorm_gemv_validation_errors():
    """qx_w4a16_lora_gemv_addnorm rejects more than 8 rows and a residual_out
    that overlaps the residual (other CTAs still read it) before any launch."""
    lib = _lib.load()
    args = lambda res, out, M: (res, 16 * 4096, 16, 1e-6, out, 16, 16, 16, 1, 0, 16, 16, 16,  # noqa: E731
                                M, 256, 128, 16, 128, 2.0, 0, None)
    assert lib.qx_w4a16_lora_gemv_addnorm(*args(16, 16 * 8192, 9)) == -1
    assert "rows" in _lib.last_error()
    assert lib.qx_w4a16_lora_gemv_addnorm(*args(16, 16 + 64, 2)) == -1
    assert "overlap" in _lib.last_error()
