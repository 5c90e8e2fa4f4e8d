"""Resident decode GEMV (csrc/w4a16_gemv_res.cu) on the GPU: the kernel that
qx_w4a16_lora_gemv routes up to 4 rows to when a CTA's weight slice fits half
an SM.  Checked against the oracle (rtol = atol = 1e-2 on fp16 outputs), the
clustered split-K kernel on the same inputs, bit-exact int4 unpacking and
dequantisation through the kernel, determinism, activations with a wide
dynamic range inside a quantisation group (the kernel's fixed-point digits),
and chains of calls on one stream (programmatic dependent launch overlaps
consecutive calls).
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import (dequantize_gptq, make_gemv_inputs, unpack_int4_rows, w4a16_gemv_ref,
                    w4a16_lora_gemv_ref)
from oracle import cbind
from tests._util import assert_close, dev_tensor, to_np

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2


@pytest.fixture(scope="module")
def C():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _C
    return _C


@pytest.fixture(scope="module")
def lib():
    from qextract_infer_b200 import _lib
    lib = _lib.load()
    lib.qx_set_gemv_resident(1)  # routed on for this module, restored after
    yield lib
    lib.qx_set_gemv_resident(0)


def route(lib, M, K, N, rank, group=128, packed=1):
    k = ctypes.c_int(-1)
    assert lib.qx_w4a16_gemv_route(M, K, N, rank, group, packed, ctypes.byref(k)) == 0
    return k.value


def _dev(d):
    return {k: dev_tensor(v) for k, v in d.items()}


def _run(C, t, group, alpha, rank):
    if rank:
        return to_np(C.w4a16_lora_gemv(t["x"], t["qweight"], t["scales"], t["zeros"], t["lora_A"],
                                       t["lora_B"], group, alpha))
    return to_np(C.w4a16_gemv(t["x"], t["qweight"], t["scales"], t["zeros"], group))


def test_routes(lib):
    assert route(lib, 1, 2560, 9728, 16) == 1       # Qwen3-4B gate_proj decode (the headline shape)
    assert route(lib, 2, 2560, 4864, 16) == 1
    assert route(lib, 4, 2560, 9728, 16) == 0       # activations of 4 rows + weights exceed half an SM
    assert route(lib, 5, 2048, 2048, 16) == 0       # more rows than the kernel takes
    assert route(lib, 1, 4096, 24576, 32) == 0      # fused gate|up: slice too large for half an SM
    assert route(lib, 1, 4096, 4096, 16) == 1       # o_proj
    lib.qx_set_gemv_resident(0)
    try:
        assert route(lib, 1, 2560, 9728, 16) == 0
    finally:
        lib.qx_set_gemv_resident(1)


@pytest.mark.parametrize("M,K,N,rank,group,packed", [
    (1, 2560, 9728, 16, 128, True),     # config 0
    (2, 2560, 4864, 16, 128, True),
    (3, 1024, 1232, 8, 128, True),      # N/8 = 154 units: CTAs of 1 and 2 units
    (4, 2048, 4096, 16, 128, True),
    (1, 4096, 4096, 16, 128, True),     # o_proj
    (1, 4096, 3072, 32, 128, True),     # clusters of 8
    (1, 2048, 4096, 64, 64, True),
    (2, 1024, 2048, 128, 32, True),
    (1, 512, 4096, 0, 128, True),
    (1, 2560, 9728, 16, 128, False),    # fp16 zeros (reference kernel format)
    (1, 768, 296, 16, 256, True),       # U = 37 < SMs: one unit per CTA
    (2, 6144, 1184, 8, 128, True),      # three weight chunks
])
def test_against_oracle_and_split_k(C, lib, M, K, N, rank, group, packed):
    assert route(lib, M, K, N, rank, group, int(packed)) == 1, "shape expected on the resident kernel"
    d = make_gemv_inputs(M, K, N, max(rank, 8), group_size=group, seed=K + N + rank + M,
                         packed_zeros=packed)
    if not packed:
        rng = np.random.default_rng(5)
        d["zeros"] = rng.uniform(0, 15, size=d["zeros"].shape).astype(np.float16)
    t = _dev(d)
    alpha = 2.0 * max(rank, 1)
    y = _run(C, t, group, alpha, rank)
    if rank:
        ref = w4a16_lora_gemv_ref(d["x"], d["qweight"], d["scales"], d["zeros"], d["lora_A"],
                                  d["lora_B"], group, alpha)
    else:
        ref = w4a16_gemv_ref(d["x"], d["qweight"], d["scales"], d["zeros"], group)
    assert_close(y, ref, RTOL, ATOL, f"resident vs oracle M={M} K={K} N={N} r={rank}")
    lib.qx_set_gemv_resident(0)
    try:
        y_split = _run(C, t, group, alpha, rank)
    finally:
        lib.qx_set_gemv_resident(1)
    assert_close(y, y_split, RTOL, ATOL, "resident vs split-K kernel")
    y2 = _run(C, t, group, alpha, rank)
    np.testing.assert_array_equal(y.view(np.uint16), y2.view(np.uint16))


def test_decode_config_against_c_oracle(C, lib):
    """Qwen3-4B gate_proj: x [1,2560], packed qzeros (all 8), LoRA r16, alpha/r = 2."""
    d = make_gemv_inputs(1, 2560, 9728, 16, seed=0)
    t = _dev(d)
    y = to_np(C.w4a16_lora_gemv(t["x"], t["qweight"], t["scales"], t["zeros"], t["lora_A"],
                                t["lora_B"], 128, 32.0))
    ref = cbind.c_w4a16_lora_gemv(d["x"], d["qweight"], d["scales"], d["zeros"], d["lora_A"],
                                  d["lora_B"], 128, 32.0)
    assert_close(y, ref, RTOL, ATOL, "decode config vs C oracle")


@pytest.mark.parametrize("spread", [1e2, 1e4])
def test_wide_dynamic_range_activations(C, lib, spread):
    """Activations spanning `spread` within every quantisation group (one large
    entry per group, the rest small): the fixed-point digits keep 2^-14 of the
    group maximum, far inside the tolerance relative to the output."""
    M, K, N = 1, 2560, 2048
    assert route(lib, M, K, N, 16) == 1
    d = make_gemv_inputs(M, K, N, 16, seed=77)
    rng = np.random.default_rng(78)
    x = (rng.standard_normal((M, K)) / spread).astype(np.float32)
    x[:, ::128] = rng.choice([-4.0, 4.0], size=(M, K // 128))
    d["x"] = x.astype(np.float16)
    t = _dev(d)
    y = _run(C, t, 128, 32.0, 16)
    ref = w4a16_lora_gemv_ref(d["x"], d["qweight"], d["scales"], d["zeros"], d["lora_A"],
                              d["lora_B"], 128, 32.0)
    assert_close(y, ref, RTOL, ATOL, f"dynamic range {spread}")


def _onehot_rows(C, qw, sc, zs, K, group=128, zero_offset=0):
    rows = []
    for k0 in range(0, K, 4):  # 4 rows per call: the resident kernel's batch limit
        x = torch.zeros(4, K, dtype=torch.float16, device="cuda")
        x[torch.arange(4), torch.arange(k0, k0 + 4)] = 1.0
        rows.append(to_np(C.w4a16_gemv(x, qw, sc, zs, group, zero_offset=zero_offset)))
    return np.concatenate(rows, axis=0)


def test_unpack_and_dequant_bit_exact(C, lib):
    K, N = 256, 200
    assert route(lib, 4, K, N, 0) == 1
    rng = np.random.default_rng(21)
    qweight = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.uint64).astype(np.uint32).view(np.int32)
    ones = np.ones((K // 128, N), dtype=np.float16)
    zero = np.zeros((K // 128, N // 8), dtype=np.int32)
    got = _onehot_rows(C, dev_tensor(qweight), dev_tensor(ones), dev_tensor(zero), K)
    np.testing.assert_array_equal(got.astype(np.int64), unpack_int4_rows(qweight).astype(np.int64))
    scales = rng.uniform(0.005, 0.02, size=(K // 128, N)).astype(np.float16)
    qzeros = rng.integers(0, 2 ** 32, size=(K // 128, N // 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
    for off in (0, 1):
        got = _onehot_rows(C, dev_tensor(qweight), dev_tensor(scales), dev_tensor(qzeros), K,
                           zero_offset=off)
        want = dequantize_gptq(qweight, scales, qzeros, 128, zero_offset=off)
        np.testing.assert_array_equal(got.view(np.uint16), want.view(np.uint16))


def test_chain_of_calls_on_one_stream(C, lib):
    """Six calls back to back with different weights, the output of each the
    activations of the next (GEMV to GEMV, so consecutive calls overlap under
    programmatic dependent launch): the dependency wait must order every read
    of x after its producer.  Each call is checked against the oracle on the
    activations the GPU produced."""
    K = N = 2048
    sets = [make_gemv_inputs(1, K, N, 16, seed=100 + i, packed_zeros=False) for i in range(6)]
    for d in sets:  # zero-mean weights (z = 7.5) and unit gain keep every call's output O(1)
        d["zeros"][:] = np.float16(7.5)
        d["scales"] = (d["scales"].astype(np.float32) * 0.36).astype(np.float16)
    assert route(lib, 1, K, N, 16, packed=0) == 1
    dev = [_dev(d) for d in sets]
    x = dev[0]["x"]
    outs = []
    for t in dev:
        x = C.w4a16_lora_gemv(x, t["qweight"], t["scales"], t["zeros"], t["lora_A"], t["lora_B"],
                              128, 32.0)
        outs.append(x)
    torch.cuda.synchronize()
    xin = sets[0]["x"]
    for i, d in enumerate(sets):
        ref = w4a16_lora_gemv_ref(xin, d["qweight"], d["scales"], d["zeros"], d["lora_A"], d["lora_B"],
                                  128, 32.0)
        got = to_np(outs[i])
        assert np.isfinite(got).all()
        assert_close(got, ref, RTOL, ATOL, f"chained call {i}")
        xin = got
