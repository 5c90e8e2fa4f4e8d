"""W4A16(-LoRA) prefill GEMM on the tcgen05 tensor cores (rows >= 128) against
the oracle (numpy, small shapes) and a torch fp32 restatement on the GPU
(large shapes).  Tolerance: rtol = atol = 1e-2 on fp16 outputs, the bar stated
for this path; the dequantised weights themselves are bit-exact fp16
s * (q - z), checked through one-hot activations.
"""

import numpy as np
import pytest
import torch

from oracle import dequantize_gptq, make_gemv_inputs, pack_qzeros, w4a16_gemv_ref, w4a16_lora_gemv_ref
from tests._util import assert_close, dev_tensor, to_np

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2


@pytest.fixture(scope="module")
def C():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _C
    return _C


def _inputs(M, K, N, rank, group=128, seed=0, random_zeros=False, packed=True):
    d = make_gemv_inputs(M, K, N, max(rank, 8), group_size=group, seed=seed, packed_zeros=packed)
    if random_zeros:
        rng = np.random.default_rng(seed + 99)
        z = rng.integers(0, 16, size=(K // group, N)).astype(np.uint8)
        d["zeros"] = pack_qzeros(z) if packed else z.astype(np.float16)
    return d


def _torch_ref(d, group, alpha, rank, zero_offset=0):
    """fp16-rounded dequantised W (oracle), then fp32 matmuls on the GPU."""
    W = dequantize_gptq(d["qweight"], d["scales"], d["zeros"], group, zero_offset=zero_offset)
    x = torch.from_numpy(d["x"]).cuda().float()
    y = x @ torch.from_numpy(np.asarray(W, dtype=np.float16)).cuda().float()
    if rank:
        A = torch.from_numpy(d["lora_A"]).cuda().float()
        B = torch.from_numpy(d["lora_B"]).cuda().float()
        y = y + float(np.float32(alpha) / np.float32(rank)) * ((x @ A) @ B)
    return y.half().cpu().numpy()


def _run(C, d, group, alpha, rank, zero_offset=0):
    t = {k: dev_tensor(v) for k, v in d.items()}
    if rank:
        return to_np(C.w4a16_lora_gemv(t["x"], t["qweight"], t["scales"], t["zeros"], t["lora_A"],
                                       t["lora_B"], group, alpha, zero_offset=zero_offset))
    return to_np(C.w4a16_gemv(t["x"], t["qweight"], t["scales"], t["zeros"], group,
                              zero_offset=zero_offset))


@pytest.mark.parametrize("M,K,N,rank,group", [
    (128, 256, 256, 16, 128), (300, 512, 512, 64, 128), (256, 1024, 768, 0, 128),
    (256, 512, 256, 8, 64), (192, 512, 512, 32, 32), (129, 256, 256, 16, 256), (256, 512, 768, 48, 128),
])
def test_against_oracle(C, M, K, N, rank, group):
    d = _inputs(M, K, N, rank, group, seed=M + K + N, random_zeros=True)
    y = _run(C, d, group, 2.0 * max(rank, 1), rank)
    if rank:
        ref = w4a16_lora_gemv_ref(d["x"], d["qweight"], d["scales"], d["zeros"], d["lora_A"],
                                  d["lora_B"], group, 2.0 * rank)
    else:
        ref = w4a16_gemv_ref(d["x"], d["qweight"], d["scales"], d["zeros"], group)
    assert y.shape == (M, N)
    assert_close(y, ref, RTOL, ATOL, f"gemm M={M} K={K} N={N} r={rank} g={group}")


def test_fp16_zeros_and_offset(C):
    d = _inputs(256, 512, 512, 16, 128, seed=5, random_zeros=True, packed=False)
    y = _run(C, d, 128, 32.0, 16)
    ref = w4a16_lora_gemv_ref(d["x"], d["qweight"], d["scales"], d["zeros"], d["lora_A"],
                              d["lora_B"], 128, 32.0)
    assert_close(y, ref, RTOL, ATOL, "fp16 zeros")
    d = _inputs(256, 512, 512, 16, 128, seed=6, random_zeros=True)
    y = _run(C, d, 128, 32.0, 16, zero_offset=1)
    ref = w4a16_lora_gemv_ref(d["x"], d["qweight"], d["scales"], d["zeros"], d["lora_A"],
                              d["lora_B"], 128, 32.0, zero_offset=1)
    assert_close(y, ref, RTOL, ATOL, "zero_offset 1")


def test_dequant_bit_exact_one_hot(C):
    """x = one-hot rows: y[i] = W[k_i, :] exactly (fp16 s*(q-z) read back)."""
    K, N = 256, 256
    d = _inputs(128, K, N, 0, 128, seed=7, random_zeros=True)
    ks = np.arange(128) * 2 + 1
    x = np.zeros((128, K), dtype=np.float16)
    x[np.arange(128), ks] = 1
    d["x"] = x
    y = _run(C, d, 128, 1.0, 0)
    W = np.asarray(dequantize_gptq(d["qweight"], d["scales"], d["zeros"], 128), dtype=np.float16)
    np.testing.assert_array_equal(y.view(np.uint16), W[ks].view(np.uint16))


@pytest.mark.parametrize("K,N", [(4096, 1024), (12288, 512)])
def test_qwen3_8b_shapes_reduced_rows(C, K, N):
    """config-3 operand sizes at 512 rows, r = 64, alpha/r = 2."""
    d = _inputs(512, K, N, 64, 128, seed=K + N)
    y = _run(C, d, 128, 128.0, 64)
    assert_close(y, _torch_ref(d, 128, 128.0, 64), RTOL, ATOL, f"K={K} N={N}")


QWEN3_8B_PROJ = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
                 ("gate", 4096, 12288), ("up", 4096, 12288), ("down", 12288, 4096)]


@pytest.mark.parametrize("name,K,N", QWEN3_8B_PROJ, ids=[p[0] for p in QWEN3_8B_PROJ])
def test_prefill_config_full_size(C, name, K, N):
    """The prefill configuration at full size: M = 4096 tokens through each of
    the 7 Qwen3-8B projections, GPTQ int4 g128 with packed qzeros (all 8),
    LoRA r = 64, alpha / r = 2, x ~ N(0, 1), against the oracle's fp16-rounded
    dequantised W followed by fp32 matmuls (reference math:
    csrc/kernels/w4a16_lora_gemv.cu:268-323, tests/test_w4a16_gemv.py:178-186)."""
    from oracle import cbind
    d = _inputs(1, K, N, 64, 128, seed=K * 7 + N)
    # x ~ N(0, 1) at 4096 rows from torch's CPU generator (the numpy one is slow at this size)
    d["x"] = torch.randn(4096, K, generator=torch.Generator().manual_seed(K + N)).half().numpy()
    y = _run(C, d, 128, 128.0, 64)
    assert y.shape == (4096, N)
    W = cbind.c_dequantize(d["qweight"], d["scales"], d["zeros"], 128)  # == oracle.dequantize_gptq
    x = torch.from_numpy(d["x"]).cuda().float()
    ref = x @ torch.from_numpy(W).cuda().float()
    A = torch.from_numpy(d["lora_A"]).cuda().float()
    B = torch.from_numpy(d["lora_B"]).cuda().float()
    ref = (ref + 2.0 * ((x @ A) @ B)).half().cpu().numpy()
    assert_close(y, ref, RTOL, ATOL, f"{name} M=4096 K={K} N={N}")


def test_matches_decode_gemv(C):
    """the GEMM at 128 rows against the decode GEMV on the same rows (32 at a time)"""
    d = _inputs(128, 1024, 512, 16, 128, seed=11, random_zeros=True)
    t = {k: dev_tensor(v) for k, v in d.items()}
    y_gemm = C.w4a16_lora_gemv(t["x"], t["qweight"], t["scales"], t["zeros"], t["lora_A"],
                               t["lora_B"], 128, 32.0)
    y_gemv = torch.cat([C.w4a16_lora_gemv(t["x"][i:i + 32], t["qweight"], t["scales"], t["zeros"],
                                          t["lora_A"], t["lora_B"], 128, 32.0)
                        for i in range(0, 128, 32)])
    assert_close(to_np(y_gemm), to_np(y_gemv), RTOL, ATOL, "gemm vs gemv")


def test_deterministic_and_no_device_error(C):
    import ctypes
    from qextract_infer_b200 import _lib
    d = _inputs(384, 1024, 768, 64, 128, seed=13)
    a = _run(C, d, 128, 128.0, 64)
    b = _run(C, d, 128, 128.0, 64)
    np.testing.assert_array_equal(a.view(np.uint16), b.view(np.uint16))
    code = ctypes.c_uint(0)
    assert _lib.load().qx_get_device_error(ctypes.byref(code), 1) == 0
    assert code.value == 0
