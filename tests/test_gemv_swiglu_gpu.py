"""The gate|up projection with the SwiGLU epilogue (``w4a16_lora_gemv_swiglu``)
against the unfused operator sequence (GEMV on the original gate|up layout,
then ``swiglu_packed``: bit-exact, the same sums rounded the same way) and
against the oracle (dequantised weights, fp32 matmuls, SwiGLU in fp32:
rtol = atol = 1e-2 on the fp16 output)."""

import numpy as np
import pytest
import torch

from oracle import make_gemv_inputs, w4a16_lora_gemv_ref
from tests._util import assert_close, dev_tensor, to_np

RTOL = ATOL = 1e-2


@pytest.fixture(scope="module")
def C():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _C
    return _C


def _inputs(M, K, inter, rank, seed):
    d = make_gemv_inputs(M, K, 2 * inter, rank, seed=seed)
    rng = np.random.default_rng(seed + 1)
    # random zero points (not all 8), so that the packed qzeros reordering matters
    d["zeros"] = rng.integers(0, 2 ** 32, size=d["zeros"].shape, dtype=np.uint64).astype(
        np.uint32).view(np.int32)
    return d


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,inter,rank", [(1, 4096, 12288, 32), (1, 4096, 1536, 32),
                                            (3, 4096, 3072, 32), (8, 2560, 9728, 16),
                                            (16, 4096, 1536, 32), (32, 4096, 12288, 32),
                                            (1, 1024, 256, 0), (5, 1024, 520, 8)])
def test_matches_unfused_sequence_and_oracle(C, M, K, inter, rank):
    d = _inputs(M, K, inter, rank, seed=M * 7 + inter)
    t = {k: dev_tensor(v) for k, v in d.items()}
    alpha = 2.0 * rank if rank else 16.0
    if rank:
        gu = C.w4a16_lora_gemv(t["x"], t["qweight"], t["scales"], t["zeros"], t["lora_A"],
                               t["lora_B"], 128, alpha)
    else:
        gu = C.w4a16_gemv(t["x"], t["qweight"], t["scales"], t["zeros"], 128)
    ref_seq = to_np(C.swiglu_packed(gu))
    il = C.interleave_gate_up
    qw, sc = il(t["qweight"], inter), il(t["scales"], inter)
    qz = il(t["zeros"], inter, packed=True)
    for _ in range(2):  # two calls in a row (cached launch parameters on the second)
        if rank:
            y = to_np(C.w4a16_lora_gemv_swiglu(t["x"], qw, sc, qz, t["lora_A"], il(t["lora_B"], inter),
                                               128, alpha))
        else:
            y = to_np(C._w4a16_swiglu(t["x"], qw, sc, qz, None, None, 128, 0.0, 0))
        assert y.shape == (M, inter)
        np.testing.assert_array_equal(y.view(np.uint16), ref_seq.view(np.uint16))
    # the gate|up sums the epilogue rounds are the GEMV's: those meet the oracle
    # at the stated tolerance (SwiGLU then amplifies an fp16 rounding of g or u
    # by up to |u| or |silu(g)|, as it does in the reference's own sequence)
    if rank:
        ref = w4a16_lora_gemv_ref(d["x"], d["qweight"], d["scales"], d["zeros"], d["lora_A"],
                                  d["lora_B"], 128, alpha)
    else:
        z = np.zeros((K, 8), np.float16)
        ref = w4a16_lora_gemv_ref(d["x"], d["qweight"], d["scales"], d["zeros"], z,
                                  np.zeros((8, 2 * inter), np.float16), 128, 16.0)
    assert_close(to_np(gu), ref, RTOL, ATOL, "gate|up sums vs oracle")


@pytest.mark.gpu
def test_prefill_rows_take_the_gemm(C):
    """128 rows route to the tensor-core GEMM and SwiGLU over the gathered
    gate and up columns: equal to the GEMM on the original layout + SwiGLU."""
    M, K, inter, rank = 128, 1024, 1536, 32
    d = _inputs(M, K, inter, rank, seed=3)
    t = {k: dev_tensor(v) for k, v in d.items()}
    gu = C.w4a16_lora_gemv(t["x"], t["qweight"], t["scales"], t["zeros"], t["lora_A"], t["lora_B"],
                           128, 64.0)
    ref_seq = to_np(C.swiglu_packed(gu))
    il = C.interleave_gate_up
    y = to_np(C.w4a16_lora_gemv_swiglu(t["x"], il(t["qweight"], inter), il(t["scales"], inter),
                                       il(t["zeros"], inter, packed=True), t["lora_A"],
                                       il(t["lora_B"], inter), 128, 64.0))
    assert_close(y, ref_seq, RTOL, ATOL, "prefill swiglu vs GEMM + swiglu_packed")


def test_interleave_layout():
    """Column 16 b + j is gate column 8 b + j, column 16 b + 8 + j up column
    8 b + j; packed words alternate gate word b, up word b."""
    from qextract_infer_b200._C import interleave_gate_up
    inter = 24
    t = torch.arange(2 * inter).view(1, -1)
    got = interleave_gate_up(t, inter)[0].tolist()
    want = []
    for b in range(inter // 8):
        want += list(range(8 * b, 8 * b + 8)) + list(range(inter + 8 * b, inter + 8 * b + 8))
    assert got == want
    w = torch.arange(2 * inter // 8).view(1, -1)
    assert interleave_gate_up(w, inter, packed=True)[0].tolist() == [0, 3, 1, 4, 2, 5]
