"""Fused RMSNorm / SwiGLU on the GPU against the oracle and the reference's
golden vectors (tolerance rtol = atol = 1e-2, as in tests/test_rmsnorm.py and
tests/test_swiglu.py of the reference)."""

import numpy as np
import pytest
import torch

from oracle import rmsnorm_ref, swiglu_ref, swiglu_ref_single_round
from tests._util import assert_close, dev_tensor, f16_ulp_diff, load_golden, to_np

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2


@pytest.fixture(scope="module")
def C():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _C
    return _C


def test_rmsnorm_golden(C):
    d = load_golden("rmsnorm")
    for i in range(5):
        y = to_np(C.fused_rmsnorm(dev_tensor(d[f"x{i}"]), dev_tensor(d[f"w{i}"]), float(d[f"eps{i}"])))
        assert_close(y, d[f"y{i}"], RTOL, ATOL, f"rmsnorm golden {i}")
        assert f16_ulp_diff(y, d[f"y{i}"]).max() <= 2


@pytest.mark.parametrize("H", [2560, 4096])
@pytest.mark.parametrize("T", [1, 8, 64, 4096])
def test_rmsnorm_config(C, H, T):
    rng = np.random.default_rng(1000 * T + H)
    x = rng.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    w = (rng.standard_normal(H, dtype=np.float32) * 0.1 + 1.0).astype(np.float16)
    y = to_np(C.fused_rmsnorm(dev_tensor(x), dev_tensor(w), 1e-6))
    assert_close(y, rmsnorm_ref(x, w, 1e-6), RTOL, ATOL, f"T={T} H={H}")


@pytest.mark.parametrize("H", [1, 7, 100, 128, 256, 512, 768, 1000, 1024, 2048, 4104, 8192, 16384])
def test_rmsnorm_hidden_sizes(C, H):
    rng = np.random.default_rng(H)
    x = rng.standard_normal((3, H), dtype=np.float32).astype(np.float16)
    w = rng.standard_normal(H, dtype=np.float32).astype(np.float16)
    for eps in (1e-5, 1e-6, 1e-8):
        y = to_np(C.fused_rmsnorm(dev_tensor(x), dev_tensor(w), eps))
        assert_close(y, rmsnorm_ref(x, w, eps), RTOL, ATOL, f"H={H} eps={eps}")


def test_rmsnorm_3d_and_misaligned(C):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 128, 2560), dtype=np.float32).astype(np.float16)
    w = rng.standard_normal(2560, dtype=np.float32).astype(np.float16)
    y = C.fused_rmsnorm(dev_tensor(x), dev_tensor(w))
    assert tuple(y.shape) == (2, 128, 2560)
    assert_close(to_np(y), rmsnorm_ref(x, w), RTOL, ATOL, "3-D")
    # a view starting 1 element in: not 16-byte aligned -> scalar path
    big = dev_tensor(rng.standard_normal(2 * 256 + 1, dtype=np.float32).astype(np.float16))
    xv = big[1:].view(2, 256)
    wv = dev_tensor(np.ones(256, dtype=np.float16))
    assert_close(to_np(C.fused_rmsnorm(xv, wv)), rmsnorm_ref(to_np(xv), np.ones(256, np.float16)),
                 RTOL, ATOL, "misaligned")


def test_rmsnorm_errors(C):
    x = torch.randn(4, 256, device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="float16"):
        C.fused_rmsnorm(x.float(), torch.ones(256, device="cuda", dtype=torch.float16))
    with pytest.raises(RuntimeError, match="size mismatch"):
        C.fused_rmsnorm(x, torch.ones(128, device="cuda", dtype=torch.float16))
    with pytest.raises(RuntimeError, match="contiguous"):
        C.fused_rmsnorm(x.t(), torch.ones(4, device="cuda", dtype=torch.float16))


def test_swiglu_golden(C):
    d = load_golden("swiglu")
    tols = [(RTOL, ATOL)] * 3 + [(0.1, 0.5), (1e-2, 1e-3), (RTOL, ATOL)]
    for i in range(6):
        y = to_np(C.fused_swiglu(dev_tensor(d[f"g{i}"]), dev_tensor(d[f"u{i}"])))
        rt, at = tols[i]
        assert_close(y, d[f"y{i}"], rt, at, f"swiglu golden {i}")


@pytest.mark.parametrize("I", [9728, 12288])
@pytest.mark.parametrize("T", [1, 8, 64, 4096])
def test_swiglu_config(C, I, T):
    rng = np.random.default_rng(7 * T + I)
    g = rng.standard_normal((T, I), dtype=np.float32).astype(np.float16)
    u = rng.standard_normal((T, I), dtype=np.float32).astype(np.float16)
    y = to_np(C.fused_swiglu(dev_tensor(g), dev_tensor(u)))
    assert_close(y, swiglu_ref(g, u), RTOL, ATOL, f"T={T} I={I}")
    assert f16_ulp_diff(y, swiglu_ref_single_round(g, u)).max() <= 2


@pytest.mark.parametrize("n", [1, 7, 8, 1001, 4096, 65536 + 3])
def test_swiglu_sizes(C, n):
    rng = np.random.default_rng(n)
    g = (rng.standard_normal(n, dtype=np.float32) * 4).astype(np.float16)
    u = rng.standard_normal(n, dtype=np.float32).astype(np.float16)
    y = to_np(C.fused_swiglu(dev_tensor(g), dev_tensor(u)))
    assert_close(y, swiglu_ref(g, u), RTOL, ATOL, f"n={n}")


def test_swiglu_extremes(C):
    g = dev_tensor(np.float16([-65504, -100, -20, -1e-4, 0, 1e-4, 20, 100, 65504, -0.0]))
    u = dev_tensor(np.float16([1, 2, 3, 4, 5, 6, 7, 8, 0.5, 1]))
    y = to_np(C.fused_swiglu(g, u)).astype(np.float32)
    ref = swiglu_ref_single_round(to_np(g), to_np(u)).astype(np.float32)
    assert np.all(np.isfinite(y[:-2]))
    assert_close(y[:8], ref[:8], RTOL, ATOL, "extremes")


def test_swiglu_errors(C):
    g = torch.randn(4, 256, device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="same shape"):
        C.fused_swiglu(g, g[:, :128].contiguous())
