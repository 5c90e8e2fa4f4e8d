"""The NVLink all-reduce's bounded peer wait and its reduction, on one GPU.

Two ranks' contexts live in this process on cuda:0 (``qx_nvlink_ar_open_local``),
so no second GPU is needed and no two waiting kernels ever run at once:

1. rank 0 calls alone: rank 1's flag is never set, so rank 0's wait runs out
   after the short limit (50 ms); the call returns, the device error word holds
   ``QX_DEVERR_PEER_TIMEOUT`` and reading it with reset clears it;
2. rank 1 calls next: rank 0 published its row in (1), so rank 1's wait is
   already satisfied; its output is the full all-reduce + residual add +
   RMSNorm of both partials, checked against a torch fp32 restatement
   (residual bit-exact, normalised output within rtol = atol = 1e-2).
"""

import ctypes
import time

import numpy as np
import pytest
import torch

from tests._util import assert_close

pytestmark = pytest.mark.gpu
QX_DEVERR_PEER_TIMEOUT = 2


def _create(lib, world, rank, rows, hidden):
    from qextract_infer_b200 import _lib
    ctx = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(int(lib.qx_nvlink_ar_handle_bytes()))
    _lib.check(lib.qx_nvlink_ar_create(world, rank, rows, hidden, ctypes.byref(ctx), handle),
               "nvlink_ar_create")
    return ctx


def _device_error(lib, reset):
    code = ctypes.c_uint(0)
    assert lib.qx_get_device_error(ctypes.byref(code), reset) == 0
    return code.value


def test_peer_wait_times_out_then_reduction_is_exact():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _lib
    lib = _lib.load()
    torch.cuda.set_device(0)
    rows, hidden, eps = 2, 4096, 1e-6
    ctx = [_create(lib, 2, r, rows, hidden) for r in range(2)]
    arr = (ctypes.c_void_p * 2)(ctx[0].value, ctx[1].value)
    try:
        for c in ctx:
            _lib.check(lib.qx_nvlink_ar_open_local(c, arr), "nvlink_ar_open_local")
        assert lib.qx_nvlink_ar_set_timeout(ctx[0], 0) < 0  # the limit must be positive
        _lib.check(lib.qx_nvlink_ar_set_timeout(ctx[0], 50_000_000), "set_timeout")
        _device_error(lib, 1)
        g = torch.Generator(device="cuda").manual_seed(5)
        part = [torch.randn(rows, hidden, generator=g, device="cuda").half() for _ in range(2)]
        x = [torch.randn(rows, hidden, generator=g, device="cuda").half() for _ in range(2)]
        x0 = [t.clone() for t in x]
        w = (torch.randn(hidden, generator=g, device="cuda") * 0.1 + 1).half()
        y = [torch.empty_like(t) for t in x]
        st = torch.cuda.current_stream().cuda_stream

        def call(r):
            _lib.check(lib.qx_nvlink_ar_add_rmsnorm(ctx[r], part[r].data_ptr(), x[r].data_ptr(),
                                                     w.data_ptr(), y[r].data_ptr(), rows,
                                                     ctypes.c_float(eps), st), "nvlink_ar_add_rmsnorm")

        torch.cuda.synchronize()
        t0 = time.monotonic()
        call(0)  # rank 1 never publishes: the bounded wait runs out
        torch.cuda.synchronize()
        assert time.monotonic() - t0 < 5.0
        assert _device_error(lib, 1) & QX_DEVERR_PEER_TIMEOUT
        assert _device_error(lib, 0) == 0  # the reset cleared it

        call(1)  # rank 0's row of this epoch is already published: no wait
        torch.cuda.synchronize()
        assert _device_error(lib, 0) == 0
        s = (part[0].float() + part[1].float()).half()          # rank-ordered fp32 sum, one rounding
        xr = (x0[1].float() + s.float()).half()                  # residual add
        np.testing.assert_array_equal(x[1].cpu().numpy().view(np.uint16), xr.cpu().numpy().view(np.uint16))
        xf = xr.float()
        ref = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).half()
        assert_close(y[1].cpu().numpy(), ref.cpu().numpy(), 1e-2, 1e-2, "all-reduce + add + RMSNorm")
    finally:
        for c in ctx:
            lib.qx_nvlink_ar_destroy(c)
