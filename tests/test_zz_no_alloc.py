"""The allocation-free decode-attention entry point, called through the C ABI.

Meant for callers that may not allocate device memory while attention runs
(a framework that owns the device heap, a server plugin given only its input
and output buffers, a path where cudaMalloc would stall the device).  It must
return the same result as the workspace entry point (the tolerance used by
every attention test here: rtol = atol = 1e-2), on two calls in a row, since
every call reuses the same built-in scratch array.  This file is collected
last so a stop-at-first-failure run has already run every other test.
"""

import numpy as np
import pytest
import torch

from tests._util import assert_close

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2


def _inputs(B, Hq, Hkv, S, W, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, 128, generator=g).half().cuda()
    k = torch.randn(B, S + W, Hkv, 128, generator=g).half().cuda()
    v = torch.randn(B, S + W, Hkv, 128, generator=g).half().cuda()
    return q, k, v


def _noalloc(lib, q, k, v, count, S, W):
    out = torch.empty_like(q)
    B, Hq, D = q.shape
    rc = lib.qx_decode_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                         B, Hq, k.size(2), D, S, W, count, 0.0,
                                         torch.cuda.current_stream().cuda_stream)
    return rc, out


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _C, _lib
    lib = _lib.load()
    S, W = 4, 4092
    for call, (B, count) in enumerate([(2, 3000), (4, 32768 + 64)]):
        q, k, v = _inputs(B, 32, 8, S, W, seed=100 + call)
        rc, out = _noalloc(lib, q, k, v, count, S, W)
        assert rc == 0, _lib.last_error()
        ref = _C.decode_attention(q, k, v, count, S, W)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref.cpu().numpy(), RTOL, ATOL, f"call {call}")


def test_noalloc_rejects_oversized_scratch():
    from qextract_infer_b200 import _lib
    lib = _lib.load()
    q, k, v = _inputs(1, 32, 8, 4, 60, seed=1)
    # 2048 sequences x 8 KV heads, full 4096-slot ring: far more scratch than built in
    rc = lib.qx_decode_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.data_ptr(),
                                         512, 128, 8, 128, 4, 4092, 4096, 0.0, None)
    assert rc < 0
    assert "scratch" in _lib.last_error()
    np.testing.assert_equal(rc, -4)
