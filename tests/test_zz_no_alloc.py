"""The allocation-free decode-attention entry point, called through the C ABI.

Meant for callers that may not allocate device memory while attention runs
(a framework that owns the device heap, a server plugin given only its input
and output buffers, a path where cudaMalloc would stall the device).  It must
return the same result as the workspace entry point and as the CPU oracle
(the tolerance used by every attention test here: rtol = atol = 1e-2), on
calls in a row, since every call reuses the same built-in scratch array.
Shapes covered: the Qwen3-8B geometry at 2, 4 and 32 sequences (the largest
batch the header promises is far above 32), 16 query heads per KV head at one
sequence (the most chunks, the largest scratch of that geometry), and the
shape right at the scratch limit, accepted, with the next larger rejected.
This file is collected last so a stop-at-first-failure run has already run
every other test.
"""

import os
import re

import numpy as np
import pytest
import torch

from oracle import gqa_decode_attention_ref
from tests._util import assert_close

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2
HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "qx_b200.h")


def _scratch_limit():
    m = re.search(r"#define QX_DECODE_ATTN_NOALLOC_SCRATCH_BYTES \((\d+) << (\d+)\)", open(HEADER).read())
    return int(m.group(1)) << int(m.group(2))


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


def _oracle(q, k, v, count, S, W, seqs):
    """fp32 attention over the valid slots (the physical prefix; order does not matter)."""
    valid = count if count <= S else S + min(count - S, W)
    qn, kn, vn = q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()
    return np.stack([gqa_decode_attention_ref(qn[b], kn[b, :valid], vn[b, :valid]) for b in seqs])


@pytest.mark.parametrize("B,Hq,Hkv,count,seqs", [
    (2, 32, 8, 3000, [0, 1]),                  # Qwen3-8B heads, ring not yet wrapped
    (4, 32, 8, 32768 + 64, [0, 3]),            # wrapped ring, 4096 valid slots
    (32, 32, 8, 32768 + 64, [0, 17, 31]),      # 32 sequences
    (1, 128, 8, 32768 + 64, [0]),              # 16 query heads per KV head: the most chunks
])
def test_noalloc_matches_workspace_entry_point_and_oracle(B, Hq, Hkv, count, seqs):
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _C, _lib
    lib = _lib.load()
    S, W = 4, 4092
    assert lib.qx_decode_attention_workspace_size(B, Hq, Hkv, 128, S, W) <= _scratch_limit()
    for call in range(2):  # two calls in a row: the array keeps the last call's contents
        q, k, v = _inputs(B, Hq, Hkv, S, W, seed=100 * B + call)
        rc, out = _noalloc(lib, q, k, v, count, S, W)
        assert rc == 0, _lib.last_error()
        ref = _C.decode_attention(q, k, v, count, S, W)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert_close(got, ref.cpu().numpy(), RTOL, ATOL, f"B={B} call {call} vs workspace entry")
        assert_close(got[seqs], _oracle(q, k, v, count, S, W, seqs), RTOL, ATOL,
                     f"B={B} call {call} vs oracle")


def test_noalloc_scratch_limit_boundary():
    """The largest accepted shape runs and matches; one more sequence is rejected."""
    from qextract_infer_b200 import _C, _lib
    lib = _lib.load()
    Hq, Hkv, S, W = 16, 1, 4, 60
    limit = _scratch_limit()
    size = lambda b: lib.qx_decode_attention_workspace_size(b, Hq, Hkv, 128, S, W)  # noqa: E731
    B = 1
    while size(B + 1) <= limit:
        B += 1
    assert size(B) <= limit < size(B + 1)
    q, k, v = _inputs(B, Hq, Hkv, S, W, seed=7)
    for call in range(2):
        rc, out = _noalloc(lib, q, k, v, 100, S, W)
        assert rc == 0, _lib.last_error()
        ref = _C.decode_attention(q, k, v, 100, S, W)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref.cpu().numpy(), RTOL, ATOL, f"B={B} at the limit, call {call}")
    assert_close(out.cpu().numpy()[:2], _oracle(q, k, v, 100, S, W, [0, 1]), RTOL, ATOL, "limit vs oracle")
    q2, k2, v2 = _inputs(B + 1, Hq, Hkv, S, W, seed=8)
    rc, _ = _noalloc(lib, q2, k2, v2, 100, S, W)
    assert rc == -4  # QX_ERR_UNSUPPORTED
    assert "scratch" in _lib.last_error()


def test_noalloc_rejects_oversized_scratch():
    from qextract_infer_b200 import _lib
    lib = _lib.load()
    q, k, v = _inputs(1, 32, 8, 4, 60, seed=1)
    # 512 sequences x 8 KV heads, full 4096-slot ring: far more scratch than built in
    rc = lib.qx_decode_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.data_ptr(),
                                         512, 128, 8, 128, 4, 4092, 4096, 0.0, None)
    assert rc < 0
    assert "scratch" in _lib.last_error()
    np.testing.assert_equal(rc, -4)
