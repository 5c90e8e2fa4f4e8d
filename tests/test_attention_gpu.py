"""GQA decode attention read in place from the ring, against the fp32 oracle
on the gathered (logical-order) K/V.  Tolerance rtol = atol = 1e-2 on the fp16
output.  Parity unpinned by the reference (it has no attention kernel)."""

import numpy as np
import pytest
import torch

from oracle import RingIndexOracle, gqa_decode_attention_ref
from tests._util import assert_close, dev_tensor, to_np

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2


@pytest.fixture(scope="module")
def C():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _C
    return _C


def _run(C, B, Hq, Hkv, S, W, count, seed, scale=None, kv_std=1.0):
    D = 128
    cap = S + W
    rng = np.random.default_rng(seed)
    k = (rng.standard_normal((B, cap, Hkv, D), dtype=np.float32) * kv_std).astype(np.float16)
    v = rng.standard_normal((B, cap, Hkv, D), dtype=np.float32).astype(np.float16)
    q = rng.standard_normal((B, Hq, D), dtype=np.float32).astype(np.float16)
    out = to_np(C.decode_attention(dev_tensor(q), dev_tensor(k), dev_tensor(v), count, S, W, scale))
    idx = RingIndexOracle(S, W).indices(count)
    for b in range(B):
        ref = gqa_decode_attention_ref(q[b], k[b][idx], v[b][idx], scale)
        assert_close(out[b], ref, RTOL, ATOL, f"b={b} count={count}")
    return out


@pytest.mark.parametrize("count", [1, 3, 4, 5, 17, 64, 65, 100, 1000, 4095, 4096, 4097, 5000,
                                   32768 + 64])
def test_qwen3_8b_geometry(C, count):
    _run(C, 1, 32, 8, 4, 4092, count, seed=count)


@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (16, 8), (32, 8), (64, 8), (128, 8), (32, 2), (4, 1)])
def test_gqa_groups(C, Hq, Hkv):
    _run(C, 2, Hq, Hkv, 4, 1020, 777, seed=Hq * 10 + Hkv)


@pytest.mark.parametrize("B", [1, 4, 32])
def test_batch(C, B):
    _run(C, B, 32, 8, 4, 4092, 4096 + 123, seed=B)


def test_small_rings_and_scale(C):
    for S, W, count in [(0, 1, 5), (1, 1, 1), (4, 8, 12), (2, 70, 200), (4, 60, 64)]:
        _run(C, 1, 8, 2, S, W, count, seed=S * 100 + W)
    _run(C, 1, 32, 8, 4, 4092, 3000, seed=9, scale=0.05)


def test_peaked_scores(C):
    """Large-magnitude keys: softmax close to one-hot exercises the running max."""
    _run(C, 1, 32, 8, 4, 4092, 4096, seed=3, kv_std=8.0)


def test_cache_object_path(C):
    import qextract_infer_b200 as q
    cache = q.QExtractKVCache(2, 8, 128, sink_size=4, window_size=60)
    rng = np.random.default_rng(1)
    ks = rng.standard_normal((100, 8, 128), dtype=np.float32).astype(np.float16)
    vs = rng.standard_normal((100, 8, 128), dtype=np.float32).astype(np.float16)
    for layer in range(2):
        cache.append(dev_tensor(ks[:70]), dev_tensor(vs[:70]), layer)
    for t in range(70, 100):
        for layer in range(2):
            cache.append(dev_tensor(ks[t]), dev_tensor(vs[t]), layer)
    qv = rng.standard_normal((32, 128), dtype=np.float32).astype(np.float16)
    out = to_np(cache.decode_attention(dev_tensor(qv), 1))
    k, v = cache.get_kv(1)
    ref = gqa_decode_attention_ref(qv, to_np(k), to_np(v))
    assert_close(out, ref, RTOL, ATOL, "cache object")
    pos = RingIndexOracle(4, 60).positions(100)
    np.testing.assert_array_equal(to_np(k), ks[pos])


def test_after_gemv_with_many_tiles(C):
    """Attention after a GEMV whose tile count exceeds 64 on the same stream
    (the two ops keep separate workspaces)."""
    from oracle import make_gemv_inputs
    d = make_gemv_inputs(1, 1024, 24576, 16, seed=1)
    t = {k: dev_tensor(v) for k, v in d.items()}
    C.w4a16_lora_gemv(t["x"], t["qweight"], t["scales"], t["zeros"], t["lora_A"], t["lora_B"])
    _run(C, 32, 32, 8, 4, 4092, 4096 + 5, seed=77)


@pytest.mark.parametrize("B,Hq,Hkv,count", [(1, 32, 8, 4096 + 7), (1, 4, 1, 4096), (1, 16, 4, 2000),
                                            (2, 32, 8, 4096), (4, 32, 8, 3000), (1, 32, 8, 130),
                                            (3, 8, 8, 1500)])
def test_merge_modes_agree(C, B, Hq, Hkv, count):
    """The cluster merge (default) and the workspace merge, each against the
    oracle, and against each other within fp32-rounding distance."""
    from qextract_infer_b200 import _lib
    lib = _lib.load()
    try:
        _lib.check(lib.qx_decode_attention_pin_merge(1), "pin_merge")
        a = _run(C, B, Hq, Hkv, 4, 4092, count, seed=count + B)
        _lib.check(lib.qx_decode_attention_pin_merge(0), "pin_merge")
        b = _run(C, B, Hq, Hkv, 4, 4092, count, seed=count + B)
    finally:
        lib.qx_decode_attention_pin_merge(0)
    assert_close(a, b, 2e-3, 2e-3, "cluster vs workspace merge")
    assert lib.qx_decode_attention_pin_merge(2) < 0
