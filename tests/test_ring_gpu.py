"""Ring-buffer KV cache on the GPU: the reference's known-answer tests
(tests/test_kv_cache.py), the golden trace produced by the reference's own
cache, and bit-exact slot / content checks against the oracle, including the
Qwen3-8B streaming geometry (4 sink + 4092 window, 2048-token chunks, then
single-token decode appends)."""

import numpy as np
import pytest
import torch

from oracle import RingCacheOracle, RingIndexOracle
from tests._util import dev_tensor, load_golden, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def Q():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    import qextract_infer_b200 as q
    assert q._C_AVAILABLE
    return q


def _cache(Q, **kw):
    d = dict(num_layers=2, num_kv_heads=8, head_dim=128, sink_size=4, window_size=8)
    d.update(kw)
    return Q.QExtractKVCache(**d)


def test_basic_append_get(Q):
    c = _cache(Q)
    for _ in range(3):
        for layer in range(2):
            c.append(torch.randn(8, 128, dtype=torch.float16, device="cuda"),
                     torch.randn(8, 128, dtype=torch.float16, device="cuda"), layer)
    assert c.valid_length == 3
    k, v = c.get_kv(0)
    assert tuple(k.shape) == (3, 8, 128) and tuple(v.shape) == (3, 8, 128)


def test_sink_preservation(Q):
    c = _cache(Q, sink_size=4, window_size=4)
    sinks = []
    for step in range(4):
        k = torch.full((8, 128), float(step), dtype=torch.float16, device="cuda")
        sinks.append(k.clone())
        for layer in range(2):
            c.append(k, torch.zeros_like(k), layer)
    for step in range(20):
        k = torch.full((8, 128), 100.0 + step, dtype=torch.float16, device="cuda")
        for layer in range(2):
            c.append(k, torch.zeros_like(k), layer)
    assert c.valid_length == 8
    k_out, _ = c.get_kv(0)
    for i in range(4):
        assert torch.equal(k_out[i], sinks[i])


def test_wrap_around_known_answer(Q):
    c = _cache(Q, sink_size=2, window_size=4)
    for step in range(10):
        k = torch.full((8, 128), float(step), dtype=torch.float16, device="cuda")
        for layer in range(2):
            c.append(k, torch.zeros_like(k), layer)
    assert c.valid_length == 6
    k_out, _ = c.get_kv(0)
    np.testing.assert_array_equal(to_np(k_out[:, 0, 0]), load_golden("ring")["wrap_k00"])


def test_valid_length_progression_and_reset(Q):
    c = _cache(Q, sink_size=4, window_size=8)
    lengths = []
    for _ in range(20):
        for layer in range(2):
            c.append(torch.randn(8, 128, dtype=torch.float16, device="cuda"),
                     torch.randn(8, 128, dtype=torch.float16, device="cuda"), layer)
        lengths.append(c.valid_length)
    assert lengths == list(range(1, 13)) + [12] * 8
    c.reset()
    assert c.valid_length == 0 and c.write_count == 0


def test_memory_usage_and_repr(Q):
    c = _cache(Q, num_layers=36, window_size=4092)
    assert c.memory_usage_bytes() == 36 * 4096 * 8 * 128 * 2 * 2
    assert c.k_cache.numel() * 2 * 2 == c.memory_usage_bytes()
    r = repr(c)
    assert "QExtractKVCache" in r and "sink=4" in r


def test_reference_trace_bit_exact(Q):
    d = load_golden("ring")
    ks, vs = dev_tensor(d["trace_k_in"]), dev_tensor(d["trace_v_in"])
    c = Q.QExtractKVCache(2, 2, 8, sink_size=4, window_size=8)
    for t in range(30):
        for layer in range(2):
            c.append(ks[t, layer].contiguous(), vs[t, layer].contiguous(), layer)
        if t + 1 in (3, 4, 12, 13, 29, 30):
            for layer in range(2):
                k_out, v_out = c.get_kv(layer)
                np.testing.assert_array_equal(to_np(k_out), d[f"trace_t{t + 1}_l{layer}_k"])
                np.testing.assert_array_equal(to_np(v_out), d[f"trace_t{t + 1}_l{layer}_v"])


@pytest.mark.parametrize("S,W", [(4, 8), (2, 4), (4, 4092), (0, 5), (1, 1)])
def test_slot_indices_bit_exact(Q, S, W):
    from qextract_infer_b200._C import ring_slot_indices
    d = load_golden("ring")
    for cnt in d[f"counts_S{S}_W{W}"]:
        got = to_np(ring_slot_indices(int(cnt), S, W, "cuda"))
        np.testing.assert_array_equal(got, d[f"idx_S{S}_W{W}_c{int(cnt)}"])
    o = RingIndexOracle(S, W)
    for cnt in list(range(0, 3 * (S + W) + 3)) + [32768, 32768 + 64]:
        np.testing.assert_array_equal(to_np(ring_slot_indices(cnt, S, W, "cuda")), o.indices(cnt))


@pytest.mark.parametrize("chunks,S,W,B", [
    ([5, 1, 9, 2, 13, 1, 1], 4, 6, 1),
    ([3, 3, 3], 0, 4, 2),
    ([40, 1, 17], 4, 8, 3),
    ([1] * 12 + [30], 2, 5, 1),
])
def test_chunked_append_equals_sequential_oracle(Q, chunks, S, W, B):
    L, H, D = 3, 2, 16
    rng = np.random.default_rng(sum(chunks) + S + W + B)
    c = Q.QExtractKVCache(L, H, D, sink_size=S, window_size=W, batch=B)
    o = RingCacheOracle(L, H, D, sink_size=S, window_size=W, batch=B)
    for T in chunks:
        k = rng.standard_normal((B, T, L, H, D)).astype(np.float16)
        v = rng.standard_normal((B, T, L, H, D)).astype(np.float16)
        for layer in range(L):
            kl, vl = np.ascontiguousarray(k[:, :, layer]), np.ascontiguousarray(v[:, :, layer])
            c.append(dev_tensor(kl), dev_tensor(vl), layer)
            o.append(kl, vl, layer)
        assert c.write_count == o.count and c.valid_length == o.valid_length
        n = c.valid_length
        # the valid region [0, valid) is bit-identical to sequential appends
        np.testing.assert_array_equal(to_np(c.k_cache)[:, :, :n], o.k[:, :, :n])
        np.testing.assert_array_equal(to_np(c.v_cache)[:, :, :n], o.v[:, :, :n])
        if B == 1:
            for layer in range(L):
                kk, vv = c.get_kv(layer)
                ok, ov = o.get_kv(layer)
                np.testing.assert_array_equal(to_np(kk), ok)
                np.testing.assert_array_equal(to_np(vv), ov)


def test_qwen3_8b_stream_geometry(Q):
    """36 layers x 8 KV heads x 128, 4 sink + 4092 window: 16 prefill chunks of
    2048 tokens then 64 decode appends.  Token values encode (token, layer) so
    the surviving slot contents are checked bit-exactly from the oracle's
    positions without materialising the whole stream on the host."""
    L, H, D, S, W = 36, 8, 128, 4, 4092
    c = Q.QExtractKVCache(L, H, D, sink_size=S, window_size=W)
    o = RingIndexOracle(S, W)

    def chunk(t0, T, layer):
        tok = torch.arange(t0, t0 + T, device="cuda", dtype=torch.float32)
        base = (tok % 2039) + layer * 0.0  # exact in fp16 (< 2048)
        k = base[:, None, None].expand(T, H, D).to(torch.float16).contiguous()
        v = (base[:, None, None] * -1.0 - layer).expand(T, H, D).to(torch.float16).contiguous()
        return k, v

    t = 0
    for step in range(16 + 64):
        T = 2048 if step < 16 else 1
        for layer in range(L):
            k, v = chunk(t, T, layer)
            c.append(k if T > 1 else k[0], v if T > 1 else v[0], layer)
        t += T
        if step in (0, 1, 2, 15, 16, 79):
            np.testing.assert_array_equal(to_np(c._backend.slot_indices()), o.indices(t))
            pos = o.positions(t)
            for layer in (0, 17, 35):
                kk, vv = c.get_kv(layer)
                want_k = (pos % 2039).astype(np.float16)
                want_v = (-(pos % 2039) - layer).astype(np.float16)
                np.testing.assert_array_equal(to_np(kk[:, 0, 0]), want_k)
                np.testing.assert_array_equal(to_np(vv[:, 3, 77]), want_v)
    assert c.write_count == 16 * 2048 + 64
    assert c.valid_length == 4096
