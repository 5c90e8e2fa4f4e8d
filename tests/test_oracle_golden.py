"""Pin the CPU oracle to golden vectors produced by the reference's own code.

CPU-only.  Fixtures come from ``tests/golden/make_golden.py``.
"""

import numpy as np
import pytest

from oracle import (RingCacheOracle, RingIndexOracle, dequantize_gptq, pack_int4_rows,
                    pack_qzeros, rmsnorm_ref, simulate_gptq_quantize, swiglu_ref,
                    unpack_int4_rows, unpack_qzeros, w4a16_gemv_ref, w4a16_lora_gemv_ref)
from oracle import cbind
from tests._util import assert_f16_match, f16_ulp_diff, load_golden

GPTQ_CASES = ["k256_n128", "k1024_n512_r32", "k2560_n256_r16", "k1024_n256_r64"]


@pytest.mark.parametrize("case", GPTQ_CASES)
def test_gptq_gemv_matches_reference(case):
    d = load_golden(f"gptq_{case}")
    qw, s, z, x = d["qweight"], d["scales"], d["zeros"], d["x"]
    if "w_dequant" in d:
        # dequantisation is bit-exact against dequantize_gptq_ref
        np.testing.assert_array_equal(dequantize_gptq(qw, s, z).view(np.uint16),
                                      d["w_dequant"].view(np.uint16))
        np.testing.assert_array_equal(cbind.c_dequantize(qw, s, z).view(np.uint16),
                                      d["w_dequant"].view(np.uint16))
    yf = w4a16_gemv_ref(x, qw, s, z, return_f32=True)
    np.testing.assert_allclose(yf, d["y_base_f32"], rtol=1e-5, atol=1e-5)
    assert_f16_match(w4a16_gemv_ref(x, qw, s, z), d["y_base"])
    yc = cbind.c_w4a16_lora_gemv(x, qw, s, z, return_f32=True)
    np.testing.assert_allclose(yc, d["y_base_f32"], rtol=1e-5, atol=1e-5)
    if "lora_A" in d:
        A, B, alpha = d["lora_A"], d["lora_B"], float(d["alpha"])
        yl = w4a16_lora_gemv_ref(x, qw, s, z, A, B, lora_alpha=alpha, return_f32=True)
        np.testing.assert_allclose(yl, d["y_lora_f32"], rtol=1e-5, atol=1e-5)
        assert_f16_match(yl.astype(np.float16), d["y_lora"])
        yc = cbind.c_w4a16_lora_gemv(x, qw, s, z, A, B, lora_alpha=alpha)
        assert_f16_match(yc, d["y_lora"])


def test_simulate_quantize_matches_reference():
    d = load_golden("gptq_k256_n128")
    qw, s, z = simulate_gptq_quantize(d["w"], 128)
    np.testing.assert_array_equal(qw, d["qweight"])
    np.testing.assert_array_equal(s.view(np.uint16), d["scales"].view(np.uint16))
    np.testing.assert_array_equal(z.view(np.uint16), d["zeros"].view(np.uint16))


def test_packed_qzeros_matches_reference():
    d = load_golden("gptq_packed_zeros")
    N = d["qweight"].shape[1]
    np.testing.assert_array_equal(unpack_qzeros(d["qzeros"], N), d["zeros_unpacked"])
    np.testing.assert_array_equal(pack_qzeros(d["zeros_unpacked"].astype(np.uint8)), d["qzeros"])
    args = (d["x"], d["qweight"], d["scales"], d["qzeros"], d["lora_A"], d["lora_B"])
    yl = w4a16_lora_gemv_ref(*args, lora_alpha=float(d["alpha"]), return_f32=True)
    np.testing.assert_allclose(yl, d["y_lora_f32"], rtol=1e-5, atol=1e-5)
    yc = cbind.c_w4a16_lora_gemv(*args, lora_alpha=float(d["alpha"]))
    assert_f16_match(yc, d["y_lora"])
    for off in (0, 1):  # the C dequantisation (large checks) equals the numpy one, bit for bit
        np.testing.assert_array_equal(
            cbind.c_dequantize(d["qweight"], d["scales"], d["qzeros"], zero_offset=off).view(np.uint16),
            dequantize_gptq(d["qweight"], d["scales"], d["qzeros"], zero_offset=off).view(np.uint16))
    # GPTQ-v1 storage (+1): identical to unpacked zeros + 1
    np.testing.assert_array_equal(unpack_qzeros(d["qzeros"], N, zero_offset=1),
                                  d["zeros_unpacked"] + 1)


def test_int4_pack_roundtrip():
    rng = np.random.default_rng(0)
    qw = rng.integers(0, 2 ** 32, size=(40, 24), dtype=np.uint64).astype(np.uint32).view(np.int32)
    q = unpack_int4_rows(qw)
    assert q.shape == (320, 24) and q.max() <= 15
    np.testing.assert_array_equal(pack_int4_rows(q), qw)
    # nibble i of word (pr, n) is row 8*pr + i (little-endian nibble order)
    w = np.uint32(qw.view(np.uint32)[3, 5])
    for i in range(8):
        assert q[3 * 8 + i, 5] == (w >> np.uint32(4 * i)) & 0xF


def test_c_half_conversions_match_ieee():
    L = cbind.lib()
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = allh.view(np.float16).astype(np.float32)
    got = np.array([L.qxo_h2f(int(h)) for h in allh[::7]], dtype=np.float32)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(ref[::7]))
    fin = ~np.isnan(ref[::7])
    np.testing.assert_array_equal(got[fin], ref[::7][fin])
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.standard_normal(3000) * s for s in (1e-7, 1e-5, 1e-2, 1, 300, 7e4)])
    vals = vals.astype(np.float32)
    ties = (np.arange(0, 4096, dtype=np.float32) + 0.5) * np.float32(2.0 ** -24)  # subnormal ties
    for v in np.concatenate([vals, ties, np.float32([65504, 65519.9, 65520, -65520, 0.0, -0.0])]):
        with np.errstate(over="ignore"):
            want = np.float32(v).astype(np.float16).view(np.uint16)
        assert L.qxo_f2h(float(v)) == want, v


def test_rmsnorm_matches_reference():
    d = load_golden("rmsnorm")
    for i in range(5):
        y = rmsnorm_ref(d[f"x{i}"], d[f"w{i}"], float(d[f"eps{i}"]))
        assert f16_ulp_diff(y, d[f"y{i}"]).max() <= 1, i


def test_swiglu_matches_reference():
    d = load_golden("swiglu")
    for i in range(6):
        y = swiglu_ref(d[f"g{i}"], d[f"u{i}"])
        assert f16_ulp_diff(y, d[f"y{i}"]).max() <= 1, i


def test_ring_indices_match_reference():
    d = load_golden("ring")
    for (S, W) in [(4, 8), (2, 4), (4, 4092), (0, 5), (1, 1)]:
        o = RingIndexOracle(S, W)
        counts = d[f"counts_S{S}_W{W}"]
        for cnt, wp, vl in zip(counts, d[f"writepos_S{S}_W{W}"], d[f"valid_S{S}_W{W}"]):
            cnt = int(cnt)
            assert o.write_pos(cnt) == wp
            assert o.valid_length(cnt) == vl
            ref_idx = d[f"idx_S{S}_W{W}_c{cnt}"]
            np.testing.assert_array_equal(o.indices(cnt), ref_idx)
            np.testing.assert_array_equal(cbind.c_ring_indices(cnt, S, W), ref_idx)


def test_ring_known_answers():
    d = load_golden("ring")
    np.testing.assert_array_equal(d["wrap_k00"], np.float16([0, 1, 6, 7, 8, 9]))
    c = RingCacheOracle(2, 8, 128, sink_size=2, window_size=4)
    for step in range(10):
        k = np.full((8, 128), step, dtype=np.float16)
        for layer in range(2):
            c.append(k, np.zeros_like(k), layer)
    k_out, _ = c.get_kv(0)
    np.testing.assert_array_equal(k_out[:, 0, 0], d["wrap_k00"])
    assert c.valid_length == int(d["wrap_valid"]) == 6
    c36 = RingCacheOracle(36, 8, 128, 4, 4092)
    assert c36.memory_usage_bytes() == int(d["mem_36x8x128_4_4092"]) == 36 * 4096 * 8 * 128 * 2 * 2


def test_ring_trace_matches_reference():
    d = load_golden("ring")
    ks, vs = d["trace_k_in"], d["trace_v_in"]
    c = RingCacheOracle(2, 2, 8, sink_size=4, window_size=8)
    for t in range(30):
        for layer in range(2):
            c.append(ks[t, layer], vs[t, layer], layer)
        if t + 1 in (3, 4, 12, 13, 29, 30):
            for layer in range(2):
                k_out, v_out = c.get_kv(layer)
                np.testing.assert_array_equal(k_out, d[f"trace_t{t + 1}_l{layer}_k"])
                np.testing.assert_array_equal(v_out, d[f"trace_t{t + 1}_l{layer}_v"])


def test_ring_chunk_append_equals_token_by_token():
    rng = np.random.default_rng(5)
    a = RingCacheOracle(3, 2, 4, sink_size=4, window_size=6)
    b = RingCacheOracle(3, 2, 4, sink_size=4, window_size=6)
    chunks = [5, 1, 9, 2, 13, 1]
    for T in chunks:
        k = rng.standard_normal((T, 3, 2, 4)).astype(np.float16)
        v = rng.standard_normal((T, 3, 2, 4)).astype(np.float16)
        for layer in range(3):
            a.append(k[:, layer], v[:, layer], layer)
        for t in range(T):
            for layer in range(3):
                b.append(k[t, layer], v[t, layer], layer)
    np.testing.assert_array_equal(a.k, b.k)
    np.testing.assert_array_equal(a.v, b.v)
    assert a.count == b.count == sum(chunks)


@pytest.mark.parametrize("case", GPTQ_CASES)
def test_torch_restatement_of_reference_cpu_path(case):
    """oracle/torch_ref.py (the timed CPU baseline) reproduces the reference's
    own dequantisation bit for bit and its outputs to 1 fp16 ulp."""
    import torch
    from oracle.torch_ref import dequantize_rows, w4a16_lora_gemv_cpu
    d = load_golden(f"gptq_{case}")
    qw, s, z, x = (torch.from_numpy(d[k]) for k in ("qweight", "scales", "zeros", "x"))
    if "w_dequant" in d:
        w = dequantize_rows(qw, s, z, qw.shape[0] * 8)
        np.testing.assert_array_equal(w.numpy().view(np.uint16), d["w_dequant"].view(np.uint16))
    assert_f16_match(w4a16_lora_gemv_cpu(x, qw, s, z).numpy(), d["y_base"])
    if "lora_A" in d:
        A, B = torch.from_numpy(d["lora_A"]), torch.from_numpy(d["lora_B"])
        y = w4a16_lora_gemv_cpu(x, qw, s, z, A, B, lora_alpha=float(d["alpha"]))
        assert_f16_match(y.numpy(), d["y_lora"])


def test_torch_restatement_packed_qzeros():
    import torch
    from oracle.torch_ref import unpack_qzeros_fp16, w4a16_lora_gemv_cpu
    d = load_golden("gptq_packed_zeros")
    N = d["qweight"].shape[1]
    zf = unpack_qzeros_fp16(torch.from_numpy(d["qzeros"]), N)
    np.testing.assert_array_equal(zf.numpy().astype(np.float32), d["zeros_unpacked"].astype(np.float32))
    args = [torch.from_numpy(d[k]) for k in ("x", "qweight", "scales", "qzeros", "lora_A", "lora_B")]
    y = w4a16_lora_gemv_cpu(*args, lora_alpha=float(d["alpha"]))
    assert_f16_match(y.numpy(), d["y_lora"])
