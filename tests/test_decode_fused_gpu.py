"""Fused decode-step kernels against the unfused operator sequence they
replace: residual add + RMSNorm and packed SwiGLU bit-exact; the GEMV with the
residual add + RMSNorm prologue against add + norm + GEMV; q/k head norm +
RoPE + ring append against the head-norm kernel followed by the fp32 torch
rotation (within one fp16 ulp: the two sum-of-squares reductions run in
different orders)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _C
    return _C


def _g(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


@pytest.mark.parametrize("rows,H", [(1, 4096), (3, 2560), (32, 4096), (2, 512), (5, 8192), (4, 200)])
def test_add_rmsnorm_bit_exact(C, rows, H):
    x = torch.randn(rows, H, generator=_g(rows + H), device="cuda").half()
    d = torch.randn(rows, H, generator=_g(rows * H), device="cuda").half()
    w = (1 + 0.1 * torch.randn(H, generator=_g(7), device="cuda")).half()
    x_ref = (x.float() + d.float()).half()  # torch's fp16 add
    y_ref = C.fused_rmsnorm(x_ref, w, 1e-6)
    xx = x.clone()
    y = C.add_rmsnorm(xx, d, w, 1e-6)
    assert torch.equal(xx.view(torch.int16), x_ref.view(torch.int16))
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))


@pytest.mark.parametrize("rows,inter", [(1, 12288), (32, 3072), (3, 8), (7, 1536)])
def test_swiglu_packed_bit_exact(C, rows, inter):
    gu = torch.randn(rows, 2 * inter, generator=_g(rows + inter), device="cuda").half()
    ref = C.fused_swiglu(gu[:, :inter].contiguous(), gu[:, inter:].contiguous())
    out = C.swiglu_packed(gu)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def _rope_ref(x, cos, sin):
    xf = x.float()
    half = x.size(-1) // 2
    rot = torch.cat([-xf[..., half:], xf[..., :half]], dim=-1)
    return (xf * cos + rot * sin).half()


@pytest.mark.parametrize("B,hq,hkv,D,pos", [(1, 32, 8, 128, 5), (32, 4, 1, 128, 8191), (3, 8, 2, 64, 2),
                                            (2, 4, 2, 256, 4100)])
def test_qk_norm_rope_append(C, B, hq, hkv, D, pos):
    sink, window = 4, 60
    qkv = torch.randn(B, (hq + 2 * hkv) * D, generator=_g(B + hq + D), device="cuda").half()
    qn = (1 + 0.1 * torch.randn(D, generator=_g(1), device="cuda")).half()
    kn = (1 + 0.1 * torch.randn(D, generator=_g(2), device="cuda")).half()
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))
    ang = pos * inv
    cos, sin = torch.cat([ang.cos(), ang.cos()]), torch.cat([ang.sin(), ang.sin()])
    kc = torch.zeros(B, sink + window, hkv, D, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    q = C.qk_norm_rope_append(qkv, hq, hkv, qn, kn, 1e-6, cos, sin, kc, vc, sink, window, pos)
    qp, kp, vp = qkv.split([hq * D, hkv * D, hkv * D], dim=-1)
    q_ref = _rope_ref(C.fused_rmsnorm(qp.reshape(B * hq, D).contiguous(), qn, 1e-6).view(B, hq, D), cos, sin)
    k_ref = _rope_ref(C.fused_rmsnorm(kp.reshape(B * hkv, D).contiguous(), kn, 1e-6).view(B, hkv, D), cos, sin)
    slot = pos if pos < sink else sink + (pos - sink) % window
    torch.testing.assert_close(q.float(), q_ref.float(), rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(kc[:, slot].float(), k_ref.float(), rtol=2e-3, atol=2e-3)
    assert torch.equal(vc[:, slot], vp.reshape(B, hkv, D))
    others = torch.ones(sink + window, dtype=torch.bool)
    others[slot] = False
    assert not kc[:, others].any() and not vc[:, others].any()


@pytest.mark.parametrize("B,pos", [(1, 8191), (1, 100), (1, 2), (4, 4095), (32, 5000)])
def test_attention_after_append_reads_the_appended_slot(C, B, pos):
    """Decode attention launched early behind qk_norm_rope_append
    (``after_append``: its first K/V tiles load while the append runs) equals
    the attention launched after the append completed, bit for bit, and the
    oracle; the appended slot held different (stale) values before."""
    import numpy as np
    from oracle import RingIndexOracle, gqa_decode_attention_ref
    from tests._util import assert_close
    hq, hkv, D, sink, window = 32, 8, 128, 4, 4092
    g = _g(pos + B)
    kc = torch.randn(B, sink + window, hkv, D, generator=g, device="cuda").half()
    vc = torch.randn(B, sink + window, hkv, D, generator=g, device="cuda").half()
    qkv = torch.randn(B, (hq + 2 * hkv) * D, generator=g, device="cuda").half()
    qn = (1 + 0.1 * torch.randn(D, generator=g, device="cuda")).half()
    kn = (1 + 0.1 * torch.randn(D, generator=g, device="cuda")).half()
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))
    ang = pos * inv
    cos, sin = torch.cat([ang.cos(), ang.cos()]), torch.cat([ang.sin(), ang.sin()])
    outs = []
    for early in (True, False):
        k2, v2 = kc.clone(), vc.clone()
        torch.cuda.synchronize()
        q = C.qk_norm_rope_append(qkv, hq, hkv, qn, kn, 1e-6, cos, sin, k2, v2, sink, window, pos)
        outs.append(C.decode_attention(q, k2, v2, pos + 1, sink, window, after_append=early))
        torch.cuda.synchronize()
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    idx = RingIndexOracle(sink, window).indices(pos + 1)
    qn_, kk, vv = q.cpu().numpy(), k2.cpu().numpy(), v2.cpu().numpy()
    for b in range(B):
        ref = gqa_decode_attention_ref(qn_[b], kk[b][idx], vv[b][idx], None)
        assert_close(outs[0][b].cpu().numpy(), ref, 1e-2, 1e-2, f"b={b}")


@pytest.mark.parametrize("B,hq,hkv,pos", [(1, 32, 8, 8191), (1, 32, 8, 100), (1, 32, 8, 2), (4, 32, 8, 4095),
                                          (32, 32, 8, 5000), (2, 16, 2, 4096), (1, 8, 8, 3)])
def test_attention_qkv_equals_append_then_attention(C, B, hq, hkv, pos):
    """decode_attention_qkv (head norm + RoPE + ring append + attention in one
    kernel) against qk_norm_rope_append followed by decode_attention: the
    output and the appended ring slot bit for bit, the other slots untouched."""
    D, sink, window = 128, 4, 4092
    g = _g(pos * 7 + B)
    kc = torch.randn(B, sink + window, hkv, D, generator=g, device="cuda").half()
    vc = torch.randn(B, sink + window, hkv, D, generator=g, device="cuda").half()
    qkv = torch.randn(B, (hq + 2 * hkv) * D, generator=g, device="cuda").half()
    qn = (1 + 0.1 * torch.randn(D, generator=g, device="cuda")).half()
    kn = (1 + 0.1 * torch.randn(D, generator=g, device="cuda")).half()
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))
    ang = pos * inv
    cos, sin = torch.cat([ang.cos(), ang.cos()]), torch.cat([ang.sin(), ang.sin()])
    k1, v1 = kc.clone(), vc.clone()
    q = C.qk_norm_rope_append(qkv, hq, hkv, qn, kn, 1e-6, cos, sin, k1, v1, sink, window, pos)
    ref = C.decode_attention(q, k1, v1, pos + 1, sink, window)
    k2, v2 = kc.clone(), vc.clone()
    for _ in range(2):  # twice: the second call rewrites the same slot with the same values
        out = C.decode_attention_qkv(qkv, hq, hkv, qn, kn, 1e-6, cos, sin, k2, v2, sink, window, pos)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        assert torch.equal(k2.view(torch.int16), k1.view(torch.int16))
        assert torch.equal(v2.view(torch.int16), v1.view(torch.int16))


def _quant_linear(K, N, r, seed):
    g = _g(seed)
    qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device="cuda", dtype=torch.int32)
    sc = (torch.rand(K // 128, N, generator=g, device="cuda") * 0.015 + 0.005).half()
    qz = torch.full((K // 128, N // 8), 0x88888888 - 2 ** 32, dtype=torch.int32, device="cuda")
    A = (torch.randn(K, r, generator=g, device="cuda") * 0.02).half()
    B = (torch.randn(r, N, generator=g, device="cuda") * 0.02).half()
    return qw, sc, qz, A, B


@pytest.mark.parametrize("M,K,N,r,swiglu", [(1, 4096, 6144, 48, False), (1, 4096, 24576, 32, True),
                                             (4, 2560, 9728, 16, False), (8, 4096, 4096, 16, True),
                                             (3, 1024, 512, 0, False)])
def test_gemv_addnorm_matches_add_rmsnorm_then_gemv(C, M, K, N, r, swiglu):
    """The GEMV with the residual add + RMSNorm prologue against qx_add_rmsnorm
    followed by the GEMV (the new residual bit-exact; the output within the
    GEMV tolerance, rtol = atol = 1e-2: the two sums of squares run in
    different orders), on two calls in a row with the residual buffers
    swapped, as the decode step alternates them."""
    qw, sc, qz, A, B = _quant_linear(K, N, max(r, 8), seed=M + K + N)
    if r == 0:
        A = B = None
    w = (1 + 0.1 * torch.randn(K, generator=_g(3), device="cuda")).half()
    res = torch.randn(M, K, generator=_g(4), device="cuda").half()
    out_buf = torch.full_like(res, float("nan"))
    for call in range(2):
        d = torch.randn(M, K, generator=_g(10 + call), device="cuda").half()
        x_ref = res.clone()
        h = C.add_rmsnorm(x_ref, d, w, 1e-6)
        scale = 2.0 if r else 0.0
        if swiglu:
            y_ref = C._w4a16_swiglu(h, qw, sc, qz, A, B, 128, scale, 0)
        else:
            y_ref = C._w4a16(h, qw, sc, qz, A, B, 128, scale, 0)
        y = C._w4a16_addnorm(res, d, w, 1e-6, out_buf, qw, sc, qz, A, B, 128, scale, 0, swiglu)
        torch.cuda.synchronize()
        assert torch.equal(out_buf.view(torch.int16), x_ref.view(torch.int16)), f"call {call}: new residual"
        assert y.shape == y_ref.shape
        err = (y.float() - y_ref.float()).abs()
        bound = 1e-2 + 1e-2 * y_ref.float().abs()
        assert bool((err <= bound).all()), f"call {call}: max err {err.max().item()}"
        res, out_buf = out_buf, res  # the residual alternates between the two buffers


def test_gemv_addnorm_rejects_aliased_residual(C):
    from qextract_infer_b200 import _lib
    qw, sc, qz, A, B = _quant_linear(512, 256, 16, seed=1)
    w = torch.ones(512, dtype=torch.float16, device="cuda")
    res = torch.randn(2, 512, device="cuda").half()
    with pytest.raises(_lib.QXError, match="overlap"):
        C._w4a16_addnorm(res, res.clone(), w, 1e-6, res, qw, sc, qz, A, B, 128, 2.0, 0)
    with pytest.raises(_lib.QXError, match="rows"):
        big = torch.randn(9, 512, device="cuda").half()
        C._w4a16_addnorm(big, big.clone(), w, 1e-6, torch.empty_like(big), qw, sc, qz, A, B, 128, 2.0, 0)
