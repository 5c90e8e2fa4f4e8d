"""Prefill attention over the ring (``prefill_attention``): a chunk's queries
over the ring's sinks and previous window (read in place) and the chunk's own
keys, causal with the sink + window mask, against the fp32 oracle
(``oracle.prefill_attention_ref``) on small wrapping rings and against the same
rule in torch fp32 on the GPU at the Qwen3-8B geometry.  rtol = atol = 1e-2 on
the fp16 output.  Parity unpinned by the reference (it has no attention)."""

import numpy as np
import pytest
import torch

from oracle import prefill_attention_ref, ring_positions
from tests._util import assert_close

RTOL = ATOL = 1e-2


@pytest.fixture(scope="module")
def C():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _C
    return _C


def _inputs(B, n, hq, hkv, S, W, seed):
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s, dtype=np.float32).astype(np.float16)
    return f(B, n, hq, 128), f(B, n, hkv, 128), f(B, n, hkv, 128), f(B, S + W, hkv, 128), f(B, S + W, hkv, 128)


def test_oracle_matches_direct_loop_cpu():
    """The oracle against a per-query loop over the logical key list."""
    q, kn, vn, kc, vc = _inputs(1, 5, 4, 2, 2, 6, seed=1)
    count, S, W = 11, 2, 6
    ref = prefill_attention_ref(q[0], kn[0], vn[0], kc[0], vc[0], count, S, W)
    slots, cpos = ring_positions(count, S, W)
    for i in range(5):
        p = count + i
        keys, vals = [], []
        for s, kp in zip(slots, cpos):
            if kp < S or kp > p - W:
                keys.append(kc[0, s]); vals.append(vc[0, s])
        for j in range(i + 1):
            kp = count + j
            if kp < S or kp > p - W:
                keys.append(kn[0, j]); vals.append(vn[0, j])
        K = np.stack(keys).astype(np.float32)
        V = np.stack(vals).astype(np.float32)
        for h in range(4):
            sc = K[:, h // 2] @ q[0, i, h].astype(np.float32) / np.sqrt(128)
            w = np.exp(sc - sc.max()); w /= w.sum()
            np.testing.assert_allclose(ref[i, h].astype(np.float32), (w @ V[:, h // 2]).astype(np.float16),
                                       rtol=2e-3, atol=2e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("B,n,hq,hkv,S,W,count", [
    (1, 100, 8, 2, 4, 60, 0), (1, 100, 8, 2, 4, 60, 3), (1, 100, 8, 2, 4, 60, 250),
    (2, 70, 4, 4, 0, 64, 129), (1, 130, 32, 8, 4, 252, 1000), (3, 1, 8, 2, 4, 60, 77),
    (1, 64, 16, 4, 1, 5, 33)])
def test_small_rings_against_oracle(C, B, n, hq, hkv, S, W, count):
    q, kn, vn, kc, vc = _inputs(B, n, hq, hkv, S, W, seed=n + count)
    d = lambda a: torch.from_numpy(a).cuda()
    out = C.prefill_attention(d(q), d(kn), d(vn), d(kc), d(vc), count, S, W).cpu().numpy()
    for b in range(B):
        ref = prefill_attention_ref(q[b], kn[b], vn[b], kc[b], vc[b], count, S, W)
        assert_close(out[b], ref, RTOL, ATOL, f"b={b}")


def _torch_ref(q, kn, vn, kc, vc, count, S, W):
    """the oracle's rule in torch fp32 on the GPU (one sequence)"""
    slots, cpos = ring_positions(count, S, W)
    sl = torch.from_numpy(slots).cuda()
    kk = torch.cat([kc[sl], kn]).float()
    vv = torch.cat([vc[sl], vn]).float()
    n = q.size(0)
    kpos = torch.cat([torch.from_numpy(cpos).cuda(), count + torch.arange(n, device="cuda")])
    qpos = count + torch.arange(n, device="cuda")
    vis = (kpos[None] <= qpos[:, None]) & ((kpos[None] < S) | (kpos[None] > qpos[:, None] - W))
    rep = q.size(1) // kn.size(1)
    kf, vf = kk.repeat_interleave(rep, 1), vv.repeat_interleave(rep, 1)
    sc = torch.einsum("nhd,lhd->hnl", q.float(), kf) / np.sqrt(q.size(-1))
    sc = sc.masked_fill(~vis[None], float("-inf")).softmax(-1)
    return torch.einsum("hnl,lhd->nhd", sc, vf).half()


@pytest.mark.gpu
@pytest.mark.parametrize("count", [0, 2048, 6144])
def test_qwen3_8b_chunk(C, count):
    """A 2048-token chunk, 32 / 8 heads, 4 sinks + 4092-slot window, at the
    prompt's first, second and fourth chunk (the ring wraps in the last)."""
    g = torch.Generator(device="cuda").manual_seed(count)
    r = lambda *s: torch.randn(*s, generator=g, device="cuda").half()
    n, S, W = 2048, 4, 4092
    q, kn, vn = r(1, n, 32, 128), r(1, n, 8, 128), r(1, n, 8, 128)
    kc, vc = r(1, S + W, 8, 128), r(1, S + W, 8, 128)
    out = C.prefill_attention(q, kn, vn, kc, vc, count, S, W)
    ref = _torch_ref(q[0], kn[0], vn[0], kc[0], vc[0], count, S, W)
    assert_close(out[0].cpu().numpy(), ref.cpu().numpy(), RTOL, ATOL, f"count={count}")
