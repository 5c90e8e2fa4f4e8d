"""Generate golden fixtures by running the reference's own PyTorch code on CPU.

Run from the repository root, with the QExtract-Infer sources available:

    python tests/golden/make_golden.py /path/to/QExtract_Infer

(or with the path in the environment variable ``QEXTRACT_REF``).  It
imports, unmodified, the reference's
CPU reference functions

* ``tests/test_w4a16_gemv.py``: ``simulate_gptq_quantize`` (:14-65),
  ``dequantize_gptq_ref`` (:68-90) and the fp32 GEMV / LoRA reference math
  of ``test_gemv_accuracy`` (:133-134) and ``test_lora_fused_accuracy`` (:178-186);
* ``tests/test_rmsnorm.py``: ``rmsnorm_pytorch_ref`` (:12-18);
* ``tests/test_swiglu.py``: ``swiglu_pytorch_ref`` (:11-13);
* ``qextract/kv_cache.py``: ``QExtractKVCache`` with ``device="cpu"`` (its
  PyTorch fallback, :63-152),

feeds them seeded inputs, and writes the inputs and outputs as ``.npz``
fixtures next to this script.  The fixtures are small (a few MB in total) so
they travel with the repository; the reference itself is not needed at test
time.
"""

from __future__ import annotations

import contextlib
import io
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    return t.detach().cpu().numpy()


def gen_gptq(ref_tests, out):
    sim = ref_tests.simulate_gptq_quantize
    deq = ref_tests.dequantize_gptq_ref
    cases = [
        # (name, K, N, rank, alpha, seed)
        ("k256_n128", 256, 128, 0, 0.0, 11),
        ("k1024_n512_r32", 1024, 512, 32, 16.0, 12),
        ("k2560_n256_r16", 2560, 256, 16, 16.0, 13),
        ("k1024_n256_r64", 1024, 256, 64, 16.0, 14),
    ]
    for name, K, N, rank, alpha, seed in cases:
        g = torch.Generator().manual_seed(seed)
        w = torch.randn(K, N, generator=g, dtype=torch.float32).to(torch.float16) * 0.1
        q = sim(w, 128)
        wd = deq(q["qweight"], q["scales"], q["zeros"], K, 128)
        x = torch.randn(K, generator=g, dtype=torch.float32).to(torch.float16)
        base = x.float() @ wd.float()
        d = dict(qweight=_np(q["qweight"]), scales=_np(q["scales"]),
                 zeros=_np(q["zeros"]), x=_np(x),
                 y_base_f32=_np(base), y_base=_np(base.half()))
        if K * N <= 256 * 128:  # keep fixtures small: full matrices for the small case only
            d.update(w=_np(w), w_dequant=_np(wd))
        if rank:
            A = (torch.randn(K, rank, generator=g) * 0.01).to(torch.float16)
            B = (torch.randn(rank, N, generator=g) * 0.01).to(torch.float16)
            lora = (x.float() @ A.float()) @ B.float()
            y = base + (alpha / rank) * lora
            d.update(lora_A=_np(A), lora_B=_np(B), alpha=np.float32(alpha),
                     y_lora_f32=_np(y), y_lora=_np(y.half()))
        out[f"gptq_{name}"] = d

    # GPTQ-packed qzeros (BASELINE decode-GEMV value distributions, reduced N):
    # the reference dequantiser takes unpacked zeros, so the nibble rule
    # ``z[g, n] = (qzeros[g, n//8] >> 4*(n%8)) & 0xF`` is applied with plain
    # torch ops before calling it.
    g = torch.Generator().manual_seed(21)
    K, N, rank, alpha = 2560, 256, 16, 32.0
    qweight = torch.randint(0, 2 ** 32, (K // 8, N), generator=g, dtype=torch.int64).to(torch.int32)
    scales = (torch.rand(K // 128, N, generator=g) * 0.015 + 0.005).to(torch.float16)
    zn = torch.randint(0, 16, (K // 128, N), generator=g, dtype=torch.int64)
    qzeros = torch.zeros(K // 128, N // 8, dtype=torch.int64)
    for i in range(8):
        qzeros |= zn[:, i::8] << (4 * i)
    qzeros = qzeros.to(torch.int32)
    x = torch.randn(3, K, generator=g).to(torch.float16)
    A = (torch.randn(K, rank, generator=g) * 0.02).to(torch.float16)
    B = (torch.randn(rank, N, generator=g) * 0.02).to(torch.float16)
    wd = deq(qweight, scales, zn.to(torch.float16), K, 128)
    base = x.float() @ wd.float()
    y = base + (alpha / rank) * ((x.float() @ A.float()) @ B.float())
    out["gptq_packed_zeros"] = dict(qweight=_np(qweight), scales=_np(scales), qzeros=_np(qzeros),
                                    zeros_unpacked=_np(zn.to(torch.int32)), x=_np(x),
                                    lora_A=_np(A), lora_B=_np(B), alpha=np.float32(alpha),
                                    y_lora_f32=_np(y), y_lora=_np(y.half()))


def gen_norms(ref_rms, ref_swi, out):
    g = torch.Generator().manual_seed(31)
    d = {}
    for i, (T, H, eps) in enumerate([(4, 2560, 1e-6), (2, 4096, 1e-6), (3, 4096, 1e-5),
                                     (2, 768, 1e-8), (5, 128, 1e-6)]):
        x = torch.randn(T, H, generator=g).to(torch.float16)
        w = (torch.randn(H, generator=g) * 0.1 + 1.0).to(torch.float16)
        d[f"x{i}"], d[f"w{i}"] = _np(x), _np(w)
        d[f"eps{i}"] = np.float32(eps)
        d[f"y{i}"] = _np(ref_rms(x, w, eps))
    out["rmsnorm"] = d
    d = {}
    for i, (shape, mul) in enumerate([((2, 9728), 1.0), ((2, 12288), 1.0), ((3, 1000), 1.0),
                                      ((2, 1024), 10.0), ((2, 1024), 0.01), ((4096,), 1.0)]):
        ga = (torch.randn(*shape, generator=g) * mul).to(torch.float16)
        up = (torch.randn(*shape, generator=g) * mul).to(torch.float16)
        d[f"g{i}"], d[f"u{i}"] = _np(ga), _np(up)
        d[f"y{i}"] = _np(ref_swi(ga, up))
    out["swiglu"] = d


def gen_ring(KVCache, out):
    quiet = contextlib.redirect_stdout(io.StringIO())
    d = {}
    # Known answer: sink 2, window 4, 10 tokens -> logical K values [0,1,6,7,8,9]
    with quiet:
        c = KVCache(2, 8, 128, sink_size=2, window_size=4, device="cpu")
    for step in range(10):
        k = torch.full((8, 128), float(step), dtype=torch.float16)
        for layer in range(2):
            c.append(k, torch.zeros_like(k), layer)
    kk, _ = c.get_kv(0)
    d["wrap_k00"] = _np(kk[:, 0, 0])
    d["wrap_valid"] = np.int64(c.valid_length)
    # write-slot and logical-order sequences for (sink, window) pairs
    for (S, W) in [(4, 8), (2, 4), (4, 4092), (0, 5), (1, 1)]:
        with quiet:
            c = KVCache(1, 1, 8, sink_size=S, window_size=W, device="cpu")
        counts = sorted(set([0, 1, 2, 3, 4, 5, 7, 8, 9, 11, 12, 13, 17, 25, 40,
                             W, W + 1, S + W - 1, S + W, S + W + 1, 2 * W + S + 3,
                             32768, 32768 + 64]))
        wp, vl = [], []
        for cnt in counts:
            c.write_count = cnt
            wp.append(c._get_write_pos())
            vl.append(c.valid_length)
            d[f"idx_S{S}_W{W}_c{cnt}"] = _np(c._build_indices()).astype(np.int32)
        d[f"counts_S{S}_W{W}"] = np.asarray(counts, dtype=np.int64)
        d[f"writepos_S{S}_W{W}"] = np.asarray(wp, dtype=np.int64)
        d[f"valid_S{S}_W{W}"] = np.asarray(vl, dtype=np.int64)
    # random-data trace through the fallback: L=2, H=2, D=8, sink 4, window 8
    g = torch.Generator().manual_seed(41)
    with quiet:
        c = KVCache(2, 2, 8, sink_size=4, window_size=8, device="cpu")
    ks = torch.randn(30, 2, 2, 8, generator=g).to(torch.float16)
    vs = torch.randn(30, 2, 2, 8, generator=g).to(torch.float16)
    d["trace_k_in"], d["trace_v_in"] = _np(ks), _np(vs)
    for t in range(30):
        for layer in range(2):
            c.append(ks[t, layer], vs[t, layer], layer)
        if t + 1 in (3, 4, 12, 13, 29, 30):
            for layer in range(2):
                k_out, v_out = c.get_kv(layer)
                d[f"trace_t{t + 1}_l{layer}_k"] = _np(k_out)
                d[f"trace_t{t + 1}_l{layer}_v"] = _np(v_out)
    with quiet:
        c = KVCache(36, 8, 128, sink_size=4, window_size=4092, device="meta")
    d["mem_36x8x128_4_4092"] = np.int64(c.memory_usage_bytes())
    out["ring"] = d


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QEXTRACT_REF")
    if not ref:
        sys.exit("usage: make_golden.py /path/to/QExtract_Infer (or set QEXTRACT_REF)")
    sys.path.insert(0, ref)
    sys.path.insert(0, os.path.join(ref, "tests"))
    import test_rmsnorm  # noqa: E402
    import test_swiglu  # noqa: E402
    import test_w4a16_gemv  # noqa: E402
    from qextract.kv_cache import QExtractKVCache  # noqa: E402

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    out = {}
    gen_gptq(test_w4a16_gemv, out)
    gen_norms(test_rmsnorm.rmsnorm_pytorch_ref, test_swiglu.swiglu_pytorch_ref, out)
    gen_ring(QExtractKVCache, out)
    for name, d in out.items():
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **d)
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
