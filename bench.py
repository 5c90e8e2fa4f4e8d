"""Benchmark of the decode W4A16-LoRA GEMV (Qwen3-4B gate_proj shape).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one W4A16-LoRA GEMV call: x [1, 2560] fp16 times a GPTQ int4
weight [2560, 9728] (group 128, packed qzeros) plus a rank-16 LoRA
(alpha / r = 2), output [1, 9728] fp16.  Algorithmic bytes per call:
qweight 12,451,840 + scales 389,120 + qzeros 97,280 + A 81,920 + B 311,296 +
x 5,120 + y 19,456 = 13,356,032 B.

value  : device throughput in GB/s (algorithmic bytes / CUDA-event time) over
         K back-to-back calls replayed from a CUDA graph; each call reads a
         different weight set from a rotation whose total size exceeds 2x L2,
         so every call streams its weights from HBM.  Summed over ranks for
         N > 1 (independent replicas, weak scaling), time = max over ranks.
e2e    : the same metric through the reference-facing C-ABI host entry point
         (qx_w4a16_lora_gemv_host, as a C / cgo / ctypes plugin calls it), with
         pinned host x and y every step: the GEMV reads x_host over the bus and
         writes y into y_host (M*K*2 bytes in, M*N*2 out per step), event-timed
         around the calls.
roofline, cpu_baseline, clocks, gpu_launches: see the keys in the JSON line.

Under torchrun every rank runs its own replica; rank 0 prints one JSON line.
``--impl reference`` times the reference's own PyTorch CPU path (restated op
for op in oracle/torch_ref.py; all host cores) on the same workload; ranks > 0
exit.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M, K, N, RANK, GROUP, ALPHA = 1, 2560, 9728, 16, 128, 32.0
BYTES_PER_CALL = (K // 8 * N * 4 + K // GROUP * N * 2 + K // GROUP * N // 8 * 4 + K * RANK * 2
                  + RANK * N * 2 + M * K * 2 + M * N * 2)
METRIC = "W4A16-LoRA GEMV µs & HBM GB/s (% peak); Qwen3-8B decode tok/s @1/2/4/8 B200"
WORKLOAD = ("decode W4A16-LoRA GEMV, Qwen3-4B gate_proj: x[1,2560] fp16 . GPTQ int4 W[2560,9728] "
            "g128 packed qzeros + LoRA r16 alpha/r=2 -> y[1,9728] fp16")
L2_BYTES = 126 * 1024 * 1024


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def gemv_kernel_name():
    """The kernel qx_w4a16_lora_gemv runs for the decode shape (one row: NT = 1,
    128-row groups: KPG = 4, LoRA-down on the helper warp: LW = false)."""
    return "qx::gemv::w4a16_gemv_kernel<1, 4, false>"


def profiled_traffic():
    """dram bytes per launch of the GEMV kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "w4a16_gemv_decode.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in a thread."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if s[3 + i].lower() in ("active", "1")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _reference_cpu_call(threads):
    """One call of the reference's own CPU path (oracle/torch_ref.py: its
    dequantise loop and fp32 matmuls restated op for op) on the decode
    workload, on `threads` host threads."""
    import torch
    from oracle import make_gemv_inputs
    from oracle.torch_ref import unpack_qzeros_fp16, w4a16_lora_gemv_cpu
    torch.set_num_threads(threads)
    d = {k: torch.from_numpy(v) for k, v in make_gemv_inputs(M, K, N, RANK, seed=0).items()}
    zeros = unpack_qzeros_fp16(d["zeros"], N)  # the reference's op takes fp16 zero points
    return lambda: w4a16_lora_gemv_cpu(d["x"], d["qweight"], d["scales"], zeros, d["lora_A"],  # noqa
                                       d["lora_B"], GROUP, ALPHA)


def cpu_gemv_baseline(seconds: float = 15.0, max_calls: int = 200, nthreads: int = 0):
    """The reference's CPU path (its PyTorch dequantise loop + fp32 GEMV +
    LoRA, restated in oracle/torch_ref.py) on all host cores, on the full
    decode workload: a bounded sample of calls."""
    threads = nthreads or os.cpu_count() or 1
    call = _reference_cpu_call(threads)
    call()
    n, t0 = 0, time.perf_counter()
    while n < max_calls and (time.perf_counter() - t0) < seconds:
        call()
        n += 1
    dt = time.perf_counter() - t0
    return {"value": BYTES_PER_CALL * n / dt / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "port", "us_per_call": dt / n * 1e6,
            "sample": f"{n} full decode-GEMV calls (K=2560, N=9728, r=16) in {dt:.1f} s: the reference's "
                      f"PyTorch CPU path (tests/test_w4a16_gemv.py dequantize_gptq_ref loop + fp32 "
                      f"matmuls) restated op for op in oracle/torch_ref.py, torch on {threads} threads"}


def run_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    call = _reference_cpu_call(threads)
    for _ in range(max(1, min(args.warmup, 3))):
        call()
    # each step is one full call; the timed steps stop after ~60 s of CPU work
    steps, t0 = 0, time.perf_counter()
    while steps < max(1, args.steps) and (steps == 0 or time.perf_counter() - t0 < 60.0):
        call()
        steps += 1
    dt = time.perf_counter() - t0
    gbs = BYTES_PER_CALL * steps / dt / 1e9
    line = {"metric": METRIC, "value": gbs, "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup,
            "ms_per_step": dt / steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16 activations, int4 weights, fp32 accumulate",
            "data": "synthetic (seeded; BASELINE decode-GEMV distributions)",
            "config": {"workload": WORKLOAD, "M": M, "K": K, "N": N, "rank": RANK, "group": GROUP},
            "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"{steps} full decode-GEMV calls: the reference's PyTorch CPU "
                                       f"path restated op for op (oracle/torch_ref.py), torch on "
                                       f"{threads} threads; timed steps capped at ~60 s"},
            "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def make_weight_sets(torch, device, nsets, seed=0):
    g = torch.Generator(device=device)
    sets = []
    for i in range(nsets):
        g.manual_seed(seed + i)
        qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=g, device=device,
                           dtype=torch.int32)
        sc = (torch.rand(K // GROUP, N, generator=g, device=device) * 0.015 + 0.005).half()
        qz = torch.full((K // GROUP, N // 8), 0x88888888 - 2 ** 32, dtype=torch.int32, device=device)
        A = (torch.randn(K, RANK, generator=g, device=device) * 0.02).half()
        B = (torch.randn(RANK, N, generator=g, device=device) * 0.02).half()
        sets.append((qw, sc, qz, A, B))
    return sets


def run_b200(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
    device = torch.device("cuda", local if world > 1 else torch.cuda.current_device())
    torch.cuda.set_device(device)
    import qextract_infer_b200 as qx
    from qextract_infer_b200 import _C
    if not qx._C_AVAILABLE:
        raise RuntimeError("native library missing")

    nsets = args.nsets or int(np.ceil(2.2 * L2_BYTES / BYTES_PER_CALL))
    sets = make_weight_sets(torch, device, nsets)
    x = torch.randn(M, K, generator=torch.Generator(device=device).manual_seed(123), device=device).half()
    # correctness gate on set 0 against the oracle (rank 0, cheap)
    if rank == 0:
        from oracle import cbind
        qw, sc, qz, A, B = sets[0]
        y = _C.w4a16_lora_gemv(x, qw, sc, qz, A, B, GROUP, ALPHA)
        ref = cbind.c_w4a16_lora_gemv(x.cpu().numpy(), qw.cpu().numpy(), sc.cpu().numpy(),
                                      qz.cpu().numpy(), A.cpu().numpy(), B.cpu().numpy(), GROUP, ALPHA)
        err = np.abs(y.float().cpu().numpy() - ref.astype(np.float32))
        bound = 1e-2 + 1e-2 * np.abs(ref.astype(np.float32))
        if not np.all(err <= bound):
            raise RuntimeError(f"bench correctness gate failed: max err {err.max()}")

    stream = torch.cuda.Stream(device)
    outs = [torch.empty(M, N, dtype=torch.float16, device=device) for _ in range(2)]

    def step(i):
        qw, sc, qz, A, B = sets[i % nsets]
        return _C.w4a16_lora_gemv(x, qw, sc, qz, A, B, GROUP, ALPHA)

    steps, warm = max(1, args.steps), max(3, args.warmup)
    with torch.cuda.stream(stream):
        for i in range(warm):  # eager warm-up (allocates the workspace)
            step(i)
    stream.synchronize()

    def capture(nsteps, offset):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for i in range(nsteps):
                step(offset + i)
        return gr

    g_warm = capture(warm, 0)
    g_timed = capture(steps, warm)
    with torch.cuda.stream(stream):
        for _ in range(2):
            g_warm.replay()
        g_timed.replay()  # the first replay of a graph also uploads it: keep that out of the timing
    stream.synchronize()
    # sustained load so the clock sampler sees the GPU busy, then the timed region
    sampler = ClockSampler(device.index)
    with sampler:
        t_end = time.time() + 1.0
        while time.time() < t_end:
            with torch.cuda.stream(stream):
                g_warm.replay()
            stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):  # replay() launches on the current stream
            ev0.record(stream)
            g_timed.replay()
            ev1.record(stream)
        ev1.synchronize()
        torch.cuda.synchronize(device)
        ms = ev0.elapsed_time(ev1)
        # e2e through the reference-facing C-ABI with host buffers, as a C, cgo
        # or ctypes caller makes it: pinned host x -> device, the GEMV, device
        # y -> pinned host, every step (qx_w4a16_lora_gemv_host)
        from qextract_infer_b200 import _lib
        lib = _lib.load()
        x_host = torch.randn(M, K).half().pin_memory()
        y_host = torch.empty(M, N, dtype=torch.float16).pin_memory()
        x_dev = torch.empty(M, K, dtype=torch.float16, device=device)
        y_dev = torch.empty(M, N, dtype=torch.float16, device=device)
        e_steps = 0 if args.skip_e2e else max(1, min(steps, 2000))
        raw = stream.cuda_stream
        xh, yh, xd, yd = x_host.data_ptr(), y_host.data_ptr(), x_dev.data_ptr(), y_dev.data_ptr()
        cargs = [(qw.data_ptr(), sc.data_ptr(), qz.data_ptr(), 1, 0, A.data_ptr(), B.data_ptr())
                 for qw, sc, qz, A, B in sets]
        scale = float(np.float32(ALPHA) / np.float32(RANK))
        call = lib.qx_w4a16_lora_gemv_host

        def e2e_step(i):  # x_host -> x_dev, GEMV, y_dev -> y_host in one C-ABI call
            rc = call(xh, yh, xd, yd, *cargs[i % nsets], M, K, N, RANK, GROUP, scale, raw)
            if rc:
                _lib.check(rc, "w4a16_lora_gemv_host")

        with torch.cuda.stream(stream):
            for i in range(nsets if e_steps else 0):  # every weight set once: cached launch plans
                e2e_step(i)
            stream.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(e_steps):
                e2e_step(i)
            e1.record(stream)
            e1.synchronize()
        e_ms = e0.elapsed_time(e1) if e_steps else float("nan")
    clocks = sampler.summary()

    if world > 1:
        t = torch.tensor([ms, e_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e_ms = float(t[0]), float(t[1])
    del sets, g_timed, g_warm
    torch.cuda.empty_cache()
    _C.check_device_error("decode GEMV bench")
    # the rest of the metric, measured in the same run: Qwen3-8B decode tok/s
    # tensor-parallel over the ranks, and at one GPU the prefill GEMM
    tp_lines = [] if args.skip_tp else tp_decode_measure(args, world, rank, device)
    gemm_line = prefill_gemm_measure(args, device) if (world == 1 and not args.skip_gemm) else None
    per_call_s = ms / 1e3 / steps
    achieved = BYTES_PER_CALL / per_call_s / 1e9  # one GPU, GB/s
    peak, peak_kind = measured_peaks()
    result = None
    if rank == 0:
        cpu = cpu_gemv_baseline() if (world == 1 and not args.skip_cpu) else None
        result = {
            "metric": METRIC,
            "value": achieved * world,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warm,
            "ms_per_step": ms / steps,
            "us_per_call": per_call_s * 1e6,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp16 activations, int4 weights, fp32 accumulate",
            "data": "synthetic (seeded, on device; BASELINE decode-GEMV value distributions)",
            "config": {"workload": WORKLOAD, "M": M, "K": K, "N": N, "rank": RANK, "group": GROUP,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": f"inputs larger than L2: {nsets} rotating weight sets, "
                             f"{nsets * BYTES_PER_CALL / 1e6:.0f} MB > 2x 126 MB"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "nominal_frac_8tbs": achieved / 8000.0,
                         "traffic": profiled_traffic(),
                         "algorithmic_bytes_per_launch": BYTES_PER_CALL,
                         "kernel": gemv_kernel_name()},
            "e2e": None if not e_steps else {
                    "value": BYTES_PER_CALL * e_steps / (e_ms / 1e3) / 1e9 * world, "unit": "GB/s",
                    "us_per_call": e_ms * 1e3 / e_steps,
                    "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
                    "api": "C-ABI qx_w4a16_lora_gemv_host (ctypes), pinned host buffers: the GEMV "
                           "reads x_host over the bus and writes y into y_host, one launch per step"},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": steps,
            "tp_decode": tp_lines or None,
            "prefill_gemm": gemm_line,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


def _graph_time_us(torch, stream, fn, nsteps, reps=3):
    """Capture fn(i) for i < nsteps into a CUDA graph; return the best of
    `reps` replays in microseconds per step (CUDA events on `stream`)."""
    with torch.cuda.stream(stream):
        for i in range(3):
            fn(i)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(nsteps):
            fn(i)
    g.replay()
    stream.synchronize()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            g.replay()
            e1.record(stream)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e3 / nsteps)
    del g
    return best


def run_kernel_suite(args):
    """Secondary kernels at the RMSNorm/SwiGLU and ring-cache configurations:
    one JSON line per (kernel, shape) with us/call, GB/s and HBM fraction.
    Inputs rotate over buffers totalling > 2x L2 where one call is smaller."""
    import numpy as np
    import torch
    import qextract_infer_b200 as qx
    from qextract_infer_b200 import _C
    dev = torch.device("cuda", torch.cuda.current_device())
    st = torch.cuda.Stream(dev)
    peak, peak_kind = measured_peaks()
    gen = torch.Generator(device=dev).manual_seed(1)
    steps = max(50, min(args.steps, 400))

    def nbuf(nbytes):
        return int(min(64, max(1, np.ceil(2.2 * L2_BYTES / max(nbytes, 1)))))

    def emit(kernel, shape, nbytes, us, extra=None):
        gbs = nbytes / us / 1e3
        d = {"metric": f"{kernel} us & HBM GB/s", "kernel": kernel, "shape": shape,
             "us_per_call": us, "bytes_per_call": int(nbytes), "GB/s": gbs,
             "hbm_frac": gbs / peak, "peak": peak, "peak_kind": peak_kind}
        if extra:
            d.update(extra)
        print(json.dumps(d), flush=True)

    for H in (2560, 4096):
        w = (torch.randn(H, generator=gen, device=dev) * 0.1 + 1).half()
        for T in (1, 8, 64, 4096):
            nb = 2 * T * H * 2 + H * 2
            xs = [torch.randn(T, H, generator=gen, device=dev).half() for _ in range(nbuf(nb))]
            us = _graph_time_us(torch, st, lambda i: _C.fused_rmsnorm(xs[i % len(xs)], w, 1e-6), steps)
            emit("fused_rmsnorm", {"T": T, "H": H}, nb, us)
    for I in (9728, 12288):
        for T in (1, 8, 64, 4096):
            nb = 3 * T * I * 2
            n = nbuf(nb)
            gs = [torch.randn(T, I, generator=gen, device=dev).half() for _ in range(n)]
            ups = [torch.randn(T, I, generator=gen, device=dev).half() for _ in range(n)]
            us = _graph_time_us(torch, st, lambda i: _C.fused_swiglu(gs[i % n], ups[i % n]), steps)
            emit("fused_swiglu", {"T": T, "I": I}, nb, us)
    # ring cache, Qwen3-8B geometry: 36 layers x 8 KV heads x 128, 4 + 4092 slots
    L, Hkv, D, S, W = 36, 8, 128, 4, 4092
    cache = qx.QExtractKVCache(L, Hkv, D, sink_size=S, window_size=W)
    for T in (2048, 1):
        kn = torch.randn(T, Hkv, D, generator=gen, device=dev).half()
        vn = torch.randn(T, Hkv, D, generator=gen, device=dev).half()
        kk, vv = (kn, vn) if T > 1 else (kn[0], vn[0])
        nb = 2 * 2 * T * Hkv * D * 2  # read new K/V + write K/V
        us = _graph_time_us(torch, st, lambda i: cache.append(kk, vv, i % L), min(steps, 2 * L))
        emit("ring_append", {"tokens": T, "kv_heads": Hkv, "head_dim": D, "sink": S, "window": W},
             nb, us, {"per": "layer"})
    # decode attention over a full ring (4096 valid slots) per layer, B = 1 and 32
    for B in (1, 32):
        c2 = qx.QExtractKVCache(L if B == 1 else 2, Hkv, D, sink_size=S, window_size=W, batch=B)
        c2.k_cache.normal_(generator=gen)
        c2.v_cache.normal_(generator=gen)
        c2._backend._write_count = 32768 + 64
        q = torch.randn(B, 32, D, generator=gen, device=dev).half()
        nl = c2.num_layers
        nb = B * (2 * (S + W) * Hkv * D * 2 + 2 * 32 * D * 2)
        us = _graph_time_us(torch, st, lambda i: c2.decode_attention(q, i % nl), min(steps, 4 * nl))
        emit("decode_attention", {"batch": B, "q_heads": 32, "kv_heads": Hkv, "head_dim": D,
                                  "valid_slots": S + W}, nb, us, {"per": "layer"})
        # the decode step's form: q/k head norm + RoPE + ring append + attention in one kernel,
        # straight from the q|k|v projection output
        qkv = torch.randn(B, (32 + 2 * Hkv) * D, generator=gen, device=dev).half()
        qn = (1 + 0.1 * torch.randn(D, generator=gen, device=dev)).half()
        cs, sn = torch.rand(D, generator=gen, device=dev), torch.rand(D, generator=gen, device=dev)
        us = _graph_time_us(torch, st, lambda i: _C.decode_attention_qkv(
            qkv, 32, Hkv, qn, qn, 1e-6, cs, sn, c2.k_cache[i % nl], c2.v_cache[i % nl], S, W, 32768 + 64),
            min(steps, 4 * nl))
        emit("decode_attention_qkv", {"batch": B, "q_heads": 32, "kv_heads": Hkv, "head_dim": D,
                                      "valid_slots": S + W}, nb + B * (32 + 2 * Hkv) * D * 2, us,
             {"per": "layer", "fused": "q/k head norm + RoPE + ring append + attention"})
        del c2
    # prefill attention: a 2048-token chunk at position 6144 (4096 ring slots + the chunk)
    for B in (1, 32):
        n = 2048
        pq = torch.randn(B, n, 32, D, generator=gen, device=dev).half()
        pk = torch.randn(B, n, Hkv, D, generator=gen, device=dev).half()
        pv = torch.randn(B, n, Hkv, D, generator=gen, device=dev).half()
        kc = torch.randn(B, S + W, Hkv, D, generator=gen, device=dev).half()
        vc = torch.randn(B, S + W, Hkv, D, generator=gen, device=dev).half()
        us = _graph_time_us(torch, st, lambda i: _C.prefill_attention(pq, pk, pv, kc, vc, 6144, S, W),
                            10 if B > 1 else 40)
        flops = 4.0 * B * 32 * D * n * ((S + W) + n / 2)
        print(json.dumps({"metric": "prefill_attention us & TFLOP/s", "kernel": "prefill_attention",
                          "shape": {"batch": B, "chunk": n, "q_heads": 32, "kv_heads": Hkv,
                                    "ring_slots": S + W, "position": 6144},
                          "us_per_call": us, "TFLOP/s": flops / us / 1e6, "bound": "mma.sync"}),
              flush=True)
        del pq, pk, pv, kc, vc
    return 0


QWEN3_8B_PREFILL = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
                    ("gate", 4096, 12288), ("up", 4096, 12288), ("down", 12288, 4096)]


def measured_tflops():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 1590.0, 1400.0, "fallback"


def run_prefill_suite(args):
    """Prefill W4A16-LoRA GEMM at M=4096 over the 7 Qwen3-8B projection shapes:
    one JSON line per shape and one for the whole set (prefill_gemm_measure)."""
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    summary = prefill_gemm_measure(args, dev, per_shape=lambda d: print(json.dumps(d), flush=True))
    print(json.dumps(summary), flush=True)
    return 0


def prefill_gemm_measure(args, dev, per_shape=None):
    """Prefill W4A16-LoRA GEMM at M=4096 over the 7 Qwen3-8B projection shapes
    (GPTQ int4 g128, packed qzeros, LoRA r=64, alpha/r=2) through the public
    API (tcgen05 path): per shape us, TFLOP/s and fraction of the measured
    dense bf16 peak (passed to ``per_shape``); returns the whole-set summary."""
    import torch
    from qextract_infer_b200 import _C
    st = torch.cuda.Stream(dev)
    peak, peak_sus, kind = measured_tflops()
    Mr, R, G = 4096, 64, 128
    gen = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(Mr, 12288, generator=gen, device=dev).half()
    total_flop, total_us = 0.0, 0.0
    shapes = {}
    for name, K, N in QWEN3_8B_PREFILL:
        qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=gen, device=dev, dtype=torch.int32)
        sc = (torch.rand(K // G, N, generator=gen, device=dev) * 0.015 + 0.005).half()
        qz = torch.full((K // G, N // 8), 0x88888888 - 2 ** 32, dtype=torch.int32, device=dev)
        A = (torch.randn(K, R, generator=gen, device=dev) * 0.02).half()
        B = (torch.randn(R, N, generator=gen, device=dev) * 0.02).half()
        xk = x[:, :K].contiguous()
        steps = max(5, min(args.steps, 50))
        us = _graph_time_us(torch, st, lambda i: _C.w4a16_lora_gemv(xk, qw, sc, qz, A, B, G, 2.0 * R), steps)
        flop = 2.0 * Mr * K * N + 2.0 * Mr * R * (K + N)
        tf = flop / us / 1e6
        total_flop += flop
        total_us += us
        if per_shape:
            per_shape({"metric": "prefill W4A16-LoRA GEMM TFLOP/s", "shape": name, "M": Mr, "K": K,
                       "N": N, "rank": R, "us_per_call": us, "TFLOP/s": tf, "peak": peak,
                       "tensor_frac": tf / peak, "peak_kind": kind})
        shapes[name] = {"us": us, "TFLOP/s": tf}
        del qw, sc, qz, A, B, xk
    del x
    torch.cuda.empty_cache()
    _C.check_device_error("prefill GEMM bench")
    tf = total_flop / total_us / 1e6
    return {"metric": "prefill W4A16-LoRA GEMM TFLOP/s (7 Qwen3-8B shapes, M=4096, r=64)",
            "value": tf, "unit": "TFLOP/s", "us_total": total_us, "flop_total": total_flop,
            "shapes": shapes,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": tf / peak, "peak_kind": kind,
                         "timing": "CUDA graph of back-to-back calls per shape, best of 3 replays"}}


def run_decode_tp(args):
    """Qwen3-8B decode alone (tp_decode_measure), one JSON line per batch size."""
    import torch
    import torch.distributed as dist
    world, rank, local = dist_setup()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=300))
    dev = torch.device("cuda", local if world > 1 else torch.cuda.current_device())
    torch.cuda.set_device(dev)
    for line in tp_decode_measure(args, world, rank, dev):
        if rank == 0:
            print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def tp_decode_measure(args, world, rank, dev):
    """Qwen3-8B-architecture decode (random init, GPTQ int4 g128 + LoRA r16
    linears, fp16 norms/embeddings/lm_head, ring of 4 sink + 4092 window),
    tensor-parallel over the ranks of the initialised process group (or one
    GPU): an 8192-token prompt prefilled in 2048-token chunks, then 64 greedy
    decode steps replayed from per-step CUDA graphs.  One dict per batch size;
    tok_s = decoded tokens per second over the whole job, time = max over
    ranks.  At more than one rank, also the device time of one NVLink
    all-reduce (+ residual add + RMSNorm) call at the batch's rows."""
    import torch
    import torch.distributed as dist
    from qextract_infer_b200 import _C
    from qextract_infer_b200.tp_decoder import DecoderConfig, TPDecoder

    cfg = DecoderConfig()
    prompt_len, decode_steps, chunk = args.prompt, args.decode, 2048
    batches = [int(b) for b in args.batches.split(",")]
    hbm = measured_peaks()[0]
    lines = []

    def max_over_ranks(v):
        if world > 1:
            t = torch.tensor([v], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            v = float(t[0])
        return v

    for B in batches:
        dec = TPDecoder(cfg, batch=B, device=dev, seed=4)
        prompt = torch.randint(0, cfg.vocab, (B, prompt_len), generator=torch.Generator().manual_seed(4))
        prompt = prompt.to(dev)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t0 = time.time()
        nxt = dec.prefill(prompt, chunk=chunk)
        torch.cuda.synchronize(dev)
        prefill_s = max_over_ranks(time.time() - t0)
        count0 = dec.cache.get_total_written()
        k0, v0 = dec.cache.k.clone(), dec.cache.v.clone()
        tok = torch.empty_like(nxt)
        st = torch.cuda.Stream(dev)

        def restore():
            dec.cache.k.copy_(k0)
            dec.cache.v.copy_(v0)
            dec.cache._write_count = count0
            tok.copy_(nxt)

        with torch.cuda.stream(st):
            restore()
            tok.copy_(dec.decode_step(tok))  # eager step: plans, workspaces, lazy state
            restore()
        st.synchronize()
        graphs, pool = [], torch.cuda.graph_pool_handle()
        for _ in range(decode_steps):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool, stream=st):
                tok.copy_(dec.decode_step(tok))
            graphs.append(g)
        for rep in range(2):  # rep 0 uploads the graphs; rep 1 is timed
            with torch.cuda.stream(st):
                restore()
            st.synchronize()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(st):
                e0.record(st)
                for g in graphs:
                    g.replay()
                e1.record(st)
            e1.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1))
        step_ms = ms / decode_steps
        dec.check_device_error()
        # bytes one decode step reads per rank: int4 weights + scales/qzeros + LoRA, lm_head
        # shard, and the ring (all layers, this rank's KV heads, every sequence)
        wbytes = sum(L[k].weight_bytes() for L in dec.layers for k in ("qkv", "o", "gate_up", "down"))
        wbytes += dec.lm_head.numel() * 2
        kvbytes = 2 * cfg.num_layers * B * (cfg.sink + cfg.window) * dec.hkv * cfg.head_dim * 2
        per_rank_gbs = (wbytes + kvbytes) / (step_ms / 1e3) / 1e9
        ar_us = None
        if dec.ar is not None:  # one NVLink all-reduce + add + RMSNorm call, device time
            part = torch.randn(B, cfg.hidden, device=dev).half()
            xr = torch.randn(B, cfg.hidden, device=dev).half()
            w = torch.ones(cfg.hidden, device=dev).half()
            with torch.cuda.stream(st):
                for _ in range(3):
                    dec.ar.add_rmsnorm(part, xr, w, cfg.rms_eps)
            st.synchronize()
            ga = torch.cuda.CUDAGraph()
            with torch.cuda.graph(ga, stream=st):
                for _ in range(72):
                    dec.ar.add_rmsnorm(part, xr, w, cfg.rms_eps)
            with torch.cuda.stream(st):
                ga.replay()
            st.synchronize()
            dist.barrier()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(st):
                a0.record(st)
                ga.replay()
                a1.record(st)
            a1.synchronize()
            ar_us = max_over_ranks(a0.elapsed_time(a1) * 1e3 / 72)
            del ga
            dec.check_device_error()
        lines.append({
            "metric": "Qwen3-8B decode tok/s", "value": B * decode_steps / (ms / 1e3), "unit": "tok/s",
            "batch": B, "n_gpus": world, "parallelism": f"tp{world}", "steps": decode_steps,
            "ms_per_step": step_ms, "scaling": "strong",
            "config": {"workload": "Qwen3-8B decoder (36 layers, hidden 4096, 32/8 heads, "
                                   "GPTQ int4 g128 + LoRA r16), TP decode",
                       "prompt": prompt_len, "decode_tokens": decode_steps, "prefill_chunk": chunk,
                       "graphs": "one CUDA graph per decode step"},
            "prefill_s": prefill_s, "prefill_tok_s": B * prompt_len / prefill_s,
            "nvlink_allreduce_us": ar_us,
            "roofline": {"bound": "hbm", "achieved": per_rank_gbs, "peak": hbm, "unit": "GB/s",
                         "frac": per_rank_gbs / hbm, "bytes_per_step_per_rank": wbytes + kvbytes}})
        del graphs, g
        dec.close()
        del dec, k0, v0
        torch.cuda.empty_cache()
    return lines


def run_profile_cases(args):
    """One launch of every secondary kernel at a representative size, twice
    (the first pass warms up): the command the committed ncu summaries under
    profiles/ were captured from.  Sizes: RMSNorm 4096 x 4096, SwiGLU
    4096 x 12288, ring append of a 2048-token chunk (8 KV heads x 128), decode
    attention B=32 over a full 4 + 4092 ring, the decode-step kernels at B=32
    (Qwen3-8B, TP 1), the prefill GEMM on the q shape (M=4096, K=N=4096, r=64),
    prefill attention of a 2048-token chunk at position 6144, the gate|up GEMV
    with the SwiGLU epilogue (one row) and the fused q/k norm + RoPE + append +
    attention (one sequence).
    Prints one line per pass; no timing."""
    import torch
    import qextract_infer_b200 as qx
    from qextract_infer_b200 import _C
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(5)
    H, I, D, Hkv, Hq, S, W, B = 4096, 12288, 128, 8, 32, 4, 4092, 32
    G = 128
    x = torch.randn(4096, H, generator=gen, device=dev).half()
    w = (torch.randn(H, generator=gen, device=dev) * 0.1 + 1).half()
    g = torch.randn(4096, I, generator=gen, device=dev).half()
    u = torch.randn(4096, I, generator=gen, device=dev).half()
    cache = qx.QExtractKVCache(2, Hkv, D, sink_size=S, window_size=W)
    kn = torch.randn(2048, Hkv, D, generator=gen, device=dev).half()
    vn = torch.randn(2048, Hkv, D, generator=gen, device=dev).half()
    c2 = qx.QExtractKVCache(1, Hkv, D, sink_size=S, window_size=W, batch=B)
    c2.k_cache.normal_(generator=gen)
    c2.v_cache.normal_(generator=gen)
    c2._backend._write_count = 32768 + 64
    q = torch.randn(B, Hq, D, generator=gen, device=dev).half()
    xr = torch.randn(B, H, generator=gen, device=dev).half()
    dr = torch.randn(B, H, generator=gen, device=dev).half()
    qkv = torch.randn(B, (Hq + 2 * Hkv) * D, generator=gen, device=dev).half()
    qn = (torch.randn(D, generator=gen, device=dev) * 0.1 + 1).half()
    cos = torch.rand(D, generator=gen, device=dev)
    sin = torch.rand(D, generator=gen, device=dev)
    kc = torch.zeros(B, S + W, Hkv, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    gu = torch.randn(B, 2 * I, generator=gen, device=dev).half()
    K = N = 4096
    R = 64
    qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=gen, device=dev, dtype=torch.int32)
    sc = (torch.rand(K // G, N, generator=gen, device=dev) * 0.015 + 0.005).half()
    qz = torch.full((K // G, N // 8), 0x88888888 - 2 ** 32, dtype=torch.int32, device=dev)
    A = (torch.randn(K, R, generator=gen, device=dev) * 0.02).half()
    Bl = (torch.randn(R, N, generator=gen, device=dev) * 0.02).half()
    # prefill attention: a 2048-token chunk at position 6144 (the ring wraps), one sequence
    pq = torch.randn(1, 2048, Hq, D, generator=gen, device=dev).half()
    pk = torch.randn(1, 2048, Hkv, D, generator=gen, device=dev).half()
    pv = torch.randn(1, 2048, Hkv, D, generator=gen, device=dev).half()
    pkc = torch.randn(1, S + W, Hkv, D, generator=gen, device=dev).half()
    pvc = torch.randn(1, S + W, Hkv, D, generator=gen, device=dev).half()
    # gate|up with the SwiGLU epilogue, one row (Qwen3-8B: K 4096, 2 x 12288 columns, r 32)
    gq = torch.randint(-2 ** 31, 2 ** 31 - 1, (H // 8, 2 * I), generator=gen, device=dev, dtype=torch.int32)
    gs = (torch.rand(H // G, 2 * I, generator=gen, device=dev) * 0.015 + 0.005).half()
    gz = torch.full((H // G, 2 * I // 8), 0x88888888 - 2 ** 32, dtype=torch.int32, device=dev)
    gA = (torch.randn(H, 32, generator=gen, device=dev) * 0.02).half()
    gB = (torch.randn(32, 2 * I, generator=gen, device=dev) * 0.02).half()
    x1 = torch.randn(1, H, generator=gen, device=dev).half()
    qkv1 = torch.randn(1, (Hq + 2 * Hkv) * D, generator=gen, device=dev).half()
    kc1 = torch.randn(1, S + W, Hkv, D, generator=gen, device=dev).half()
    vc1 = torch.randn(1, S + W, Hkv, D, generator=gen, device=dev).half()
    for rep in range(2):
        _C.prefill_attention(pq, pk, pv, pkc, pvc, 6144, S, W)
        _C.w4a16_lora_gemv_swiglu(x1, gq, gs, gz, gA, gB, G, 64.0)
        _C.decode_attention_qkv(qkv1, Hq, Hkv, qn, qn, 1e-6, cos, sin, kc1, vc1, S, W, 8191)
        _C.fused_rmsnorm(x, w, 1e-6)
        _C.fused_swiglu(g, u)
        cache.append(kn, vn, 0)
        c2.decode_attention(q, 0)
        _C.add_rmsnorm(xr, dr, w, 1e-6)
        _C.qk_norm_rope_append(qkv, Hq, Hkv, qn, qn, 1e-6, cos, sin, kc, vc, S, W, 100)
        _C.swiglu_packed(gu)
        _C.w4a16_lora_gemv(x, qw, sc, qz, A, Bl, G, 2.0 * R)
        torch.cuda.synchronize(dev)
        print(json.dumps({"profile_cases": "pass", "rep": rep}), flush=True)
    return 0


def run_profile_decode_step(args):
    """One Qwen3-8B decode step at TP 1 inside an NVTX range named "step" (the
    ring pre-filled with 8192 random positions, two eager steps before it): the
    command the committed decode-step launch list was captured from, with
    ``ncu --nvtx --nvtx-include "step/"``.  Batch from ``--batches`` (first value)."""
    import torch
    from qextract_infer_b200.tp_decoder import DecoderConfig, TPDecoder
    B = int(args.batches.split(",")[0])
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = DecoderConfig()
    dec = TPDecoder(cfg, batch=B, device=dev, seed=4)
    dec.cache.k.normal_()
    dec.cache.v.normal_()
    dec.cache._write_count = args.prompt
    tok = torch.randint(0, cfg.vocab, (B,), device=dev)
    for _ in range(2):
        tok = dec.decode_step(tok)
    torch.cuda.synchronize(dev)
    torch.cuda.nvtx.range_push("step")
    tok = dec.decode_step(tok)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    print(json.dumps({"profile_decode_step": "done", "batch": B}), flush=True)
    dec.close()
    return 0


def _trace_lib():
    """The profiling build of the library (per-CTA phase timestamps), loaded
    beside the package's product library; built on demand."""
    import ctypes
    from qextract_infer_b200 import _lib, build
    path = build.LIB_TRACE
    if not os.path.exists(path):
        build.build(trace=True)
    lib = ctypes.CDLL(path)
    for name, (res, argt) in _lib.SIGNATURES.items():
        getattr(lib, name).restype = res
        getattr(lib, name).argtypes = argt
    return lib


def _timeline_summary(t, names, calls):
    """t [calls, grid, 16] int64 ns stamps -> per phase the median over calls
    1..calls-1 of (median over CTAs of the phase - the call's first CTA entry),
    in us; plus the previous call's last exit and the call period."""
    import numpy as np
    out = {}
    firsts = [t[c, :, 0][t[c, :, 0] > 0].min() for c in range(calls)]
    for slot, name in names:
        vals = []
        for c in range(1, calls):
            v = t[c, :, slot]
            v = v[v > 0]
            if len(v):
                vals.append((np.median(v) - firsts[c]) / 1e3)
        if vals:
            out[name] = round(float(np.median(vals)), 3)
    last_exit = []
    for c in range(1, calls):
        ex = t[c - 1, :, names[-1][0]]
        ex = ex[ex > 0]
        if len(ex):
            last_exit.append((ex.max() - firsts[c]) / 1e3)
    out["previous_call_last_exit"] = round(float(np.median(last_exit)), 3) if last_exit else None
    out["period"] = round(float((firsts[calls - 1] - firsts[1]) / (calls - 2) / 1e3), 3)
    return out


def run_timeline(args):
    """Per-CTA phase timeline (%globaltimer) of a graph-replayed chain of
    calls, from the profiling build of the library (libqx_b200_trace.so,
    ``python -m qextract_infer_b200.build --trace``): the decode GEMV at the
    Qwen3-4B gate_proj shape (8 calls over rotating weight sets) and the decode
    attention of one sequence over a full 4 + 4092 ring (8 calls over 12
    layers' caches).  One JSON line per kernel: each phase as the median over
    the calls of (median CTA time - the call's first CTA entry), in us."""
    import ctypes
    import numpy as np
    import torch
    lib = _trace_lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    st = torch.cuda.Stream(dev)
    calls = 8
    # ---- decode GEMV, config 0
    nsets = int(np.ceil(2.2 * L2_BYTES / BYTES_PER_CALL))
    sets = make_weight_sets(torch, dev, nsets)
    x = torch.randn(M, K, device=dev).half()
    ys = [torch.empty(M, N, dtype=torch.float16, device=dev) for _ in range(2)]
    scale = float(np.float32(ALPHA) / np.float32(RANK))
    plan = (ctypes.c_int * 5)()
    assert lib.qx_w4a16_gemv_plan(M, K, N, RANK, GROUP, 1, plan) == 0
    grid = plan[0] * plan[1]

    def gemv(i):
        qw, sc, qz, A, B = sets[i % nsets]
        rc = lib.qx_w4a16_lora_gemv(x.data_ptr(), qw.data_ptr(), sc.data_ptr(), qz.data_ptr(), 1, 0,
                                    A.data_ptr(), B.data_ptr(), ys[i & 1].data_ptr(), M, K, N, RANK, GROUP,
                                    scale, ctypes.c_void_p(st.cuda_stream))
        if rc:
            raise RuntimeError(lib.qx_last_error().decode())

    def traced_chain(kernel, fn, nwarm, grid_max):
        buf = torch.zeros(calls * grid_max * 16, dtype=torch.int64, device=dev)
        with torch.cuda.stream(st):
            for i in range(nwarm):
                fn(i)
        st.synchronize()
        if lib.qx_trace_launches(kernel, ctypes.c_void_p(buf.data_ptr()), calls):
            raise RuntimeError(lib.qx_last_error().decode())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for i in range(calls):
                fn(i)
        lib.qx_trace_launches(kernel, None, 0)
        with torch.cuda.stream(st):
            for _ in range(3):
                g.replay()
        st.synchronize()
        buf.zero_()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            e0.record(st)
            g.replay()
            e1.record(st)
        st.synchronize()
        flat = buf.view(-1, 16).cpu().numpy()
        n = int((flat[:, 0] > 0).sum()) // calls
        del g
        return flat[:calls * n].reshape(calls, n, 16), n, e0.elapsed_time(e1) * 1e3 / calls

    t, n, us = traced_chain(0, gemv, nsets, grid)
    names = [(0, "entry"), (1, "dependency_wait_passed"), (2, "first_group_landed"), (3, "weight_loop_done"),
             (4, "helper_lora_down_done"), (5, "lora_up_done"), (6, "partials_sent"),
             (7, "partials_received"), (8, "exit")]
    d = {"timeline": "w4a16_lora_gemv", "workload": WORKLOAD, "grid": n, "calls": calls,
         "us_per_call_traced": round(us, 3), "unit": "us from the call's first CTA entry",
         "ctas_entered_before_previous_call_ended": round(float(np.mean(
             [np.mean(t[c, :, 0] < t[c - 1, :, 8][t[c - 1, :, 8] > 0].max()) for c in range(1, calls)])), 3)}
    d.update(_timeline_summary(t, names, calls))
    print(json.dumps(d), flush=True)
    del sets
    torch.cuda.empty_cache()
    # ---- decode attention, one sequence over a full ring
    L, Hkv, D, S, W, Hq = 12, 8, 128, 4, 4092, 32
    k = torch.randn(L, 1, S + W, Hkv, D, device=dev).half()
    v = torch.randn(L, 1, S + W, Hkv, D, device=dev).half()
    q = torch.randn(1, Hq, D, device=dev).half()
    out = torch.empty_like(q)
    wsb = lib.qx_decode_attention_workspace_size(1, Hq, Hkv, D, S, W)
    ws = torch.zeros(wsb + 256, dtype=torch.uint8, device=dev)
    count = 32768 + 64

    def attn(i):
        rc = lib.qx_decode_attention(q.data_ptr(), k[i % L].data_ptr(), v[i % L].data_ptr(), out.data_ptr(), 1,
                                     Hq, Hkv, D, S, W, count, 0.0, ws.data_ptr(), wsb,
                                     ctypes.c_void_p(st.cuda_stream))
        if rc:
            raise RuntimeError(lib.qx_last_error().decode())

    t, n, us = traced_chain(1, attn, L, 64 * Hkv)
    names = [(0, "entry"), (1, "dependency_wait_passed"), (2, "first_tile_landed"), (3, "tile_loop_done"),
             (4, "warps_merged"), (5, "chunk_barrier_passed"), (6, "exit")]
    d = {"timeline": "decode_attention", "workload": "one sequence, 32/8 heads x 128, 4 + 4092 ring full",
         "grid": n, "calls": calls, "us_per_call_traced": round(us, 3),
         "unit": "us from the call's first CTA entry"}
    d.update(_timeline_summary(t, names, calls))
    print(json.dumps(d), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--nsets", type=int, default=0,
                    help="weight sets in the rotation (default: enough for > 2x L2)")
    ap.add_argument("--skip-e2e", action="store_true", help="omit the public-API timing")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline")
    ap.add_argument("--skip-tp", action="store_true", help="omit the Qwen3-8B TP decode keys")
    ap.add_argument("--skip-gemm", action="store_true", help="omit the prefill GEMM key")
    ap.add_argument("--batches", default="1,32", help="decode_tp: batch sizes")
    ap.add_argument("--prompt", type=int, default=8192, help="decode_tp: prompt tokens")
    ap.add_argument("--decode", type=int, default=64, help="decode_tp: greedy decode tokens")
    ap.add_argument("--workload", choices=["decode_gemv", "kernels", "prefill_gemm", "decode_tp",
                                           "profile_cases", "profile_decode_step", "timeline"],
                    default="decode_gemv",
                    help="decode_gemv: the headline line; kernels: RMSNorm/SwiGLU/ring/attention lines; "
                         "prefill_gemm: the tcgen05 GEMM over the Qwen3-8B shapes at M=4096")
    args = ap.parse_args()
    if args.workload == "kernels":
        return run_kernel_suite(args)
    if args.workload == "prefill_gemm":
        return run_prefill_suite(args)
    if args.workload == "decode_tp":
        return run_decode_tp(args)
    if args.workload == "profile_cases":
        return run_profile_cases(args)
    if args.workload == "profile_decode_step":
        return run_profile_decode_step(args)
    if args.workload == "timeline":
        return run_timeline(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
