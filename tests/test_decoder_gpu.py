"""Tensor-parallel Qwen3-architecture decoder (TP = 1 on one GPU) against its
fp32 torch restatement: prefill in chunks that exercise both the tensor-core
GEMM (128-row chunks) and the decode GEMV, a sink + window ring that wraps,
then greedy decode steps.  Tolerance: rtol = atol = 1e-2 on the final hidden
state and on the logits, relative to their scale."""

import pytest
import torch

from tests.decoder_ref import RefDecoder

pytestmark = pytest.mark.gpu


def _tiny_cfg():
    from qextract_infer_b200.tp_decoder import DecoderConfig
    return DecoderConfig(num_layers=2, hidden=512, intermediate=1024, num_q_heads=4, num_kv_heads=2,
                         head_dim=128, vocab=1024, sink=4, window=60, init_std=0.5)


def _close(a, b, what, tol=1e-2):
    a, b = a.float(), b.float()
    scale = b.abs().max().item()
    err = (a - b).abs().max().item()
    assert err <= tol * scale + tol, f"{what}: max err {err} at scale {scale}"


@pytest.mark.parametrize("fused_attention", [True, False])
def test_prefill_and_decode_match_reference(fused_attention):
    """Both decode-step attention forms: the fused norm/RoPE/append/attention
    kernel and the append kernel followed by attention."""
    from qextract_infer_b200.tp_decoder import TPDecoder
    assert torch.cuda.is_available()
    dev = torch.device("cuda", 0)
    cfg = _tiny_cfg()
    B, T = 2, 100
    dec = TPDecoder(cfg, batch=B, device=dev, seed=7)
    dec.fused_attention = fused_attention
    ref = RefDecoder(dec)
    toks = torch.randint(0, cfg.vocab, (B, T), generator=torch.Generator().manual_seed(4)).to(dev)
    nxt, hid = dec.prefill(toks, chunk=64, return_hidden=True)
    for t in range(T):
        xr = ref.token(toks[:, t])
    _close(hid, xr, "prefill hidden")
    _close(dec._greedy_logits(hid), ref.logits(xr), "prefill logits")
    cur = toks[:, -1]
    for step in range(6):
        cur_in = torch.randint(0, cfg.vocab, (B,), generator=torch.Generator().manual_seed(50 + step)).to(dev)
        nxt, hid = dec.decode_step(cur_in, return_hidden=True)
        xr = ref.token(cur_in)
        _close(hid, xr, f"decode step {step} hidden")
        _close(dec._greedy_logits(hid), ref.logits(xr), f"decode step {step} logits")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="tensor parallelism needs two GPUs")
def test_tensor_parallel_two_ranks_match_reference():
    """TP = 2 over NCCL (torchrun, one process per GPU): column/row-parallel
    linears, the all-reduces and the vocab-split greedy against the unsharded
    reference on each rank."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29531",
           os.path.join(root, "tests", "tp_decoder_check.py")]
    r = subprocess.run(cmd, cwd=root, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert r.stdout.count("ok=True") == 2, r.stdout[-2000:]
