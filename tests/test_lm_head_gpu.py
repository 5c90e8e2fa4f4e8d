"""Greedy head (``lm_head_argmax``): fp16 logits h W (fp32 accumulation) and
per row the largest logit with its index, against torch fp32 on the GPU.  The
chosen logit must be the maximum within fp16 rounding (rtol = atol = 1e-2 on
the logit scale, the tolerance of every fp16 output here) and exact ties must
go to the smallest index."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from qextract_infer_b200 import _C
    return _C


@pytest.mark.parametrize("B,H,V,off", [(1, 4096, 151936, 0), (3, 4096, 18992, 5 * 18992), (16, 512, 1024, 0),
                                       (17, 4096, 37984, 37984), (32, 4096, 151936, 0), (2, 64, 520, 7)])
def test_matches_torch(C, B, H, V, off):
    g = torch.Generator(device="cuda").manual_seed(B * 7 + V)
    h = torch.randn(B, H, generator=g, device="cuda").half()
    W = (torch.randn(H, V, generator=g, device="cuda") * 0.02).half()
    val, idx = C.lm_head_argmax(h, W, off)
    ref = (h.float() @ W.float()).half().float()
    rv, ri = ref.max(-1)
    scale = ref.abs().max().item()
    tol = 1e-2 * scale + 1e-2
    assert torch.all((val - rv).abs() <= tol), (val, rv)
    picked = ref.gather(1, (idx - off).view(-1, 1)).view(-1)
    assert torch.all(picked >= rv - tol), (picked, rv)
    assert torch.all((idx - off >= 0) & (idx - off < V))
    # where the maximum is clear, the index is torch's
    top2 = ref.topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > tol
    assert torch.equal(idx[clear] - off, ri[clear])


def test_ties_take_the_smallest_index(C):
    H, V = 256, 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    h = torch.randn(2, H, generator=g, device="cuda").half()
    W = (torch.randn(H, V, generator=g, device="cuda") * 0.02).half()
    ref = (h.float() @ W.float()).half().float()
    best = ref[0].argmax().item()
    # the same column at a smaller and at a larger index: equal logits
    lo, hi = (best // 2), (best + V) // 2 + 1
    W[:, lo] = W[:, best]
    W[:, min(hi, V - 1)] = W[:, best]
    val, idx = C.lm_head_argmax(h, W, 100)
    assert idx[0].item() == 100 + min(lo, best)
