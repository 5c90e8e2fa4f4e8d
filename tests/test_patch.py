"""patch_qwen on a tiny HF Qwen3 model with GPTQ + LoRA stand-ins.

CPU tests cover the host logic (which modules get patched, counters, flags);
the GPU test compares the patched model's logits with the unpatched model
(reference math in torch fp32 inside the mocks), rtol = atol = 1e-2 on a
logit scale.
"""

import pytest
import torch

from tests.qwen_mocks import make_tiny_qwen3


def test_patch_counters_cpu():
    import qextract_infer_b200 as qx
    model = make_tiny_qwen3(num_layers=3)
    qx.patch_qwen(model, verbose=False)
    assert model._qextract_patched == {"rmsnorm": 7, "swiglu": 3, "lora_gemv": 21, "w4a16_gemv": 0}


def test_patch_flags_cpu():
    import qextract_infer_b200 as qx
    m = make_tiny_qwen3(num_layers=2)
    qx.patch_qwen(m, enable_rmsnorm=False, enable_swiglu=False, verbose=False)
    assert m._qextract_patched["rmsnorm"] == 0 and m._qextract_patched["swiglu"] == 0
    assert m._qextract_patched["lora_gemv"] == 14
    plain = make_tiny_qwen3(num_layers=2, lora=False)
    qx.patch_qwen(plain, verbose=False)
    assert plain._qextract_patched["lora_gemv"] == 0  # reference: only PEFT-wrapped layers
    plain2 = make_tiny_qwen3(num_layers=2, lora=False)
    qx.patch_qwen(plain2, patch_plain_gptq=True, verbose=False)
    assert plain2._qextract_patched["w4a16_gemv"] == 14


def test_patched_forward_rejects_cpu_inputs():
    import qextract_infer_b200 as qx
    model = make_tiny_qwen3(num_layers=1)
    qx.patch_qwen(model, verbose=False)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        model(torch.zeros(1, 4, dtype=torch.long))


@pytest.mark.gpu
@pytest.mark.parametrize("lora,act_order", [(True, False), (False, False), (True, True), (False, True)])
def test_patched_model_matches_unpatched(lora, act_order):
    import qextract_infer_b200 as qx
    assert torch.cuda.is_available()
    model = make_tiny_qwen3(num_layers=2, lora=lora, act_order=act_order).half().cuda().eval()
    ids = torch.randint(0, 512, (2, 9), generator=torch.Generator().manual_seed(0)).cuda()
    with torch.no_grad():
        ref = model(ids).logits.float()
        qx.patch_qwen(model, patch_plain_gptq=not lora, verbose=False)
        got = model(ids).logits.float()
    n = model._qextract_patched
    assert n["rmsnorm"] == 5 and n["swiglu"] == 2
    assert (n["lora_gemv"] if lora else n["w4a16_gemv"]) == 14
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    assert err <= 1e-2 * scale + 1e-2, (err, scale)


def test_act_order_repack_cpu():
    """act_order_repack: the re-ordered packed rows with the gathered input
    columns give the same product as the act-order layer (oracle dequant with
    g_idx); a g_idx of k // group is left alone; unequal groups are refused."""
    import numpy as np
    from qextract_infer_b200.patch import act_order_repack
    from tests.qwen_mocks import dequant_torch
    K, N, G = 512, 64, 128
    rng = np.random.default_rng(3)
    qw = torch.from_numpy(rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.uint64)
                          .astype(np.uint32).view(np.int32))
    sc = torch.from_numpy(rng.uniform(0.005, 0.02, size=(K // G, N)).astype(np.float16))
    qz = torch.from_numpy(rng.integers(0, 2 ** 32, size=(K // G, N // 8), dtype=np.uint64)
                          .astype(np.uint32).view(np.int32))
    g_idx = torch.from_numpy(rng.permutation(np.arange(K) // G).astype(np.int32))
    x = torch.randn(3, K, generator=torch.Generator().manual_seed(1))
    ref = x @ dequant_torch(qw, sc, qz, G, g_idx).float()
    qw2, perm = act_order_repack(qw, g_idx, G)
    got = x[:, perm] @ dequant_torch(qw2, sc, qz, G).float()
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-4)
    assert torch.equal(g_idx.long()[perm], torch.arange(K) // G)
    assert act_order_repack(qw, torch.arange(K) // G, G) is None
    with pytest.raises(RuntimeError, match="exactly group_size"):
        act_order_repack(qw, torch.zeros(K, dtype=torch.int32), G)
