"""``patch_qwen``: swap the hot ops of a HuggingFace Qwen3 model for the
sm_100a kernels (reference: ``qextract/patch.py:10-162``).

Same entry point, flags and counters as the reference.  Fixes relative to it:

* GPTQ ``qzeros`` (int32 ``[G, N/8]``) are used as packed zeros instead of
  being handed to an fp16-zeros kernel (``patch.py:131`` vs
  ``w4a16_lora_gemv.cu:310``); ``gptq_zero_offset=1`` selects the GPTQ-v1
  "+1" storage convention;
* projection inputs ``[B, T, K]`` keep their leading dims (the reference
  kernel returned a 1-D ``[N]``);
* everything runs on the current CUDA stream.

Optional extension: ``patch_plain_gptq=True`` also routes GPTQ layers that
carry no LoRA adapter through ``w4a16_gemv`` (counted as ``w4a16_gemv``).
"""

from __future__ import annotations

import types

import torch

_PROJ_NAMES = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]


def patch_qwen(model, enable_rmsnorm: bool = True, enable_swiglu: bool = True,
               enable_lora_gemv: bool = True, *, patch_plain_gptq: bool = False,
               gptq_zero_offset: int = 0, verbose: bool = True):
    """Patch ``model`` in place and return it (reference ``patch.py:10-70``)."""
    try:
        from ._C import fused_rmsnorm, fused_swiglu, w4a16_gemv, w4a16_lora_gemv
    except ImportError as e:
        raise RuntimeError("[qextract_infer_b200] native library not built: run "
                           "`python -m qextract_infer_b200.build`") from e

    patched = {"rmsnorm": 0, "swiglu": 0, "lora_gemv": 0, "w4a16_gemv": 0}
    for layer in model.model.layers:
        if enable_rmsnorm:
            for norm_name in ("input_layernorm", "post_attention_layernorm"):
                norm = getattr(layer, norm_name, None)
                if norm is not None:
                    _patch_rmsnorm(norm, fused_rmsnorm)
                    patched["rmsnorm"] += 1
        if enable_swiglu and hasattr(layer, "mlp"):
            _patch_swiglu(layer.mlp, fused_swiglu)
            patched["swiglu"] += 1
        if enable_lora_gemv:
            for sub in (getattr(layer, "self_attn", None), getattr(layer, "mlp", None)):
                if sub is None:
                    continue
                for name in _PROJ_NAMES:
                    proj = getattr(sub, name, None)
                    if proj is None:
                        continue
                    if _patch_lora_gemv(proj, w4a16_lora_gemv, gptq_zero_offset):
                        patched["lora_gemv"] += 1
                    elif patch_plain_gptq and _patch_plain_gptq(proj, w4a16_gemv, gptq_zero_offset):
                        patched["w4a16_gemv"] += 1
    if enable_rmsnorm and hasattr(model.model, "norm"):
        _patch_rmsnorm(model.model.norm, fused_rmsnorm)
        patched["rmsnorm"] += 1
    if verbose:
        print("[qextract_infer_b200] patched ops:")
        print(f"  - RMSNorm: {patched['rmsnorm']}")
        print(f"  - SwiGLU:  {patched['swiglu']}")
        print(f"  - LoRA GEMV: {patched['lora_gemv']}")
        if patch_plain_gptq:
            print(f"  - W4A16 GEMV: {patched['w4a16_gemv']}")
    model._qextract_patched = patched
    return model


def _patch_rmsnorm(norm_module, fused_fn):
    """Reference ``patch.py:73-87``: snapshot ``weight.half()`` and eps."""
    weight = norm_module.weight.data.half().contiguous()
    eps = getattr(norm_module, "variance_epsilon", getattr(norm_module, "eps", 1e-6))

    def new_forward(self, hidden_states):
        in_dtype = hidden_states.dtype
        h = hidden_states.half() if in_dtype != torch.float16 else hidden_states
        out = fused_fn(h.contiguous(), weight, eps)
        return out.to(in_dtype)

    norm_module.forward = types.MethodType(new_forward, norm_module)


def _patch_swiglu(mlp_module, fused_fn):
    """Reference ``patch.py:90-114``: silu(gate) * up fused; projections
    called through the (possibly patched) modules."""

    def new_forward(self, x):
        gate = self.gate_proj(x)
        up = self.up_proj(x)
        if gate.dtype != torch.float16:
            gate, up = gate.half(), up.half()
        act = fused_fn(gate.contiguous(), up.contiguous())
        return self.down_proj(act.to(x.dtype))

    mlp_module.forward = types.MethodType(new_forward, mlp_module)


def _gptq_tensors(layer):
    if not hasattr(layer, "qweight") or not hasattr(layer, "scales"):
        return None
    zeros = getattr(layer, "qzeros", getattr(layer, "zeros", None))
    if zeros is None:
        return None
    group = int(getattr(layer, "group_size", 128))
    scales = layer.scales.half().contiguous()
    return layer.qweight.contiguous(), scales, zeros.contiguous(), group, getattr(layer, "bias", None)


def _patch_lora_gemv(proj_module, fused_fn, zero_offset: int) -> bool:
    """Reference ``patch.py:117-162``: PEFT LoRA wrapper over a GPTQ base layer."""
    base = getattr(proj_module, "base_layer", None)
    if base is None:
        return False
    t = _gptq_tensors(base)
    if t is None:
        return False
    qweight, scales, zeros, group, bias = t
    lora_A = getattr(proj_module, "lora_A", None)
    if lora_A is None or "default" not in lora_A:
        return False
    # PEFT keeps nn.Linear weights: A [r, in] -> [in, r]; B [out, r] -> [r, out]
    A = proj_module.lora_A["default"].weight.detach().t().contiguous().half()
    B = proj_module.lora_B["default"].weight.detach().t().contiguous().half()
    alpha = getattr(proj_module, "lora_alpha", {}).get("default", 16.0)

    def new_forward(self, x):
        in_dtype = x.dtype
        xh = x.half() if in_dtype != torch.float16 else x
        y = fused_fn(xh.contiguous(), qweight, scales, zeros, A, B, group, alpha,
                     zero_offset=zero_offset)
        if bias is not None:
            y = y + bias.to(y.dtype)
        return y.to(in_dtype)

    proj_module.forward = types.MethodType(new_forward, proj_module)
    return True


def _patch_plain_gptq(proj_module, fused_fn, zero_offset: int) -> bool:
    t = _gptq_tensors(proj_module)
    if t is None:
        return False
    qweight, scales, zeros, group, bias = t

    def new_forward(self, x):
        in_dtype = x.dtype
        xh = x.half() if in_dtype != torch.float16 else x
        y = fused_fn(xh.contiguous(), qweight, scales, zeros, group, zero_offset=zero_offset)
        if bias is not None:
            y = y + bias.to(y.dtype)
        return y.to(in_dtype)

    proj_module.forward = types.MethodType(new_forward, proj_module)
    return True
