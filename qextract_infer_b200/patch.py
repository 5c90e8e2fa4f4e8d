"""``patch_qwen``: swap the hot ops of a HuggingFace Qwen3 model for the
sm_100a kernels (reference: ``qextract/patch.py:10-162``).

Same entry point, flags and counters as the reference.  Fixes relative to it:

* GPTQ ``qzeros`` (int32 ``[G, N/8]``) are used as packed zeros instead of
  being handed to an fp16-zeros kernel (``patch.py:131`` vs
  ``w4a16_lora_gemv.cu:310``); ``gptq_zero_offset=1`` selects the GPTQ-v1
  "+1" storage convention;
* projection inputs ``[B, T, K]`` keep their leading dims (the reference
  kernel returned a 1-D ``[N]``);
* GPTQ act-order checkpoints (a ``g_idx`` that is not ``k // group_size``) are
  accepted: the packed rows are re-ordered once so that every quantisation
  group is contiguous (``act_order_repack``), the LoRA A rows alike, and each
  call gathers the input columns in the same order (the reference kernel
  assumes ``group = k // group_size``, ``w4a16_lora_gemv.cu:181``);
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


def act_order_repack(qweight: torch.Tensor, g_idx: torch.Tensor, group: int):
    """GPTQ act-order: ``g_idx[k]`` is the quantisation group of input row k.
    Returns ``(qweight', perm)`` with the packed rows re-ordered so that row j
    of ``qweight'`` is input row ``perm[j]`` and belongs to group
    ``j // group`` (``perm`` sorts the rows by group, stably), or ``None`` when
    ``g_idx`` already is ``k // group``.  Raises if a group does not hold
    exactly ``group`` rows.  Then ``x . W == x[..., perm] . W'`` with the
    scales and zero points unchanged."""
    K = qweight.size(0) * 8
    g = g_idx.to(device=qweight.device, dtype=torch.int64).reshape(-1)
    if g.numel() != K:
        raise RuntimeError(f"g_idx has {g.numel()} entries, qweight {K} rows")
    ar = torch.arange(K, device=qweight.device)
    if torch.equal(g, ar // group):
        return None
    counts = torch.bincount(g, minlength=K // group)
    if counts.numel() != K // group or not bool((counts == group).all()):
        raise RuntimeError("act-order g_idx: every group must hold exactly group_size rows")
    perm = torch.sort(g, stable=True).indices
    shifts = torch.arange(0, 32, 4, device=qweight.device, dtype=torch.int64)
    q = (qweight.to(torch.int64)[:, None, :] >> shifts[None, :, None]) & 0xF  # [K/8, 8, N]
    q = q.reshape(K, -1).index_select(0, perm).reshape(K // 8, 8, -1)
    packed = (q << shifts[None, :, None]).sum(1)
    packed = torch.where(packed >= 2 ** 31, packed - 2 ** 32, packed).to(torch.int32)
    return packed.contiguous(), perm


def _gptq_tensors(layer):
    """(qweight, scales, zeros, group, bias, perm): ``perm`` is the input-column
    order of an act-order checkpoint (None otherwise)."""
    if not hasattr(layer, "qweight") or not hasattr(layer, "scales"):
        return None
    zeros = getattr(layer, "qzeros", getattr(layer, "zeros", None))
    if zeros is None:
        return None
    group = int(getattr(layer, "group_size", 128))
    scales = layer.scales.half().contiguous()
    qweight, perm = layer.qweight.contiguous(), None
    g_idx = getattr(layer, "g_idx", None)
    if g_idx is not None:
        r = act_order_repack(qweight, g_idx, group)
        if r is not None:
            qweight, perm = r
    return qweight, scales, zeros.contiguous(), group, getattr(layer, "bias", None), perm


def _patch_lora_gemv(proj_module, fused_fn, zero_offset: int) -> bool:
    """Reference ``patch.py:117-162``: PEFT LoRA wrapper over a GPTQ base layer."""
    base = getattr(proj_module, "base_layer", None)
    if base is None:
        return False
    t = _gptq_tensors(base)
    if t is None:
        return False
    qweight, scales, zeros, group, bias, perm = t
    lora_A = getattr(proj_module, "lora_A", None)
    if lora_A is None or "default" not in lora_A:
        return False
    # PEFT keeps nn.Linear weights: A [r, in] -> [in, r]; B [out, r] -> [r, out]
    A = proj_module.lora_A["default"].weight.detach().t().contiguous().half()
    if perm is not None:
        A = A.index_select(0, perm.to(A.device)).contiguous()
    B = proj_module.lora_B["default"].weight.detach().t().contiguous().half()
    alpha = getattr(proj_module, "lora_alpha", {}).get("default", 16.0)

    def new_forward(self, x):
        in_dtype = x.dtype
        xh = x.half() if in_dtype != torch.float16 else x
        if perm is not None:
            xh = xh.index_select(-1, perm)
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
    qweight, scales, zeros, group, bias, perm = t

    def new_forward(self, x):
        in_dtype = x.dtype
        xh = x.half() if in_dtype != torch.float16 else x
        if perm is not None:
            xh = xh.index_select(-1, perm)
        y = fused_fn(xh.contiguous(), qweight, scales, zeros, group, zero_offset=zero_offset)
        if bias is not None:
            y = y + bias.to(y.dtype)
        return y.to(in_dtype)

    proj_module.forward = types.MethodType(new_forward, proj_module)
    return True
