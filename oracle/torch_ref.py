"""The reference's own PyTorch CPU path for the W4A16-LoRA GEMV, restated in
torch operation for operation.  TEST INFRASTRUCTURE ONLY: it is a checker in
``tests/`` and the timed CPU baseline of ``bench.py`` (the reference's Python
cannot travel to the GPU box, so its steps are restated here).

Steps followed (paths relative to the QExtract-Infer project root):

* ``tests/test_w4a16_gemv.py:68-90`` (``dequantize_gptq_ref``): a Python loop
  over the packed rows; for each of the 8 nibbles of a packed row, one torch
  expression ``((q - z) * s).half()`` over all N columns, with ``s`` and ``z``
  the fp32 copies of the row's group scales / zero points;
* ``tests/test_w4a16_gemv.py:178-186``: ``x.float() @ W.float()``, the LoRA
  term ``(x.float() @ A.float()) @ B.float()`` scaled by ``alpha / rank``, one
  fp16 rounding of the sum.

The reference's test feeds fp16 zero points ``[G, N]``; GPTQ checkpoints carry
packed ``qzeros`` int32 ``[G, N/8]``, which ``unpack_qzeros_fp16`` expands
first (nibble ``n % 8`` of word ``n / 8``, the layout ``oracle/gptq.py``
restates), outside the timed reference steps.
"""

from __future__ import annotations

import torch

__all__ = ["unpack_qzeros_fp16", "dequantize_rows", "w4a16_lora_gemv_cpu"]


def unpack_qzeros_fp16(qzeros: torch.Tensor, n: int, zero_offset: int = 0) -> torch.Tensor:
    """int32 ``[G, N/8]`` GPTQ qzeros -> fp16 ``[G, N]`` zero points."""
    q = qzeros.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(8, dtype=torch.int64) * 4
    nib = (q[:, :, None] >> shifts[None, None, :]) & 0xF
    return (nib.reshape(q.shape[0], n) + zero_offset).to(torch.float16)


def dequantize_rows(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                    hidden: int, group_size: int = 128) -> torch.Tensor:
    """fp16 ``[hidden, N]`` from GPTQ packing, one packed row and one nibble at
    a time (``tests/test_w4a16_gemv.py:68-90``)."""
    n_packed, n_out = qweight.shape
    w = torch.zeros(hidden, n_out, dtype=torch.float16)
    for p in range(n_packed):
        word = qweight[p]
        first = 8 * p
        grp = first // group_size
        s = scales[grp].float()
        z = zeros[grp].float()
        for i in range(8):
            if first + i >= hidden:
                break
            q = ((word >> (4 * i)) & 0xF).float()
            w[first + i] = ((q - z) * s).half()
    return w


def w4a16_lora_gemv_cpu(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                        zeros: torch.Tensor, lora_A: torch.Tensor | None = None,
                        lora_B: torch.Tensor | None = None, group_size: int = 128,
                        lora_alpha: float = 16.0, zero_offset: int = 0) -> torch.Tensor:
    """``fp16(x W + (alpha / r) (x A) B)`` the reference's way
    (``tests/test_w4a16_gemv.py:178-186``); ``zeros`` fp16 ``[G, N]`` or packed
    int32 qzeros ``[G, N/8]``; ``x`` ``[K]`` or ``[M, K]``."""
    if zeros.dtype == torch.int32:
        zeros = unpack_qzeros_fp16(zeros, qweight.shape[1], zero_offset)
    hidden = qweight.shape[0] * 8
    w = dequantize_rows(qweight, scales, zeros, hidden, group_size)
    xf = x.float()
    y = xf @ w.float()
    if lora_A is not None:
        rank = lora_A.shape[1]
        y = y + (lora_alpha / rank) * ((xf @ lora_A.float()) @ lora_B.float())
    return y.half()
