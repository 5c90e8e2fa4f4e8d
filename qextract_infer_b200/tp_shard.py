"""Tensor-parallel sharding rules of the decoder, as pure tensor functions.

The reference has no tensor parallelism; the linears these rules split are
the seven projections ``patch_qwen`` patches (``qextract/patch.py:51-58``),
each a GPTQ int4 weight (``qweight int32 [K/8, N]``, ``scales [K/g, N]``,
``qzeros int32 [K/g, N/8]``) with a LoRA pair (``A [K, r]``, ``B [r, N]``):

* column-parallel (q, k, v, gate, up): rank ``i`` keeps output columns
  ``[i N/tp, (i+1) N/tp)`` of ``qweight``, ``scales`` and LoRA ``B`` and the
  matching ``qzeros`` words (``N/tp`` must be a multiple of 8); LoRA ``A`` is
  replicated.  The rank's output is its column slice of the full output.
* row-parallel (o, down): rank ``i`` keeps input rows ``[i K/tp, (i+1) K/tp)``
  (``K/tp`` a multiple of the quantisation group) of ``qweight`` (packed rows),
  ``scales``, ``qzeros`` and LoRA ``A``; LoRA ``B`` is replicated.  The
  partial outputs sum to the full output: ``sum_i x_i W_i = x W`` and
  ``sum_i (x_i A_i) B = (x A) B``, so the LoRA partials ride in the same
  all-reduce as the base partials.
* vocabulary-parallel lm_head: rank ``i`` keeps vocabulary columns
  ``[i V/tp, (i+1) V/tp)``; greedy decoding gathers every rank's
  (max logit, global index) and keeps the largest (lowest rank on ties, which
  is the lowest index: the first maximum, as ``argmax`` over the full row).

The functions take and return torch tensors on any device (the decoder calls
them on the GPU; the CPU test suite checks them over ``gloo`` ranks).
"""

from __future__ import annotations

import torch

__all__ = ["shard_quant_linear", "shard_vocab", "merge_greedy"]


def shard_quant_linear(qweight, scales, qzeros, lora_A, lora_B, split, rank: int, world: int,
                       group: int):
    """This rank's ``(qweight, scales, qzeros, lora_A, lora_B)`` for ``split``
    "col" (output columns), "row" (input rows) or None (replicated).  Views;
    the caller makes them contiguous."""
    K, N = qweight.size(0) * 8, qweight.size(1)
    if world <= 1 or split is None:
        return qweight, scales, qzeros, lora_A, lora_B
    if split == "col":
        if N % world or (N // world) % 8:
            raise ValueError(f"column split of N={N} over {world} ranks needs N/tp % 8 == 0")
        n = N // world
        c0, c1 = rank * n, (rank + 1) * n
        return (qweight[:, c0:c1], scales[:, c0:c1], qzeros[:, c0 // 8:c1 // 8], lora_A,
                None if lora_B is None else lora_B[:, c0:c1])
    if split == "row":
        if K % world or (K // world) % group:
            raise ValueError(f"row split of K={K} over {world} ranks needs K/tp % group == 0")
        k = K // world
        k0, k1 = rank * k, (rank + 1) * k
        return (qweight[k0 // 8:k1 // 8], scales[k0 // group:k1 // group],
                qzeros[k0 // group:k1 // group], None if lora_A is None else lora_A[k0:k1], lora_B)
    raise ValueError(f"unknown split {split!r}")


def shard_vocab(lm_head: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's vocabulary columns of ``lm_head [H, V]``."""
    V = lm_head.size(1)
    if V % world:
        raise ValueError(f"vocabulary {V} does not split over {world} ranks")
    vs = V // world
    return lm_head[:, rank * vs:(rank + 1) * vs]


def merge_greedy(vals: torch.Tensor, idxs: torch.Tensor) -> torch.Tensor:
    """``vals``/``idxs`` ``[world, B]``: every rank's max logit and its global
    vocabulary index -> the greedy token ``[B]`` (first rank on ties)."""
    best = vals.argmax(dim=0)
    return idxs.gather(0, best[None, :])[0]
