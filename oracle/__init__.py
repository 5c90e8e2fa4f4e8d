"""CPU oracle for the QExtract-Infer hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package
(``qextract_infer_b200``) imports this package; only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
call it, and only as the checker or as the timed CPU baseline.

Every function restates, in numpy (or plain C in ``qx_oracle.c``), the
algorithm of the reference implementation and cites the reference file:line
it follows.  Paths in citations are relative to the QExtract-Infer project
root.

Parity pinning: ``tests/golden/make_golden.py`` imported the reference's own
PyTorch functions (``tests/test_w4a16_gemv.py``, ``tests/test_rmsnorm.py``,
``tests/test_swiglu.py``, ``qextract/kv_cache.py``) and wrote their outputs as
fixtures under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this
oracle against those fixtures (bit-exact for integer/index work, bit-exact or
1-ulp for fp16 outputs).  The GQA decode-attention oracle has no reference
implementation to pin against (the reference has no attention kernel); it
restates HF transformers' Qwen3 eager attention and is marked
"parity unpinned" in ``attention.py``.
"""

from .gptq import (  # noqa: F401
    unpack_int4_rows,
    pack_int4_rows,
    unpack_qzeros,
    pack_qzeros,
    dequantize_gptq,
    w4a16_gemv_ref,
    w4a16_lora_gemv_ref,
    simulate_gptq_quantize,
    make_gemv_inputs,
)
from .norms import rmsnorm_ref, swiglu_ref, swiglu_ref_single_round  # noqa: F401
from .ring import RingIndexOracle, RingCacheOracle  # noqa: F401
from .attention import gqa_decode_attention_ref, prefill_attention_ref, ring_positions  # noqa: F401
