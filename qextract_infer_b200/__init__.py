"""qextract_infer_b200 -- sm_100a (B200) kernels behind the QExtract-Infer API.

Drop-in for the reference package ``qextract`` (``qextract/__init__.py:11-33``):
the same op names (``fused_rmsnorm``, ``fused_swiglu``, ``w4a16_gemv``,
``w4a16_lora_gemv``, ``RingBufferKVCache``), ``patch_qwen``,
``QExtractKVCache``, ``_C_AVAILABLE`` and ``check_backend()``.
The ops run hand-written CUDA for sm_100a through the C ABI of
``libqx_b200.so``; there is no CPU fallback.
"""

__version__ = "0.1.0"

try:
    from ._C import (  # noqa: F401
        RingBufferKVCache,
        decode_attention,
        fused_rmsnorm,
        fused_swiglu,
        w4a16_gemv,
        w4a16_lora_gemv,
    )
    _C_AVAILABLE = True
except ImportError:
    _C_AVAILABLE = False

from .kv_cache import QExtractKVCache  # noqa: E402,F401
from .patch import patch_qwen  # noqa: E402,F401


def check_backend() -> bool:
    """True when the native library is loaded (reference: ``qextract/__init__.py:27-33``)."""
    if _C_AVAILABLE:
        print("[qextract_infer_b200] native sm_100a library loaded")
    else:
        print("[qextract_infer_b200] native library missing: run "
              "`python -m qextract_infer_b200.build`")
    return _C_AVAILABLE
