"""Loader for ``libqx_b200.so`` (the C ABI declared in ``include/qx_b200.h``).

There is no fallback: if the library is missing or cannot be loaded, every op
raises.  Build it with ``python -m qextract_infer_b200.build``.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqx_b200.so")

_lock = threading.Lock()
_lib = None

c_int, c_int64, c_float, c_size_t, c_void_p, c_char_p = (
    ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_char_p)

# name -> (restype, argtypes); mirrors include/qx_b200.h
SIGNATURES = {
    "qx_last_error": (c_char_p, []),
    "qx_version": (c_char_p, []),
    "qx_copy_async": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "qx_trace_launches": (c_int, [c_int, c_void_p, c_int]),
    "qx_w4a16_lora_gemv": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p,
                                   c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float,
                                   c_void_p]),
    "qx_w4a16_lora_gemv_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                          c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                          c_int, c_float, c_void_p]),
    "qx_w4a16_lora_gemv_addnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
                                           c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                           c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_void_p]),
    "qx_set_pdl": (c_int, [c_int]),
    "qx_w4a16_lora_gemv_host": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_int,
                                        c_int, c_int, c_float, c_void_p]),
    "qx_w4a16_gemv_plan": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "qx_w4a16_gemv_pin_plan": (c_int, [c_int, c_int]),
    "qx_w4a16_lora_gemm_sm100_workspace_size": (c_size_t, [c_int, c_int]),
    "qx_w4a16_lora_gemm_sm100": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                         c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                         c_int, c_float, c_void_p, c_size_t, c_void_p]),
    "qx_get_device_error": (c_int, [c_void_p, c_int]),
    "qx_fused_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_void_p]),
    "qx_fused_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "qx_add_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float,
                               c_void_p]),
    "qx_qk_norm_rope_append": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                       c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_int, c_int, c_int64, c_void_p]),
    "qx_swiglu_packed": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "qx_nvlink_ar_handle_bytes": (c_size_t, []),
    "qx_nvlink_ar_create": (c_int, [c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "qx_nvlink_ar_open": (c_int, [c_void_p, c_void_p]),
    "qx_nvlink_ar_open_local": (c_int, [c_void_p, c_void_p]),
    "qx_nvlink_ar_set_timeout": (c_int, [c_void_p, c_int64]),
    "qx_nvlink_ar_add_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                         c_float, c_void_p]),
    "qx_nvlink_ar_destroy": (c_int, [c_void_p]),
    "qx_ring_append": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                               c_int, c_int, c_int64, c_void_p]),
    "qx_ring_slot_indices": (c_int64, [c_void_p, c_int, c_int, c_int64, c_void_p]),
    "qx_ring_gather": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                               c_int, c_int64, c_void_p]),
    "qx_decode_attention_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "qx_decode_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                    c_int, c_int, c_int, c_int64, c_float, c_void_p, c_size_t,
                                    c_void_p]),
    "qx_decode_attention_ex": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                       c_int, c_int, c_int, c_int64, c_float, c_void_p, c_size_t,
                                       c_int, c_void_p]),
    "qx_prefill_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int64,
                                     c_float, c_void_p]),
    "qx_decode_attention_qkv": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
                                        c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                        c_int, c_int64, c_float, c_void_p, c_size_t, c_void_p]),
    "qx_lm_head_argmax_workspace_size": (c_size_t, [c_int]),
    "qx_lm_head_argmax": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int64, c_void_p, c_void_p,
                                  c_void_p, c_size_t, c_void_p]),
    "qx_decode_attention_pin_merge": (c_int, [c_int]),
    "qx_decode_attention_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                            c_int, c_int, c_int, c_int, c_int64, c_float,
                                            c_void_p]),
}


class QXError(RuntimeError):
    """A C-ABI call returned a negative status."""


def load(path: str | None = None):
    """Load (once) and return the ctypes handle; raises if the library is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(
                f"qextract_infer_b200: native library not built ({p} missing); run "
                "`python -m qextract_infer_b200.build`")
        try:
            lib = ctypes.CDLL(p)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
        except (OSError, AttributeError) as e:  # unloadable or stale build
            raise ImportError(f"qextract_infer_b200: cannot use {p}: {e}; rebuild with "
                              "`python -m qextract_infer_b200.build --force`") from e
        _lib = lib
        return lib


def last_error() -> str:
    lib = load()
    return lib.qx_last_error().decode(errors="replace")


def check(rc: int, what: str) -> int:
    if rc < 0:
        raise QXError(f"{what}: {last_error()} (status {rc})")
    return rc
