"""Shared helpers for the test-suite (comparison utilities, fixture loading)."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as f:
        return {k: f[k] for k in f.files}


def f16_ulp_diff(a, b):
    """Elementwise distance in fp16 ulps (monotonic integer mapping)."""
    def key(x):
        i = np.ascontiguousarray(x, dtype=np.float16).view(np.int16).astype(np.int32)
        return np.where(i < 0, -(i & 0x7FFF), i)
    return np.abs(key(a) - key(b))


def assert_close(actual, expected, rtol, atol, msg=""):
    a = np.asarray(actual, dtype=np.float32)
    e = np.asarray(expected, dtype=np.float32)
    assert a.shape == e.shape, (a.shape, e.shape, msg)
    err = np.abs(a - e)
    bound = atol + rtol * np.abs(e)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), a.shape)
        raise AssertionError(f"{msg}: {bad.sum()} / {a.size} elements out of tolerance "
                             f"(rtol={rtol}, atol={atol}); worst at {i}: "
                             f"actual={a[i]} expected={e[i]}")


def assert_f16_match(actual, expected, max_ulp=1, atol=5e-4, msg=""):
    """fp16 arrays agree to ``max_ulp`` ulps, or to ``atol`` absolute where the
    values are near zero (fp32 summation-order differences before rounding)."""
    a = np.asarray(actual, dtype=np.float16)
    e = np.asarray(expected, dtype=np.float16)
    assert a.shape == e.shape, (a.shape, e.shape, msg)
    ok = (f16_ulp_diff(a, e) <= max_ulp) | (np.abs(a.astype(np.float32) - e.astype(np.float32)) <= atol)
    if not ok.all():
        i = np.argwhere(~ok)[0]
        raise AssertionError(f"{msg}: {(~ok).sum()} mismatches; first at {tuple(i)}: "
                             f"{a[tuple(i)]} vs {e[tuple(i)]}")


def dev_tensor(a, device="cuda"):
    """numpy -> torch on the GPU (same bytes; int32 stays int32)."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def to_np(t):
    return t.detach().cpu().numpy()
