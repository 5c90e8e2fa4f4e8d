"""Per-(device, stream) scratch buffers for the kernels that reduce across CTAs.

The library allocates nothing itself.  The split-K GEMV and the split-slot
decode attention need a small workspace whose counters start at zero; every
kernel leaves its counters at zero again, so one zero-filled buffer per
stream is reused across calls (calls on one stream are ordered, so they never
overlap on the buffer).
"""

from __future__ import annotations

import threading

import torch

_lock = threading.Lock()
_buffers: dict = {}


def get(device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> torch.Tensor:
    """A zero-initialised uint8 buffer of at least ``nbytes`` (256-byte aligned)
    dedicated to ``stream`` on ``device``."""
    key = (device.index, stream.cuda_stream)
    with _lock:
        buf = _buffers.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(int(nbytes), 1 << 20)
            if buf is not None:
                size = max(size, 2 * buf.numel())
            with torch.cuda.stream(stream):
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
            _buffers[key] = buf
        return buf


def clear() -> None:
    with _lock:
        _buffers.clear()
