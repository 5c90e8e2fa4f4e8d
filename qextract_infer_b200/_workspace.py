"""Per-(device, stream, op) scratch buffers for the kernels that take a workspace.

The library allocates nothing itself.  The split-slot decode attention needs a
workspace whose counter region starts at zero (it leaves its counters at zero
again; the rest of the buffer holds partial results) and the prefill GEMM one
for its LoRA down-projection, so one zero-filled buffer per (stream, op) is
reused across calls.  Calls on one stream are ordered and never overlap on the
buffer; ops of different kinds get different buffers because one op's partials
would otherwise sit where the other keeps its counters.  (The decode GEMV
reduces through distributed shared memory and takes no workspace.)
"""

from __future__ import annotations

import threading

import torch

_lock = threading.Lock()
_buffers: dict = {}


def get(device: torch.device, stream: torch.cuda.Stream, nbytes: int, op: str) -> torch.Tensor:
    """A zero-initialised uint8 buffer of at least ``nbytes`` (256-byte aligned)
    dedicated to ``op`` on ``stream`` of ``device``."""
    key = (device.index, stream.cuda_stream, op)
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
