"""One-shot all-reduce over NVLink peer memory, fused with the residual add
and RMSNorm that follow the row-parallel projections of the tensor-parallel
decode step (C-ABI ``qx_nvlink_ar_*``, ``csrc/nvlink_allreduce.cu``).  New
component: the reference has no tensor parallelism; NCCL's all-reduce is what
it replaces for the few rows of a decode step."""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

_LIB = _lib.load()


class NVLinkAllReduce:
    """Per-rank communicator over the ranks of ``group`` (one GPU each, one
    node).  Collective to construct: every rank allocates its shared buffer,
    the IPC handles are all-gathered and opened, then a barrier."""

    def __init__(self, group, max_rows: int, hidden: int, device):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_rows, self.hidden = int(max_rows), int(hidden)
        self.device = torch.device(device)
        hb = int(_LIB.qx_nvlink_ar_handle_bytes())
        handle = ctypes.create_string_buffer(hb)
        ctx = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(_LIB.qx_nvlink_ar_create(self.world, self.rank, self.max_rows, self.hidden,
                                                ctypes.byref(ctx), handle), "nvlink_ar_create")
        self._ctx = ctx
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        allh = ctypes.create_string_buffer(b"".join(handles), hb * self.world)
        with torch.cuda.device(self.device):
            _lib.check(_LIB.qx_nvlink_ar_open(self._ctx, allh), "nvlink_ar_open")
        dist.barrier(group=group)

    def add_rmsnorm(self, partial: torch.Tensor, x: torch.Tensor, weight: torch.Tensor,
                    eps: float) -> torch.Tensor:
        """``x += all_reduce(partial)`` (in place) and returns ``rmsnorm(x) * weight``;
        ``partial``, ``x`` fp16 ``[rows, hidden]``, rows <= max_rows."""
        if partial.shape != x.shape or x.dim() != 2 or x.size(1) != self.hidden:
            raise RuntimeError(f"nvlink all-reduce: expected [rows, {self.hidden}] tensors")
        for t in (partial, x, weight):
            if not (t.is_cuda and t.is_contiguous() and t.dtype == torch.float16):
                raise RuntimeError("nvlink all-reduce: fp16 contiguous CUDA tensors required")
        y = torch.empty_like(x)
        st = torch.cuda.current_stream(x.device)
        _lib.check(_LIB.qx_nvlink_ar_add_rmsnorm(self._ctx, partial.data_ptr(), x.data_ptr(),
                                                 weight.data_ptr(), y.data_ptr(), x.size(0),
                                                 float(eps), st.cuda_stream), "nvlink_ar_add_rmsnorm")
        return y

    def close(self) -> None:
        if self._ctx:
            _lib.check(_LIB.qx_nvlink_ar_destroy(self._ctx), "nvlink_ar_destroy")
            self._ctx = None
