"""Host-side plumbing shared by the linear wrappers: device/stream
selection, the per-stream split-K workspace and the launch flags."""
from __future__ import annotations

import os
import threading

import torch

from .. import _lib

_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_MIN_WS = 1 << 20


def default_flags() -> int:
    """Programmatic dependent launch is on unless QLINEAR_PDL=0: the kernels
    stream their (static) weights while the previous kernel finishes."""
    return 0 if os.environ.get("QLINEAR_PDL", "1") == "0" else _lib.QL_FLAG_PDL


def workspace(device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> torch.Tensor | None:
    """Zero-filled scratch for split-K, one per (device, stream).

    The kernels leave it zero-filled after every call, so it is created once
    and reused; calls on one stream are ordered, so they never overlap.  A
    first (eager) call sizes it, which keeps later CUDA-graph captures free
    of allocations."""
    if nbytes == 0:
        return None
    key = (device.index, stream.cuda_stream)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        with _ws_lock:
            buf = _workspaces.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(_MIN_WS, 1 << (int(nbytes) - 1).bit_length())
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
                _workspaces[key] = buf
    return buf


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def ld(t: torch.Tensor, row_len: int) -> int:
    """Leading dimension (elements between rows) of a 2-D tensor with unit
    inner stride.  A single-row tensor may report any row stride (torch
    treats size-1 dims as contiguous whatever their stride), so its row
    length is used instead."""
    return t.stride(0) if t.shape[0] > 1 else row_len


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float16:
        return _lib.QL_DTYPE_F16
    if dt == torch.float32:
        return _lib.QL_DTYPE_F32
    if dt == torch.bfloat16:
        return _lib.QL_DTYPE_BF16
    raise TypeError(f"unsupported dtype {dt}")


class on_device:
    """Make `device` current for the C call (the ABI uses the current device)."""

    def __init__(self, device: torch.device):
        self.idx = device.index
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False
