"""NVLink peer-memory exchange for the sharded lm_head's argmax.

Each rank of the node allocates one exchange buffer in libqlinear, shares its
CUDA IPC handle with the other ranks over the process group (a one-time
host-side exchange) and opens theirs.  ``PeerExchange.argmax`` then runs
``ql_argmax_exchange_f16``: one kernel per rank that reduces the rank's logit
shard to per-row keys, stores them straight into every rank's buffer over
NVLink, waits (bounded) for the other ranks' keys and writes the global
argmax column — no NCCL call and no gather of the logits.

The reference has no multi-GPU code; this is the B200 build's exchange for
the column-sharded greedy head (its argmax: src/engine/paged_engine.py:146-147).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib


class PeerExchange:
    """Exchange buffers of `world` ranks (one process per GPU, one node).

    Collective: every rank constructs it (same world, max_m), calls
    ``argmax`` in the same order, and calls ``close`` (which synchronises the
    ranks before the buffers go away)."""

    def __init__(self, rank: int, world: int, max_m: int, group: Optional[dist.ProcessGroup] = None):
        if not 1 <= world <= _lib.QL_XCHG_MAX_RANKS:
            raise ValueError(f"world size {world} outside 1..{_lib.QL_XCHG_MAX_RANKS}")
        lib = _lib.load()
        self.rank, self.world, self.max_m, self.group = rank, world, max_m, group
        self.device = torch.device("cuda", torch.cuda.current_device())
        nbytes = lib.ql_xchg_buffer_bytes(world, max_m)
        if nbytes == 0:
            raise ValueError(f"bad exchange size (world {world}, max_m {max_m})")
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        _lib.check(lib.ql_xchg_alloc(nbytes, ctypes.byref(own), handle))
        self._own = own.value
        handles = [bytes(handle)] * world
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        ptrs = []
        for q in range(world):
            if q == rank:
                ptrs.append(self._own)
                continue
            peer = ctypes.c_void_p()
            buf = (ctypes.c_char * 64).from_buffer_copy(handles[q])
            _lib.check(lib.ql_xchg_open(buf, ctypes.byref(peer)))
            self._opened.append(peer.value)
            ptrs.append(peer.value)
        self._peers = (ctypes.c_void_p * world)(*ptrs)

    def argmax(self, logits: torch.Tensor, col_offset: int) -> torch.Tensor:
        """Global argmax column of every row; `logits` is this rank's
        [M, N_local] fp16 shard starting at column `col_offset`."""
        assert logits.is_cuda and logits.dtype == torch.float16 and logits.dim() == 2
        if logits.stride(-1) != 1:
            logits = logits.contiguous()
        M, N = logits.shape
        assert 1 <= M <= self.max_m, f"batch {M} exceeds the exchange's max_m {self.max_m}"
        out = torch.empty(M, dtype=torch.int64, device=logits.device)
        stream = torch.cuda.current_stream(logits.device)
        ldx = logits.stride(0) if M > 1 else N
        _lib.check(_lib.load().ql_argmax_exchange_f16(
            logits.data_ptr(), M, N, ldx, col_offset, self.rank, self.world, self.max_m, self._peers,
            out.data_ptr(), stream.cuda_stream))
        return out

    def close(self) -> None:
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)        # nobody writes into a buffer after this
        lib = _lib.load()
        for p in self._opened:
            lib.ql_xchg_close(p)
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)        # peers have unmapped ours
        lib.ql_xchg_free(self._own)
        self._own = None


__all__ = ["PeerExchange"]
