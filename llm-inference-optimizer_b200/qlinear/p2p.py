"""NVLink peer-memory exchanges for column-sharded layers: the lm_head's
argmax (``PeerExchange``) and the all-gather of the outputs (``PeerGather``).

Each rank of the node allocates one exchange buffer in libqlinear, shares its
CUDA IPC handle with the other ranks over the process group (a one-time
host-side exchange) and opens theirs.  ``PeerExchange.argmax`` then runs
``ql_argmax_exchange_f16``: one kernel per rank that reduces the rank's logit
shard to per-row keys, stores them straight into every rank's buffer over
NVLink, waits (bounded) for the other ranks' keys and writes the global
argmax column — no NCCL call and no gather of the logits.
``PeerGather.gather`` runs ``ql_allgather_f16`` on buffers of its own: the
rank's output columns go to every peer by plain stores, a flag per rank and
call says they are complete, and every rank copies the peers' columns into
its output — the all-gather of a sharded layer without NCCL.

The reference has no multi-GPU code; this is the B200 build's exchange for
the column-sharded greedy head (its argmax: src/engine/paged_engine.py:146-147)
and for the full outputs of a column-sharded layer.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib
from .kernels._launch import default_flags, dtype_code, ld, on_device, ptr


class _PeerBuffers:
    """One device buffer per rank of the node, shared through CUDA IPC.

    Collective: every rank allocates its own (zero-filled) buffer of `nbytes`,
    the 64-byte IPC handles are exchanged once over the process group, and
    each rank opens the others'.  ``peers`` is the ctypes array of every
    rank's buffer as seen from this rank (peers[rank] = own); ``close``
    synchronises the ranks before the buffers go away."""

    def __init__(self, rank: int, world: int, nbytes: int, group: Optional[dist.ProcessGroup]):
        lib = _lib.load()
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device("cuda", torch.cuda.current_device())
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
        self.peers = (ctypes.c_void_p * world)(*ptrs)

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
        nbytes = lib.ql_xchg_buffer_bytes(world, max_m)
        if nbytes == 0:
            raise ValueError(f"bad exchange size (world {world}, max_m {max_m})")
        self._bufs = _PeerBuffers(rank, world, nbytes, group)
        self.device = self._bufs.device
        self._peers = self._bufs.peers

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

    def linear_argmax(self, x: torch.Tensor, module, col_offset: int) -> Optional[torch.Tensor]:
        """Global argmax column of every row of ``module(x)`` (this rank's
        column shard starting at `col_offset`) in ONE launch: the decode
        kernel reduces its fp16-rounded outputs to keys in its epilogue and
        its last CTA runs the exchange — the logits are never written.
        Returns None (nothing launched) for shapes the fused kernel does not
        take (more than 8 rows, K-split plans, tensor-core shapes, unaligned
        operands); the caller then runs the linear and ``argmax``."""
        from .quantization.int4 import QuantizedLinearInt4
        from .quantization.int8 import QuantizedLinearInt8
        assert x.is_cuda and x.dtype == torch.float16
        K = module.in_features
        x2 = x.reshape(-1, K)
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        M, N = x2.shape[0], module.out_features
        if not 1 <= M <= self.max_m:
            return None
        lib = _lib.load()
        wbits = 4 if isinstance(module, QuantizedLinearInt4) else 8 if isinstance(module, QuantizedLinearInt8) else 0
        if wbits == 0 or not lib.ql_linear_argmax_supported(wbits, M, N, K):
            return None
        out = torch.empty(M, dtype=torch.int64, device=x.device)
        bias = module.bias
        bias_dt = dtype_code(bias.dtype) if bias is not None else 0
        with on_device(x.device):
            stream = torch.cuda.current_stream(x.device).cuda_stream
            if wbits == 4:
                w, sc = module.weight_packed, module.scales
                st = lib.ql_w4a16_linear_argmax(
                    ptr(x2), _lib.QL_DTYPE_F16, ptr(w), module.layout, ptr(sc), ptr(bias), bias_dt, M, N, K,
                    ld(x2, K), ld(w, K // 2), ld(sc, N), col_offset, self.rank, self.world, self.max_m,
                    self._peers, ptr(out), default_flags(), stream)
            else:
                w, sc = module.weight_q, module.scale
                st = lib.ql_w8a16_linear_argmax(
                    ptr(x2), _lib.QL_DTYPE_F16, ptr(w), ptr(sc), dtype_code(sc.dtype), ptr(bias), bias_dt, M, N,
                    K, ld(x2, K), ld(w, K), col_offset, self.rank, self.world, self.max_m, self._peers, ptr(out),
                    default_flags(), stream)
        if st == _lib.QL_ERR_UNSUPPORTED:
            return None
        _lib.check(st)
        return out

    def close(self) -> None:
        self._bufs.close()


class PeerGather:
    """All-gather of a column-sharded layer's fp16 outputs over NVLink.

    Every rank holds the columns [r*block, min(ng, (r+1)*block)) of each of
    the `groups` blocks of ng = n_cols / groups output columns (the layout of
    ``ShardedQuantizedLinear``).  ``gather`` runs ``ql_allgather_f16``: one
    kernel per rank that stores the rank's columns into every peer's gather
    buffer, signals, waits (bounded) for the peers' columns and copies them
    into the caller's output — no NCCL call.  Collective like
    ``PeerExchange``: every rank constructs it with the same arguments, calls
    ``gather`` in the same order with the same shapes, and calls ``close``."""

    def __init__(self, rank: int, world: int, max_m: int, n_cols: int,
                 group: Optional[dist.ProcessGroup] = None):
        if not 1 <= world <= _lib.QL_XCHG_MAX_RANKS:
            raise ValueError(f"world size {world} outside 1..{_lib.QL_XCHG_MAX_RANKS}")
        nbytes = _lib.load().ql_gather_buffer_bytes(max_m, n_cols)
        if nbytes == 0:
            raise ValueError(f"bad gather size (max_m {max_m}, n_cols {n_cols})")
        self.rank, self.world, self.max_m, self.n_cols = rank, world, max_m, n_cols
        self._bufs = _PeerBuffers(rank, world, nbytes, group)
        self.device = self._bufs.device

    def gather(self, out: torch.Tensor, block: int, groups: int = 1, src: Optional[torch.Tensor] = None) -> None:
        """Complete `out` [M, n_cols] (fp16, unit inner stride) in place on
        every rank.  This rank's columns are already in `out` (src None) or
        in `src` [M, groups*w], gate columns then up columns for groups 2."""
        assert out.is_cuda and out.dtype == torch.float16 and out.dim() == 2 and out.shape[1] == self.n_cols
        assert out.stride(-1) == 1, "out must have unit stride along the columns"
        M = out.shape[0]
        assert 1 <= M <= self.max_m, f"batch {M} exceeds the gather's max_m {self.max_m}"
        lds = 0
        if src is not None:
            assert src.dtype == torch.float16 and src.device == out.device and src.dim() == 2 and src.shape[0] == M
            if src.stride(-1) != 1:
                src = src.contiguous()
            lds = ld(src, src.shape[1])
        with on_device(out.device):
            stream = torch.cuda.current_stream(out.device).cuda_stream
            _lib.check(_lib.load().ql_allgather_f16(
                ptr(src), lds, out.data_ptr(), ld(out, self.n_cols), M, self.n_cols, groups, block, self.rank,
                self.world, self.max_m, self._bufs.peers, default_flags(), stream))

    def close(self) -> None:
        self._bufs.close()


__all__ = ["PeerExchange", "PeerGather"]
