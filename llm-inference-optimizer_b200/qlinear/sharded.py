"""Column-sharded quantized linear layers across the GPUs of one node.

Large-N layers (the lm_head, a fused gate+up projection) are split by
output column: rank p of P holds the weight rows (output columns)
[p*Np, (p+1)*Np) with Np = ceil(N/P) (the last shard may be short), runs the
unchanged single-GPU quantized linear on its rows, and one all-gather of the
fp16 outputs over NVLink rebuilds the full [M, N] result on every rank:
NCCL through ``torch.distributed`` by default, or, with a
``qlinear.p2p.PeerGather`` attached as ``gatherer``, one kernel per rank that
stores the columns into the peers' memory itself.

``groups`` handles layers whose output is a concatenation of equally sized
blocks that must be sharded alike — a fused gate+up projection [gate; up]
with groups=2 gives every rank the same column range of gate and of up, so
the pair stays local (a SwiGLU epilogue needs no exchange) and the gathered
output is reassembled as [gate | up].

The reference has no multi-GPU code (its README lists multi-GPU as future
work); this module is the B200 build's addition for the sharded
configuration of the quantized-linear path.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from .kernels.argmax import argmax_keys, combine_keys, key_columns
from .kernels.w4a16_matmul import GROUP_SIZE, w4a16_linear
from .kernels.w8a16_matmul import w8a16_linear
from .quantization.int4 import QuantizedLinearInt4
from .quantization.int8 import QuantizedLinearInt8


def shard_bounds(n: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of the output columns rank `rank` owns (Np = ceil(n/world))."""
    per = (n + world - 1) // world
    lo = min(rank * per, n)
    return lo, min(lo + per, n)


def _group_rows(t: Optional[torch.Tensor], groups: int, rank: int, world: int) -> Optional[torch.Tensor]:
    """Rows of each of `groups` equal blocks that `rank` owns, concatenated."""
    if t is None:
        return None
    n = t.shape[0] // groups
    lo, hi = shard_bounds(n, rank, world)
    return torch.cat([t[g * n + lo:g * n + hi] for g in range(groups)], dim=0).contiguous()


def _group_cols(t: torch.Tensor, groups: int, rank: int, world: int) -> torch.Tensor:
    n = t.shape[1] // groups
    lo, hi = shard_bounds(n, rank, world)
    return torch.cat([t[:, g * n + lo:g * n + hi] for g in range(groups)], dim=1).contiguous()


def local_linear_cuda(module: nn.Module, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The shard's own compute: the single-GPU B200 kernels (into `out`, a
    [M, N_local] view with unit inner stride, when given)."""
    if isinstance(module, QuantizedLinearInt4):
        return w4a16_linear(x, module.weight_packed, module.scales, module.bias, layout=module.layout, out=out)
    return w8a16_linear(x, module.weight_q, module.scale, module.bias, out=out)


class ShardedQuantizedLinear(nn.Module):
    """One rank's shard of a column-sharded QuantizedLinearInt4/Int8.

    forward(x[..., K]) -> [..., N] (the full output on every rank).
    """

    def __init__(self, local: nn.Module, out_features: int, rank: int, world: int, groups: int = 1,
                 group: Optional[dist.ProcessGroup] = None,
                 local_fn: Callable[[nn.Module, torch.Tensor], torch.Tensor] = local_linear_cuda,
                 key_fn: Callable[[torch.Tensor, int], torch.Tensor] = argmax_keys):
        super().__init__()
        self.local = local
        self.out_features = out_features
        self.in_features = local.in_features
        self.rank, self.world, self.groups = rank, world, groups
        self.group = group
        self.local_fn = local_fn
        self.key_fn = key_fn
        self.exchange = None          # optional qlinear.p2p.PeerExchange for argmax
        self.gatherer = None          # optional qlinear.p2p.PeerGather for forward
        n = out_features // groups
        self.block = (n + world - 1) // world          # padded per-rank width of one group
        self.widths = [shard_bounds(n, r, world)[1] - shard_bounds(n, r, world)[0] for r in range(world)]

    # ----------------------------------------------------------- builders
    @classmethod
    def from_quantized(cls, q: nn.Module, rank: int, world: int, groups: int = 1,
                       group: Optional[dist.ProcessGroup] = None, **kw) -> "ShardedQuantizedLinear":
        """Cut rank `rank`'s rows out of a full quantized module."""
        N = q.out_features
        assert N % groups == 0, f"out_features {N} not divisible into {groups} groups"
        if isinstance(q, QuantizedLinearInt4):
            local = QuantizedLinearInt4(_group_rows(q.weight_packed, groups, rank, world),
                                        _group_cols(q.scales, groups, rank, world),
                                        _group_rows(q.bias, groups, rank, world), layout=q.layout)
        elif isinstance(q, QuantizedLinearInt8):
            local = QuantizedLinearInt8(_group_rows(q.weight_q, groups, rank, world),
                                        _group_rows(q.scale, groups, rank, world),
                                        _group_rows(q.bias, groups, rank, world))
        else:
            raise TypeError(f"expected QuantizedLinearInt4/Int8, got {type(q).__name__}")
        return cls(local, N, rank, world, groups, group, **kw)

    @classmethod
    def from_linear(cls, linear: nn.Linear, wbits: int, rank: int, world: int, groups: int = 1,
                    group: Optional[dist.ProcessGroup] = None, **kw) -> "ShardedQuantizedLinear":
        """Quantize only this rank's rows of an fp16 nn.Linear (per-row int8
        and group-wise int4 quantization are row-local, so this equals
        sharding the fully quantized layer)."""
        w = _group_rows(linear.weight.detach(), groups, rank, world)
        b = _group_rows(linear.bias.detach(), groups, rank, world) if linear.bias is not None else None
        part = nn.Linear(w.shape[1], w.shape[0], bias=b is not None, device=w.device, dtype=w.dtype)
        with torch.no_grad():
            part.weight.copy_(w)
            if b is not None:
                part.bias.copy_(b)
        if wbits == 4:
            assert w.shape[1] % GROUP_SIZE == 0
            local = QuantizedLinearInt4.from_linear(part)
        else:
            local = QuantizedLinearInt8.from_linear(part)
        return cls(local, linear.out_features, rank, world, groups, group, **kw)

    # ------------------------------------------------------------ forward
    def local_forward(self, x2: torch.Tensor) -> torch.Tensor:
        """This rank's columns, padded to groups*block: [M, groups*block]."""
        y = self.local_fn(self.local, x2)
        mine = self.widths[self.rank]
        if mine == self.block:
            return y
        pad = torch.zeros((y.shape[0], self.groups * self.block), dtype=y.dtype, device=y.device)
        for g in range(self.groups):
            pad[:, g * self.block:g * self.block + mine] = y[:, g * mine:(g + 1) * mine]
        return pad

    def gather(self, y_local: torch.Tensor) -> torch.Tensor:
        """All-gather the ranks' padded shards and reassemble [M, N]."""
        M = y_local.shape[0]
        if self.world == 1:
            return y_local
        flat = y_local.contiguous().view(-1)
        buf = torch.empty(self.world * flat.numel(), dtype=y_local.dtype, device=y_local.device)
        dist.all_gather_into_tensor(buf, flat, group=self.group)   # rank-major concatenation
        # buf: [P, M, groups, block] -> [M, groups, P, block] -> trim padding
        full = buf.view(self.world, M, self.groups, self.block).permute(1, 2, 0, 3)
        if all(wd == self.block for wd in self.widths):
            return full.reshape(M, self.out_features)
        n = self.out_features // self.groups
        full = full.reshape(M, self.groups, self.world * self.block)[:, :, :n]
        return full.reshape(M, self.out_features)

    def argmax(self, x: torch.Tensor, fused: bool = True) -> torch.Tensor:
        """argmax over the full output row, without gathering the outputs.

        Each rank reduces its columns to one key per row (value, global
        column; ties to the smallest column, as torch.argmax), the ranks
        exchange the keys (8 bytes per row and rank) and every rank takes the
        max: with an attached PeerExchange in one kernel over NVLink (for
        decode-sized batches the shard's linear itself, whose epilogue makes
        the keys: one launch per rank and no logits), else through an NCCL
        all-gather.  Equals torch.argmax(self(x), dim=-1).  groups == 1 only;
        fused=False keeps the linear and the exchange as two launches."""
        assert self.groups == 1, "argmax is defined for a single output block"
        K = self.in_features
        x2 = x.reshape(-1, K)
        lo = shard_bounds(self.out_features, self.rank, self.world)[0]
        if fused and self.exchange is not None and self.local_fn is local_linear_cuda:
            ids = self.exchange.linear_argmax(x2, self.local, lo)
            if ids is not None:
                return ids.reshape(x.shape[:-1])
        y = self.local_fn(self.local, x2)                       # [M, widths[rank]]
        if self.exchange is not None:                           # one kernel, keys over NVLink
            return self.exchange.argmax(y, lo).reshape(x.shape[:-1])
        keys = self.key_fn(y, lo)                               # [M] int64 key bits
        if self.world > 1:
            buf = torch.empty(self.world * keys.numel(), dtype=keys.dtype, device=keys.device)
            dist.all_gather_into_tensor(buf, keys, group=self.group)
            keys = combine_keys(buf.view(self.world, -1), dim=0)
        return key_columns(keys).reshape(x.shape[:-1])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        K = self.in_features
        x2 = x.reshape(-1, K)
        M = x2.shape[0]
        g = self.gatherer
        if (g is not None and self.local_fn is local_linear_cuda and x2.dtype == torch.float16
                and 1 <= M <= g.max_m):
            # all-gather over NVLink peer memory: the shard's kernel writes
            # its columns straight into the full output (one block), or into
            # a [gate | up] staging tensor that the gather kernel spreads
            out = torch.empty((M, self.out_features), dtype=x2.dtype, device=x2.device)
            if self.groups == 1:
                lo, hi = shard_bounds(self.out_features, self.rank, self.world)
                if hi > lo:
                    local_linear_cuda(self.local, x2, out=out[:, lo:hi])
                g.gather(out, self.block)
            else:
                g.gather(out, self.block, self.groups, src=self.local_fn(self.local, x2))
            return out.reshape(*x.shape[:-1], self.out_features)
        out = self.gather(self.local_forward(x2))
        return out.reshape(*x.shape[:-1], self.out_features)
