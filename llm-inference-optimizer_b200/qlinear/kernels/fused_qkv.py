"""Fused q/k/v projections: one launch, three outputs.

The reference's attention calls q_proj, k_proj and v_proj on the same hidden
states (src/engine/paged_engine.py:98-105; HF Qwen2Attention), three small
launches — k/v (1536 -> 256) are too small to load the GPU alone.  Here the
three quantized weights are stacked into one [Nq + Nk + Nv, K] module and run
as one linear; q, k and v are column views of its [M, Nq + Nk + Nv] output.

``fuse_attention_qkv(model)`` keeps the attention code unchanged: q_proj,
k_proj and v_proj become thin views on one shared module, which computes
all three on the first of the three calls and hands out the other two
slices for the same input tensor.
"""
from __future__ import annotations

import weakref
from typing import Optional

import torch
import torch.nn as nn

from ..quantization.int4 import QuantizedLinearInt4
from ..quantization.int8 import QuantizedLinearInt8


def stack_rows(mods) -> nn.Module:
    """One quantized module with the rows of `mods` in order (quantization is
    row-local, so this equals quantizing the stacked fp16 weight).  Missing
    biases become zeros when any module has one."""
    dev = None
    if all(isinstance(m, QuantizedLinearInt4) for m in mods):
        assert len({m.layout for m in mods}) == 1
        dev = mods[0].scales.device
    elif all(isinstance(m, QuantizedLinearInt8) for m in mods):
        dev = mods[0].scale.device
    else:
        raise TypeError("modules must share one quantized format")
    bias = None
    if any(m.bias is not None for m in mods):
        bias = torch.cat([m.bias if m.bias is not None else torch.zeros(m.out_features, dtype=torch.float16,
                                                                         device=dev) for m in mods])
    if isinstance(mods[0], QuantizedLinearInt4):
        return QuantizedLinearInt4(torch.cat([m.weight_packed for m in mods]).contiguous(),
                                   torch.cat([m.scales for m in mods], dim=1).contiguous(), bias,
                                   layout=mods[0].layout)
    return QuantizedLinearInt8(torch.cat([m.weight_q for m in mods]).contiguous(),
                               torch.cat([m.scale for m in mods]).contiguous(), bias)


def _version(x: torch.Tensor) -> int:
    try:
        return x._version
    except RuntimeError:            # inference tensors have no version counter (and are immutable)
        return 0


class QuantizedQKV(nn.Module):
    """q, k, v = column views of one stacked quantized linear."""

    def __init__(self, stacked: nn.Module, sizes):
        super().__init__()
        assert sum(sizes) == stacked.out_features
        self.stacked = stacked
        self.sizes = tuple(int(s) for s in sizes)
        self.in_features = stacked.in_features
        self._last_x: Optional[weakref.ref] = None
        self._last_version = -1
        self._last_out = None

    @classmethod
    def from_quantized(cls, q: nn.Module, k: nn.Module, v: nn.Module) -> "QuantizedQKV":
        return cls(stack_rows([q, k, v]), (q.out_features, k.out_features, v.out_features))

    def forward(self, x: torch.Tensor):
        return torch.split(self.stacked(x), self.sizes, dim=-1)

    def part(self, x: torch.Tensor, index: int) -> torch.Tensor:
        """Projection `index` (0 q, 1 k, 2 v) of x; the three come from one
        launch when called on the same tensor one after another."""
        version = _version(x)
        hit = self._last_x is not None and self._last_x() is x and version == self._last_version
        if not hit:
            self._last_out = self.forward(x)
            self._last_x = weakref.ref(x)
            self._last_version = version
        return self._last_out[index]


class _QKVView(nn.Module):
    """Stands in for q_proj / k_proj / v_proj."""

    def __init__(self, owner: QuantizedQKV, index: int):
        super().__init__()
        self.owner = [owner]            # not a submodule: the owner is registered once, on the attention
        self.index = index
        self.in_features = owner.in_features
        self.out_features = owner.sizes[index]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.owner[0].part(x, self.index)


def fuse_attention_qkv(model: nn.Module) -> int:
    """Stack q/k/v of every attention under model.model.layers whose three
    projections are quantized alike.  Returns the number fused."""
    fused = 0
    for layer in model.model.layers:
        attn = getattr(layer, "self_attn", None)
        if attn is None or not all(hasattr(attn, n) for n in ("q_proj", "k_proj", "v_proj")):
            continue
        q, k, v = attn.q_proj, attn.k_proj, attn.v_proj
        kinds = {type(m) for m in (q, k, v)}
        if len(kinds) != 1 or kinds.pop() not in (QuantizedLinearInt4, QuantizedLinearInt8):
            continue
        qkv = QuantizedQKV.from_quantized(q, k, v)
        attn.qkv_proj = qkv
        attn.q_proj, attn.k_proj, attn.v_proj = _QKVView(qkv, 0), _QKVView(qkv, 1), _QKVView(qkv, 2)
        fused += 1
    return fused


__all__ = ["stack_rows", "QuantizedQKV", "fuse_attention_qkv"]
