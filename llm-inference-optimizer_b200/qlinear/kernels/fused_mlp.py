"""Fused gate+up projection with the SwiGLU activation (libqlinear).

The reference's Qwen2 MLP computes ``down_proj(act_fn(gate_proj(x)) *
up_proj(x))`` (HF Qwen2MLP, SiLU activation) with two quantized projections
and, in its fused variant, a separate elementwise kernel
(src/kernels/fused_swiglu_triton.py:21-53, src/engine/fused_norm_activation_patch.py:60-64).
Here gate and up are one quantized weight of 2N stacked rows and
``gate_up_silu`` returns ``silu(x @ gate^T) * (x @ up^T)`` from one call: in
the decode kernel's epilogue without storing the [M, 2N] product, else
through the workspace and an elementwise kernel.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .. import _lib
from ..quantization.int4 import QuantizedLinearInt4
from ..quantization.int8 import QuantizedLinearInt8
from ._launch import default_flags, dtype_code, ld, on_device, ptr, workspace


def gate_up_silu(x: torch.Tensor, stacked: nn.Module) -> torch.Tensor:
    """x (..., K) fp16; `stacked` a QuantizedLinearInt4/Int8 with 2N output
    rows (gate then up).  Returns (..., N) fp16."""
    assert x.is_cuda and x.dtype == torch.float16
    N2, K = stacked.out_features, stacked.in_features
    assert N2 % 2 == 0, "stacked gate+up needs an even number of rows"
    assert x.shape[-1] == K, f"x last dim {x.shape[-1]} != weight in_features {K}"
    N = N2 // 2
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=torch.float16, device=x.device)
    if M == 0:
        return out.reshape(*x.shape[:-1], N)
    lib = _lib.load()
    bias = stacked.bias
    with on_device(x.device):
        stream = torch.cuda.current_stream(x.device)
        if isinstance(stacked, QuantizedLinearInt4):
            ws = workspace(x.device, stream, lib.ql_w4a16_gate_up_silu_workspace_size(M, N, K))
            st = lib.ql_w4a16_gate_up_silu(
                ptr(x2), _lib.QL_DTYPE_F16, ptr(stacked.weight_packed), stacked.layout, ptr(stacked.scales),
                ptr(bias), dtype_code(bias.dtype) if bias is not None else 0, ptr(out), M, N, K,
                ld(x2, K), ld(stacked.weight_packed, K // 2), ld(stacked.scales, N2), ld(out, N),
                ptr(ws), ws.numel() if ws is not None else 0, default_flags(), stream.cuda_stream)
        elif isinstance(stacked, QuantizedLinearInt8):
            ws = workspace(x.device, stream, lib.ql_w8a16_gate_up_silu_workspace_size(M, N, K))
            st = lib.ql_w8a16_gate_up_silu(
                ptr(x2), _lib.QL_DTYPE_F16, ptr(stacked.weight_q), ptr(stacked.scale),
                dtype_code(stacked.scale.dtype), ptr(bias), dtype_code(bias.dtype) if bias is not None else 0,
                ptr(out), M, N, K, ld(x2, K), ld(stacked.weight_q, K), ld(out, N),
                ptr(ws), ws.numel() if ws is not None else 0, default_flags(), stream.cuda_stream)
        else:
            raise TypeError(f"expected QuantizedLinearInt4/Int8, got {type(stacked).__name__}")
    _lib.check(st)
    return out.reshape(*x.shape[:-1], N)


def stack_gate_up(gate: nn.Module, up: nn.Module) -> nn.Module:
    """One quantized module with gate's rows then up's rows (quantization is
    row-local, so this equals quantizing the stacked fp16 weight)."""
    from .fused_qkv import stack_rows
    return stack_rows([gate, up])


class QuantizedGateUpSiLU(nn.Module):
    """silu(gate(x)) * up(x) from one stacked quantized weight."""

    def __init__(self, stacked: nn.Module):
        super().__init__()
        self.stacked = stacked
        self.in_features = stacked.in_features
        self.out_features = stacked.out_features // 2

    @classmethod
    def from_quantized(cls, gate: nn.Module, up: nn.Module) -> "QuantizedGateUpSiLU":
        return cls(stack_gate_up(gate, up))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return gate_up_silu(x, self.stacked)


def fuse_mlp_gate_up(model: nn.Module) -> int:
    """For every MLP under model.model.layers whose gate_proj / up_proj are
    quantized and whose activation is SiLU, compute act(gate) * up with one
    fused call (down_proj unchanged).  Returns the number of MLPs fused; the
    separate gate/up modules are dropped (their buffers live in the stacked one)."""
    fused = 0
    for layer in model.model.layers:
        mlp = getattr(layer, "mlp", None)
        if mlp is None or not hasattr(mlp, "gate_proj") or not hasattr(mlp, "up_proj"):
            continue
        act = getattr(mlp, "act_fn", None)
        if not isinstance(act, nn.SiLU) and type(act).__name__ not in ("SiLU", "SiLUActivation"):
            continue
        if not isinstance(mlp.gate_proj, (QuantizedLinearInt4, QuantizedLinearInt8)):
            continue
        gate_up = QuantizedGateUpSiLU.from_quantized(mlp.gate_proj, mlp.up_proj)
        mlp.gate_up_silu = gate_up
        del mlp.gate_proj, mlp.up_proj
        mlp.forward = (lambda m: lambda x: m.down_proj(m.gate_up_silu(x)))(mlp)
        fused += 1
    return fused


__all__ = ["gate_up_silu", "stack_gate_up", "QuantizedGateUpSiLU", "fuse_mlp_gate_up"]
