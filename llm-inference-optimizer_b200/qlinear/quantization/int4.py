"""INT4 group-wise weight quantization of a loaded model (W4A16, g=128).

Drop-in for src/quantization/int4.py of the reference: the class, buffer
names (``weight_packed``, ``scales``, ``bias``), ``from_linear`` (:37-49),
``dequantized_weight`` (:51-52), ``num_bytes`` (:54-59), ``forward``
(:61-62) and ``quantize_model_int4`` (:72-97) keep their behaviour.
Plain round-to-nearest with max-abs group scales, as in the reference.

Two optional keyword arguments select the variant format (q in [-8, 7],
adjacent-pair nibbles); their defaults are the reference's format.
"""
import gc
from typing import Optional

import torch
import torch.nn as nn

from ..kernels.w4a16_matmul import (
    GROUP_SIZE, LAYOUT_SPLIT_HALF, LAYOUT_ADJACENT, dequantize_int4, pack_int4,
    pack_int4_adjacent, w4a16_linear, w4a16_quantize_cuda,
)


class QuantizedLinearInt4(nn.Module):
    """Drop-in nn.Linear replacement: packed 4-bit weights, fp16 group
    scales of shape (K//128, N), optional bias.  Inference-only buffers."""

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor, bias: Optional[torch.Tensor],
                 layout: int = LAYOUT_SPLIT_HALF):
        super().__init__()
        self.register_buffer("weight_packed", packed)
        self.register_buffer("scales", scales)
        self.register_buffer("bias", bias)
        self.out_features = packed.shape[0]
        self.in_features = packed.shape[1] * 2
        self.layout = layout

    @classmethod
    def from_linear(cls, linear: nn.Linear, qmin: int = -7,
                    layout: int = LAYOUT_SPLIT_HALF) -> "QuantizedLinearInt4":
        """scale = max(|W[n, group]|)/7 (>= 1e-5) stored fp16; q =
        round-half-even(W / float(scale16)) clamped to [qmin, 7]; nibble q+8.
        On a CUDA fp16 weight the device quantizer produces the same bits as
        the PyTorch expression used otherwise."""
        wt = linear.weight.detach()
        N, K = wt.shape
        assert K % GROUP_SIZE == 0, f"in_features {K} must be a multiple of {GROUP_SIZE}"
        if wt.is_cuda and wt.dtype == torch.float16 and N > 0:
            packed, scales = w4a16_quantize_cuda(wt, qmin=qmin, layout=layout)
        else:
            w = wt.float()                                              # (N, K)
            wg = w.reshape(N, K // GROUP_SIZE, GROUP_SIZE)
            scale = (wg.abs().amax(dim=2) / 7.0).clamp(min=1e-5)          # (N, G)
            scale16 = scale.half()                                        # what is actually stored
            q = torch.round(wg / scale16.float()[:, :, None]).clamp(qmin, 7) + 8
            q = q.reshape(N, K).to(torch.uint8)
            packed = pack_int4(q) if layout == LAYOUT_SPLIT_HALF else pack_int4_adjacent(q)
            scales = scale16.t().contiguous()                             # (G, N)
        bias = linear.bias.detach().clone() if linear.bias is not None else None
        return cls(packed, scales, bias, layout=layout)

    def dequantized_weight(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return dequantize_int4(self.weight_packed, self.scales, self.layout).to(dtype)

    def num_bytes(self) -> int:
        total = self.weight_packed.numel() * self.weight_packed.element_size()
        total += self.scales.numel() * self.scales.element_size()
        if self.bias is not None:
            total += self.bias.numel() * self.bias.element_size()
        return total

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return w4a16_linear(x, self.weight_packed, self.scales, self.bias, layout=self.layout)


def _linear_bytes(linear: nn.Linear) -> int:
    total = linear.weight.numel() * linear.weight.element_size()
    if linear.bias is not None:
        total += linear.bias.numel() * linear.bias.element_size()
    return total


def quantize_model_int4(model: nn.Module) -> dict:
    """Replaces every nn.Linear inside model.model.layers with a
    QuantizedLinearInt4, in place.  Returns stats; callers should check
    layers_quantized > 0."""
    layers_quantized = 0
    bytes_before = 0
    bytes_after = 0

    for parent in list(model.model.layers.modules()):
        for child_name, child in list(parent.named_children()):
            if isinstance(child, nn.Linear):
                bytes_before += _linear_bytes(child)
                quantized = QuantizedLinearInt4.from_linear(child)
                bytes_after += quantized.num_bytes()
                setattr(parent, child_name, quantized)
                layers_quantized += 1

    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.empty_cache()

    return {
        "layers_quantized": layers_quantized,
        "bytes_before": bytes_before,
        "bytes_after": bytes_after,
    }


__all__ = ["QuantizedLinearInt4", "quantize_model_int4", "LAYOUT_SPLIT_HALF", "LAYOUT_ADJACENT"]
