"""W4A16 module: 4-bit weights in groups of 128 along K, fp16 group scales.

Stands in for the reference's ``src/quantization/int4.py`` without any change
visible to its callers.  Kept as the reference has them, because the engines,
``state_dict`` and the reference's tests depend on them:

* the class name and constructor ``(packed, scales, bias)``, and the buffer
  names ``weight_packed`` (uint8 [N, K/2]), ``scales`` (fp16 [K/128, N]) and
  ``bias`` (``int4.py:29-35``);
* ``from_linear``'s arithmetic (``int4.py:37-49``), bit for bit: the group
  scale is max|w| / 7 floored at 1e-5 and rounded to fp16 *before* the
  weights are divided by it; codes are round-half-even, clamped, offset by 8;
* ``dequantized_weight`` / ``num_bytes`` / ``forward`` (``:51-62``) and
  ``quantize_model_int4``'s return value (``:72-97``).

``forward`` runs the sm_100a kernels of libqlinear.so through
``w4a16_linear``.  Two keyword arguments, both defaulting to the reference's
format, select the variant that the benchmark's config 1 describes: codes down to
-8 (``qmin=-8``) and adjacent-pair nibbles (``layout=LAYOUT_ADJACENT``).
"""
from typing import Optional

import torch
import torch.nn as nn

from ..kernels.w4a16_matmul import (
    GROUP_SIZE, LAYOUT_ADJACENT, LAYOUT_SPLIT_HALF, dequantize_int4, pack_int4, pack_int4_adjacent,
    w4a16_linear, w4a16_quantize_cuda,
)
from ._replace import replace_linears, tensor_bytes


def _quantize_groups_torch(weight: torch.Tensor, qmin: int, layout: int):
    """PyTorch form of the group quantizer (any device or dtype): returns
    (packed uint8 [N, K/2], scales fp16 [K/128, N])."""
    n_out, n_in = weight.shape
    groups = weight.float().reshape(n_out, n_in // GROUP_SIZE, GROUP_SIZE)
    step16 = torch.clamp(groups.abs().amax(dim=-1) / 7.0, min=1e-5).to(torch.float16)
    codes = torch.round(groups / step16.float().unsqueeze(-1)).clamp(qmin, 7) + 8
    codes = codes.to(torch.uint8).reshape(n_out, n_in)
    pack = pack_int4 if layout == LAYOUT_SPLIT_HALF else pack_int4_adjacent
    return pack(codes), step16.transpose(0, 1).contiguous()


class QuantizedLinearInt4(nn.Module):
    """Inference-only replacement for an ``nn.Linear`` whose weight is held as
    packed 4-bit codes with one fp16 scale per 128 inputs of each output.
    Everything is a registered buffer (no Parameters), so ``state_dict``
    carries the packed form."""

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor, bias: Optional[torch.Tensor],
                 layout: int = LAYOUT_SPLIT_HALF):
        super().__init__()
        self.register_buffer("weight_packed", packed)
        self.register_buffer("scales", scales)
        self.register_buffer("bias", bias)
        self.out_features = packed.shape[0]
        self.in_features = 2 * packed.shape[1]
        self.layout = layout

    @classmethod
    def from_linear(cls, linear: nn.Linear, qmin: int = -7,
                    layout: int = LAYOUT_SPLIT_HALF) -> "QuantizedLinearInt4":
        """Quantize ``linear`` group by group (codes in [qmin, 7] plus 8).  A
        CUDA fp16 weight is quantized by the device kernel, which yields the
        same bytes as the PyTorch form used for every other input."""
        weight = linear.weight.detach()
        N, K = weight.shape
        assert K % GROUP_SIZE == 0, f"in_features {K} must be a multiple of {GROUP_SIZE}"
        if weight.is_cuda and weight.dtype == torch.float16 and N > 0:
            packed, scales = w4a16_quantize_cuda(weight, qmin=qmin, layout=layout)
        else:
            packed, scales = _quantize_groups_torch(weight, qmin, layout)
        bias = None if linear.bias is None else linear.bias.detach().clone()
        return cls(packed, scales, bias, layout=layout)

    def dequantized_weight(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """The weight the kernels multiply by, as a dense [N, K] tensor."""
        return dequantize_int4(self.weight_packed, self.scales, self.layout).to(dtype)

    def num_bytes(self) -> int:
        """Bytes held on the device: packed codes, group scales and bias."""
        return tensor_bytes(self.weight_packed, self.scales, self.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return w4a16_linear(x, self.weight_packed, self.scales, self.bias, layout=self.layout)


def quantize_model_int4(model: nn.Module) -> dict:
    """Put a ``QuantizedLinearInt4`` in place of every linear projection of the
    decoder layers (``model.model.layers``); see ``replace_linears`` for the
    returned statistics."""
    return replace_linears(model, QuantizedLinearInt4.from_linear)


__all__ = ["QuantizedLinearInt4", "quantize_model_int4", "LAYOUT_SPLIT_HALF", "LAYOUT_ADJACENT"]
