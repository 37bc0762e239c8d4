"""W8A16 module: int8 weights with one scale per output row.

Stands in for the reference's ``src/quantization/int8.py`` without any change
visible to its callers: class name, constructor ``(weight_q, scale, bias)``,
buffers ``weight_q`` (int8 [N, K]), ``scale`` (fp32 [N]) and ``bias``
(``int8.py:37-42``), ``from_linear``'s arithmetic (``:44-50``: max|w| / 127
floored at 1e-8, round-half-even, clamp to [-127, 127]),
``dequantized_weight`` / ``num_bytes`` / ``forward`` (``:52-63``) and
``quantize_model_int8``'s return value (``:73-100``).  The engines of the
reference look every projection up on its parent module at call time, so
they run on these modules as they are; ``forward`` goes to the sm_100a
kernels through ``w8a16_linear``.  The embeddings and the lm_head (tied to
them) are outside the decoder layers and stay fp16.
"""
from typing import Optional

import torch
import torch.nn as nn

from ..kernels.w8a16_matmul import w8a16_linear, w8a16_quantize_cuda
from ._replace import replace_linears, tensor_bytes


def _quantize_rows_torch(weight: torch.Tensor):
    """PyTorch form of the row quantizer (any device or dtype): returns
    (int8 [N, K], fp32 scales [N])."""
    w32 = weight.float()
    step = torch.clamp(w32.abs().amax(dim=1) / 127.0, min=1e-8)
    codes = torch.round(w32 / step.unsqueeze(1)).clamp(-127, 127).to(torch.int8)
    return codes, step


class QuantizedLinearInt8(nn.Module):
    """Inference-only replacement for an ``nn.Linear`` whose weight is held as
    int8 codes times a float32 scale per output row; weights, scales and bias
    are registered buffers, not Parameters."""

    def __init__(self, weight_q: torch.Tensor, scale: torch.Tensor, bias: Optional[torch.Tensor]):
        super().__init__()
        self.register_buffer("weight_q", weight_q)
        self.register_buffer("scale", scale)
        self.register_buffer("bias", bias)
        self.out_features, self.in_features = weight_q.shape

    @classmethod
    def from_linear(cls, linear: nn.Linear) -> "QuantizedLinearInt8":
        """Quantize ``linear`` row by row.  A CUDA fp16 weight is quantized by
        the device kernel, which yields the same bytes as the PyTorch form
        used for every other input."""
        weight = linear.weight.detach()
        if weight.is_cuda and weight.dtype == torch.float16 and weight.dim() == 2 and weight.shape[0] > 0:
            codes, step = w8a16_quantize_cuda(weight)
        else:
            codes, step = _quantize_rows_torch(weight)
        bias = None if linear.bias is None else linear.bias.detach().clone()
        return cls(codes.contiguous(), step.float().contiguous(), bias)

    def dequantized_weight(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """The weight the kernels multiply by, as a dense [N, K] tensor."""
        return (self.weight_q.float() * self.scale.unsqueeze(1)).to(dtype)

    def num_bytes(self) -> int:
        """Bytes held on the device: int8 codes, row scales and bias."""
        return tensor_bytes(self.weight_q, self.scale, self.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return w8a16_linear(x, self.weight_q, self.scale, self.bias)


def quantize_model_int8(model: nn.Module) -> dict:
    """Put a ``QuantizedLinearInt8`` in place of every linear projection of the
    decoder layers (``model.model.layers``); see ``replace_linears`` for the
    returned statistics."""
    return replace_linears(model, QuantizedLinearInt8.from_linear)


__all__ = ["QuantizedLinearInt8", "quantize_model_int8"]
