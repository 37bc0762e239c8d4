"""INT8 weight quantization of a loaded model (W8A16).

Drop-in for src/quantization/int8.py of the reference: the class, its
constructor arguments, buffer names (``weight_q``, ``scale``, ``bias``),
``from_linear`` (:44-50), ``dequantized_weight`` (:52-53), ``num_bytes``
(:55-60), ``forward`` (:62-63) and ``quantize_model_int8`` (:73-100) keep
their behaviour, so the reference's engines (HF forward, paged, continuous
batching, CUDA-graph decode), which look the projections up as attributes on
every call, run on these modules unchanged.  ``forward`` goes to the B200
kernels through ``w8a16_linear``.

Scope as in the reference: every nn.Linear inside ``model.model.layers``;
embeddings and the (tied) lm_head stay fp16.
"""
import gc
from typing import Optional

import torch
import torch.nn as nn

from ..kernels.w8a16_matmul import w8a16_linear, w8a16_quantize_cuda


class QuantizedLinearInt8(nn.Module):
    """Drop-in replacement for nn.Linear holding int8 weights plus a
    per-output-channel float32 scale.  Weights and scales are buffers, not
    Parameters: this is an inference-only module."""

    def __init__(self, weight_q: torch.Tensor, scale: torch.Tensor, bias: Optional[torch.Tensor]):
        super().__init__()
        self.register_buffer("weight_q", weight_q)
        self.register_buffer("scale", scale)
        self.register_buffer("bias", bias)  # None is allowed
        self.out_features, self.in_features = weight_q.shape

    @classmethod
    def from_linear(cls, linear: nn.Linear) -> "QuantizedLinearInt8":
        """Per-row symmetric quantization: scale = max(|W[n,:]|)/127 (>= 1e-8),
        w_q = round-half-even(W / scale) clamped to [-127, 127].  On a CUDA
        fp16 weight the device quantizer produces the same bits as the
        PyTorch expression used for other devices/dtypes."""
        wt = linear.weight.detach()
        if wt.is_cuda and wt.dtype == torch.float16 and wt.dim() == 2 and wt.shape[0] > 0:
            w_q, scale = w8a16_quantize_cuda(wt)
        else:
            w = wt.float()
            scale = (w.abs().amax(dim=1) / 127.0).clamp(min=1e-8)
            w_q = torch.round(w / scale[:, None]).clamp(-127, 127).to(torch.int8)
        bias = linear.bias.detach().clone() if linear.bias is not None else None
        return cls(w_q.contiguous(), scale.float().contiguous(), bias)

    def dequantized_weight(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return (self.weight_q.float() * self.scale[:, None]).to(dtype)

    def num_bytes(self) -> int:
        total = self.weight_q.numel() * self.weight_q.element_size()
        total += self.scale.numel() * self.scale.element_size()
        if self.bias is not None:
            total += self.bias.numel() * self.bias.element_size()
        return total

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return w8a16_linear(x, self.weight_q, self.scale, self.bias)


def _linear_bytes(linear: nn.Linear) -> int:
    total = linear.weight.numel() * linear.weight.element_size()
    if linear.bias is not None:
        total += linear.bias.numel() * linear.bias.element_size()
    return total


def quantize_model_int8(model: nn.Module) -> dict:
    """Replaces every nn.Linear inside model.model.layers with a
    QuantizedLinearInt8, in place.  Returns {layers_quantized, bytes_before,
    bytes_after}; callers should check layers_quantized > 0."""
    layers_root = model.model.layers
    layers_quantized = 0
    bytes_before = 0
    bytes_after = 0

    for parent in list(layers_root.modules()):
        for child_name, child in list(parent.named_children()):
            if isinstance(child, nn.Linear):
                bytes_before += _linear_bytes(child)
                quantized = QuantizedLinearInt8.from_linear(child)
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
