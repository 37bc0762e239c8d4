"""Weight-only INT8 linear (W8A16) on B200.

Drop-in for src/kernels/w8a16_matmul_triton.py of the reference:
``w8a16_linear`` (:102-134) and ``w8a16_reference`` (:137-149) keep their
signatures, argument meaning and assert messages.  The math is the
reference's: per-output-channel symmetric int8 weights, fp32 accumulation of
x @ Wq^T, scale applied once per output column, optional bias, output in
x's dtype.

``w8a16_linear`` runs only the CUDA kernels of libqlinear.so (sm_100a):
a TMA-fed dequant-fused GEMV / skinny GEMM for decode-sized M, and a
portable CUDA-core kernel for shapes the TMA path cannot take (K not a
multiple of 16, misaligned strides).  It has no CPU or PyTorch fallback.
It launches on the current stream, allocates only its output (and, once per
stream, a zeroed split-K workspace), never synchronises, and picks its
kernel from a fixed shape table, so it can be captured in a CUDA graph
after one eager call.
"""
from __future__ import annotations

import torch

from .. import _lib
from ._launch import default_flags, dtype_code, ld, on_device, ptr, workspace


def w8a16_linear(
    x: torch.Tensor,
    w_q: torch.Tensor,
    scale: torch.Tensor,
    bias: torch.Tensor = None,
    out: torch.Tensor = None,
) -> torch.Tensor:
    """x: (..., K) fp16. w_q: (N, K) int8. scale: (N,) float32 (fp16 also
    accepted). bias: optional (N,). Returns (..., N) in x's dtype.
    ``out`` (optional, not in the reference): a preallocated (M, N) fp16
    tensor with unit stride along N to write into."""
    assert x.is_cuda and w_q.is_cuda
    assert w_q.dtype == torch.int8, f"w_q must be int8, got {w_q.dtype}"
    N, K = w_q.shape
    assert x.shape[-1] == K, f"x last dim {x.shape[-1]} != weight in_features {K}"
    if x.dtype != torch.float16:
        raise TypeError(f"w8a16_linear: this build takes fp16 activations, got {x.dtype}")
    lib = _lib.load()

    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    else:
        assert out.shape == (M, N) and out.dtype == x.dtype and out.device == x.device, \
            f"out must be ({M}, {N}) {x.dtype} on {x.device}"
        assert out.stride(-1) == 1, "out must have unit stride along N"
    if M == 0 or N == 0:
        return out.reshape(*x.shape[:-1], N)

    if w_q.stride(-1) != 1:
        w_q = w_q.contiguous()
    scale = scale.reshape(-1)
    if not scale.is_contiguous():
        scale = scale.contiguous()
    if bias is not None and not bias.is_contiguous():
        bias = bias.contiguous()
    dev = x.device
    with on_device(dev):
        stream = torch.cuda.current_stream(dev)
        ws_need = lib.ql_w8a16_workspace_size(M, N, K)
        ws = workspace(dev, stream, ws_need)
        status = lib.ql_w8a16_linear(
            ptr(x2), _lib.QL_DTYPE_F16, ptr(w_q),
            ptr(scale), dtype_code(scale.dtype),
            ptr(bias), dtype_code(bias.dtype) if bias is not None else 0,
            ptr(out), M, N, K, ld(x2, K), ld(w_q, K), ld(out, N),
            ptr(ws), ws.numel() if ws is not None else 0,
            default_flags(), stream.cuda_stream)
    _lib.check(status)
    return out.reshape(*x.shape[:-1], N)


def w8a16_reference(
    x: torch.Tensor,
    w_q: torch.Tensor,
    scale: torch.Tensor,
    bias: torch.Tensor = None,
) -> torch.Tensor:
    """The reference's verification helper (w8a16_matmul_triton.py:137-149):
    dequantize the whole weight to fp32, then an ordinary fp32 linear.  Plain
    PyTorch on any device; never called by ``w8a16_linear``."""
    w = w_q.float() * scale.float()[:, None]
    b = bias.float() if bias is not None else None
    return torch.nn.functional.linear(x.float(), w, b).to(x.dtype)


def w8a16_dequantize_cuda(w_q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """``w_q.float() * scale[:, None]`` computed by the device decoder the
    GEMV uses (bit-exact with the reference's dequantized_weight)."""
    assert w_q.is_cuda and w_q.dtype == torch.int8
    lib = _lib.load()
    if w_q.stride(-1) != 1:
        w_q = w_q.contiguous()
    scale = scale.contiguous()
    N, K = w_q.shape
    out = torch.empty((N, K), dtype=torch.float32, device=w_q.device)
    with on_device(w_q.device):
        st = lib.ql_w8a16_dequantize(ptr(w_q), ptr(scale), dtype_code(scale.dtype), ptr(out), N, K,
                                     w_q.stride(0), torch.cuda.current_stream(w_q.device).cuda_stream)
    _lib.check(st)
    return out


def w8a16_quantize_cuda(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """On-device ``QuantizedLinearInt8.from_linear`` math (int8.py:44-50):
    returns (w_q int8 [N, K], scale fp32 [N]), bit-exact with the reference."""
    assert w.is_cuda and w.dtype == torch.float16 and w.dim() == 2
    lib = _lib.load()
    if w.stride(-1) != 1:
        w = w.contiguous()
    N, K = w.shape
    w_q = torch.empty((N, K), dtype=torch.int8, device=w.device)
    scale = torch.empty((N,), dtype=torch.float32, device=w.device)
    with on_device(w.device):
        st = lib.ql_w8a16_quantize(ptr(w), N, K, w.stride(0), ptr(w_q), ptr(scale),
                                   torch.cuda.current_stream(w.device).cuda_stream)
    _lib.check(st)
    return w_q, scale
