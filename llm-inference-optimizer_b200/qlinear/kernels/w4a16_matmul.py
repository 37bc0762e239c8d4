"""Weight-only INT4 linear (W4A16, group 128) on B200.

Drop-in for src/kernels/w4a16_matmul_triton.py of the reference:
``GROUP_SIZE``/``HALF`` (:37-38), ``pack_int4`` (:42-49), ``unpack_int4``
(:52-58), ``w4a16_linear`` (:134-170), ``dequantize_int4`` (:173-178) and
``w4a16_reference`` (:181-187) keep their signatures, argument meaning and
assert messages.

Format (the reference's): offset-binary nibbles q+8 with q in [-7, 7];
inside each group of 128 along K, byte j (0..63) holds element j in its low
nibble and element j+64 in its high nibble; fp16 scales laid out
(K/128, N).  ``layout=LAYOUT_ADJACENT`` selects the variant where byte i
holds k=2i (low) and 2i+1 (high); the kernels read both in place.

``w4a16_linear`` runs only the CUDA kernels of libqlinear.so (sm_100a); no
CPU or PyTorch fallback.  Launches on the current stream, allocates only its
output (plus a per-stream zeroed split-K workspace, once), never
synchronises, and is CUDA-graph capturable after one eager call.
"""
from __future__ import annotations

import torch

from .. import _lib
from ._launch import default_flags, dtype_code, ld, on_device, ptr, workspace

GROUP_SIZE = 128
HALF = GROUP_SIZE // 2

LAYOUT_SPLIT_HALF = _lib.QL_W4_LAYOUT_SPLIT_HALF
LAYOUT_ADJACENT = _lib.QL_W4_LAYOUT_ADJACENT


# ---------------------------------------------------------------- packing
def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """Pack 4-bit codes (values 0..15, shape [N, K], K a multiple of 128)
    into [N, K/2] bytes, split-half within every 128-group: byte j of a group
    carries code j in bits 0-3 and code j + 64 in bits 4-7."""
    N, K = q.shape
    assert K % GROUP_SIZE == 0, f"K={K} must be a multiple of {GROUP_SIZE}"
    first, second = q.to(torch.uint8).reshape(N, K // GROUP_SIZE, 2, HALF).unbind(dim=2)
    return (first | (second << 4)).reshape(N, K // 2).contiguous()


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """Codes of a split-half packed [N, K/2] byte tensor, as uint8 [N, K]:
    per group of 64 bytes, the 64 low nibbles followed by the 64 high ones."""
    N, half_k = packed.shape
    per_group = packed.reshape(N, half_k // HALF, HALF)
    return torch.cat((per_group & 0xF, per_group >> 4), dim=2).reshape(N, 2 * half_k)


def pack_int4_adjacent(q: torch.Tensor) -> torch.Tensor:
    """Adjacent-pair packing: byte i = q[:, 2i] | q[:, 2i+1] << 4."""
    q = q.to(torch.uint8)
    return (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()


def unpack_int4_adjacent(packed: torch.Tensor) -> torch.Tensor:
    N, half_k = packed.shape
    return torch.stack([packed & 0xF, packed >> 4], dim=2).reshape(N, half_k * 2)


def _unpack(packed: torch.Tensor, layout: int) -> torch.Tensor:
    if layout == LAYOUT_SPLIT_HALF:
        return unpack_int4(packed)
    if layout == LAYOUT_ADJACENT:
        return unpack_int4_adjacent(packed)
    raise ValueError(f"unknown int4 layout {layout}")


# ----------------------------------------------------------------- linear
def w4a16_linear(
    x: torch.Tensor,
    w_packed: torch.Tensor,
    scales: torch.Tensor,
    bias: torch.Tensor = None,
    layout: int = LAYOUT_SPLIT_HALF,
    out: torch.Tensor = None,
) -> torch.Tensor:
    """x: (..., K) fp16. w_packed: (N, K//2) uint8. scales: (K//128, N)
    fp16. bias: optional (N,). Returns (..., N) in x's dtype.
    ``layout`` and ``out`` are additions: the int4 packing variant, and a
    preallocated (M, N) fp16 tensor with unit stride along N."""
    assert x.is_cuda and w_packed.is_cuda
    assert w_packed.dtype == torch.uint8, f"w_packed must be uint8, got {w_packed.dtype}"
    N, half_k = w_packed.shape
    K = half_k * 2
    assert x.shape[-1] == K, f"x last dim {x.shape[-1]} != weight in_features {K}"
    assert K % GROUP_SIZE == 0
    assert scales.shape == (K // GROUP_SIZE, N), f"scales shape {tuple(scales.shape)}"
    if x.dtype != torch.float16:
        raise TypeError(f"w4a16_linear: this build takes fp16 activations, got {x.dtype}")
    if scales.dtype != torch.float16:
        raise TypeError(f"w4a16_linear: scales must be fp16, got {scales.dtype}")
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

    if w_packed.stride(-1) != 1:
        w_packed = w_packed.contiguous()
    if scales.stride(-1) != 1:
        scales = scales.contiguous()
    if bias is not None and not bias.is_contiguous():
        bias = bias.contiguous()
    dev = x.device
    with on_device(dev):
        stream = torch.cuda.current_stream(dev)
        ws_need = lib.ql_w4a16_workspace_size(M, N, K)
        ws = workspace(dev, stream, ws_need)
        status = lib.ql_w4a16_linear(
            ptr(x2), _lib.QL_DTYPE_F16, ptr(w_packed), layout, ptr(scales),
            ptr(bias), dtype_code(bias.dtype) if bias is not None else 0,
            ptr(out), M, N, K, ld(x2, K), ld(w_packed, K // 2), ld(scales, N), ld(out, N),
            ptr(ws), ws.numel() if ws is not None else 0,
            default_flags(), stream.cuda_stream)
    _lib.check(status)
    return out.reshape(*x.shape[:-1], N)


def dequantize_int4(w_packed: torch.Tensor, scales: torch.Tensor,
                    layout: int = LAYOUT_SPLIT_HALF) -> torch.Tensor:
    """(N, K//2) uint8 + (K//128, N) scales -> (N, K) float32 weights.
    Plain PyTorch on any device, as in the reference."""
    q = _unpack(w_packed, layout).float() - 8.0                # (N, K)
    N, K = q.shape
    s = scales.float().t().reshape(N, K // GROUP_SIZE, 1)       # (N, G, 1)
    return (q.reshape(N, K // GROUP_SIZE, GROUP_SIZE) * s).reshape(N, K)


def w4a16_reference(x, w_packed, scales, bias=None, layout: int = LAYOUT_SPLIT_HALF):
    """The reference's verification helper (w4a16_matmul_triton.py:181-187):
    dequantize to fp32, then an ordinary fp32 linear.  Plain PyTorch; never
    called by ``w4a16_linear``."""
    w = dequantize_int4(w_packed, scales, layout)
    b = bias.float() if bias is not None else None
    return torch.nn.functional.linear(x.float(), w, b).to(x.dtype)


# ------------------------------------------------- device format helpers
def dequantize_int4_cuda(w_packed: torch.Tensor, scales: torch.Tensor,
                         layout: int = LAYOUT_SPLIT_HALF) -> torch.Tensor:
    """dequantize_int4 computed by the device nibble decoder the GEMV uses."""
    assert w_packed.is_cuda and w_packed.dtype == torch.uint8 and scales.dtype == torch.float16
    lib = _lib.load()
    if w_packed.stride(-1) != 1:
        w_packed = w_packed.contiguous()
    if scales.stride(-1) != 1:
        scales = scales.contiguous()
    N, half_k = w_packed.shape
    K = half_k * 2
    out = torch.empty((N, K), dtype=torch.float32, device=w_packed.device)
    with on_device(w_packed.device):
        st = lib.ql_w4a16_dequantize(ptr(w_packed), layout, ptr(scales), ptr(out), N, K,
                                     w_packed.stride(0), scales.stride(0),
                                     torch.cuda.current_stream(w_packed.device).cuda_stream)
    _lib.check(st)
    return out


def unpack_int4_cuda(w_packed: torch.Tensor, layout: int = LAYOUT_SPLIT_HALF) -> torch.Tensor:
    assert w_packed.is_cuda and w_packed.dtype == torch.uint8
    lib = _lib.load()
    if w_packed.stride(-1) != 1:
        w_packed = w_packed.contiguous()
    N, half_k = w_packed.shape
    out = torch.empty((N, half_k * 2), dtype=torch.uint8, device=w_packed.device)
    with on_device(w_packed.device):
        st = lib.ql_w4a16_unpack(ptr(w_packed), layout, ptr(out), N, half_k * 2, w_packed.stride(0),
                                 torch.cuda.current_stream(w_packed.device).cuda_stream)
    _lib.check(st)
    return out


def w4a16_quantize_cuda(w: torch.Tensor, qmin: int = -7, layout: int = LAYOUT_SPLIT_HALF):
    """On-device ``QuantizedLinearInt4.from_linear`` math (int4.py:37-49):
    returns (packed uint8 [N, K//2], scales fp16 [K//128, N]), bit-exact."""
    assert w.is_cuda and w.dtype == torch.float16 and w.dim() == 2
    N, K = w.shape
    assert K % GROUP_SIZE == 0, f"in_features {K} must be a multiple of {GROUP_SIZE}"
    lib = _lib.load()
    if w.stride(-1) != 1:
        w = w.contiguous()
    packed = torch.empty((N, K // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((K // GROUP_SIZE, N), dtype=torch.float16, device=w.device)
    with on_device(w.device):
        st = lib.ql_w4a16_quantize(ptr(w), N, K, w.stride(0), qmin, layout, ptr(packed), ptr(scales),
                                   torch.cuda.current_stream(w.device).cuda_stream)
    _lib.check(st)
    return packed, scales
