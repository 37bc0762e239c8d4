"""CPU oracle for the weight-only quantized linear path (W8A16 / W4A16).

TEST INFRASTRUCTURE ONLY.  This module is the checker: it may be imported by
``tests/``, by ``__graft_entry__.smoke()`` and by the CPU-baseline / reference
legs of ``bench.py``, and by nothing else.  The product path (the CUDA kernels
behind ``libqlinear.so``) never calls into it.

It restates, in numpy, the reference implementation of SriramL1/
LLM-inference-optimizer for this path.  Every function cites the reference
file and lines it follows (paths relative to the reference repository root).

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own functions
(imported from the reference checkout) on seeded inputs and stores their
outputs in ``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this
module against those fixtures bit-for-bit (integer, packed and dequantized
arrays) and to fp32 rounding (matmul outputs).

Arithmetic notes
----------------
* ``torch.round`` and ``numpy.round`` both round half to even, and both do
  IEEE-754 fp32 division, so the quantizers are bit-exact restatements.
* ``tensor.half()`` and ``ndarray.astype(float16)`` both round to nearest even.
* The fp32 matmul is numpy's BLAS sgemm where the reference uses torch's
  ``F.linear``; the summation order differs, so fp32 outputs agree to a few
  ulp, not bit-for-bit.  That is why the GPU parity tests compare with a
  tolerance and the dequantized weights (no summation) bit-for-bit.
"""
from __future__ import annotations

import numpy as np

GROUP_SIZE = 128          # w4a16_matmul_triton.py:37
HALF = GROUP_SIZE // 2    # w4a16_matmul_triton.py:38

# Layout ids shared with the C-ABI (include/qlinear.h).
LAYOUT_SPLIT_HALF = 0     # the reference's packing (w4a16_matmul_triton.py:10-20)
LAYOUT_ADJACENT = 1       # low nibble = even k (the variant benchmark config 1 describes)


# --------------------------------------------------------------------- INT8
def quantize_int8_rows(w: np.ndarray):
    """Per-output-row symmetric int8 quantization.

    Follows ``QuantizedLinearInt8.from_linear`` (src/quantization/int8.py:44-50):
    ``w = W.float(); scale = clamp(amax_k |w| / 127, min=1e-8);
    w_q = round(w / scale[:, None]).clamp(-127, 127).to(int8)``.
    Returns (w_q int8 [N, K], scale float32 [N]).
    """
    w = np.asarray(w).astype(np.float32)
    if w.shape[1] == 0:
        amax = np.zeros((w.shape[0],), np.float32)
    else:
        amax = np.abs(w).max(axis=1)
    scale = np.maximum(amax / np.float32(127.0), np.float32(1e-8)).astype(np.float32)
    q = np.round(w / scale[:, None]).clip(-127, 127).astype(np.int8)
    return q, scale


def dequantize_int8(w_q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """``w_q.float() * scale.float()[:, None]`` in fp32.

    Follows ``QuantizedLinearInt8.dequantized_weight`` (int8.py:52-53) and the
    first line of ``w8a16_reference`` (w8a16_matmul_triton.py:147).  The scale
    may be fp32 (the reference's buffer) or fp16 (benchmark config 0).
    """
    return w_q.astype(np.float32) * np.asarray(scale).astype(np.float32)[:, None]


def linear_f32(x: np.ndarray, w_deq: np.ndarray, bias=None) -> np.ndarray:
    """``F.linear(x.float(), w, b.float())`` before the final dtype cast."""
    x2 = np.asarray(x).astype(np.float32)
    y = x2 @ w_deq.T
    if bias is not None:
        y = y + np.asarray(bias).astype(np.float32)[None, :]
    return y.astype(np.float32)


def w8a16_reference_f32(x, w_q, scale, bias=None):
    """``w8a16_reference`` (w8a16_matmul_triton.py:137-149) without the fp16 cast."""
    K = w_q.shape[1]
    x2 = np.asarray(x).reshape(-1, K)
    return linear_f32(x2, dequantize_int8(w_q, scale), bias)


def w8a16_reference(x, w_q, scale, bias=None):
    """``w8a16_reference`` (w8a16_matmul_triton.py:137-149): fp32 dequant,
    fp32 linear, cast to x's dtype (fp16 here).  Leading dims preserved."""
    x = np.asarray(x)
    y = w8a16_reference_f32(x, w_q, scale, bias)
    return y.astype(np.float16).reshape(*x.shape[:-1], w_q.shape[0])


# --------------------------------------------------------------------- INT4
def pack_int4(q: np.ndarray) -> np.ndarray:
    """Split-half packing of offset-binary nibbles.

    Follows ``pack_int4`` (w4a16_matmul_triton.py:42-49): inside each group of
    128, byte j (0..63) holds element j in its low nibble and element j+64 in
    its high nibble.  q: [N, K] integers in 0..15, K % 128 == 0.
    """
    N, K = q.shape
    assert K % GROUP_SIZE == 0, f"K={K} must be a multiple of {GROUP_SIZE}"
    g = q.astype(np.uint8).reshape(N, K // GROUP_SIZE, 2, HALF)
    packed = g[:, :, 0, :] | (g[:, :, 1, :] << 4)
    return np.ascontiguousarray(packed.reshape(N, K // 2)).astype(np.uint8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Inverse of ``pack_int4`` (w4a16_matmul_triton.py:52-58)."""
    N, half_k = packed.shape
    p = packed.reshape(N, half_k // HALF, HALF)
    lo = p & 0xF
    hi = p >> 4
    return np.stack([lo, hi], axis=2).reshape(N, half_k * 2).astype(np.uint8)


def pack_int4_adjacent(q: np.ndarray) -> np.ndarray:
    """Adjacent-pair packing: byte i holds k=2i (low nibble) and 2i+1 (high).

    The reference has no code for this layout; it is the format benchmark
    config 1 words ("two nibbles per uint8 along K, low nibble = even k").
    Nibble values are the same offset-binary q+8 as the reference's.
    """
    N, K = q.shape
    assert K % 2 == 0
    q = q.astype(np.uint8)
    return np.ascontiguousarray(q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)


def unpack_int4_adjacent(packed: np.ndarray) -> np.ndarray:
    N, half_k = packed.shape
    out = np.empty((N, half_k * 2), np.uint8)
    out[:, 0::2] = packed & 0xF
    out[:, 1::2] = packed >> 4
    return out


def unpack_layout(packed: np.ndarray, layout: int) -> np.ndarray:
    if layout == LAYOUT_SPLIT_HALF:
        return unpack_int4(packed)
    if layout == LAYOUT_ADJACENT:
        return unpack_int4_adjacent(packed)
    raise ValueError(f"unknown layout {layout}")


def pack_layout(q: np.ndarray, layout: int) -> np.ndarray:
    if layout == LAYOUT_SPLIT_HALF:
        return pack_int4(q)
    if layout == LAYOUT_ADJACENT:
        return pack_int4_adjacent(q)
    raise ValueError(f"unknown layout {layout}")


def quantize_int4_groups(w: np.ndarray, qmin: int = -7, qmax: int = 7,
                         layout: int = LAYOUT_SPLIT_HALF):
    """Group-128 symmetric RTN int4 quantization.

    Follows ``QuantizedLinearInt4.from_linear`` (src/quantization/int4.py:37-49):
    ``scale = clamp(amax_group |w| / 7, min=1e-5); scale16 = scale.half();
    q = round(wg / scale16.float()).clamp(-7, 7) + 8; packed = pack_int4(q);
    scales = scale16.t()`` -> (packed uint8 [N, K/2], scales fp16 [K/128, N]).
    ``qmin=-8`` with ``layout=LAYOUT_ADJACENT`` gives the benchmark-config-1
    variant ([-8, 7], low nibble = even k).
    """
    w = np.asarray(w).astype(np.float32)
    N, K = w.shape
    assert K % GROUP_SIZE == 0, f"in_features {K} must be a multiple of {GROUP_SIZE}"
    wg = w.reshape(N, K // GROUP_SIZE, GROUP_SIZE)
    scale = np.maximum(np.abs(wg).max(axis=2) / np.float32(7.0), np.float32(1e-5)).astype(np.float32)
    scale16 = scale.astype(np.float16)
    q = np.round(wg / scale16.astype(np.float32)[:, :, None]).clip(qmin, qmax) + 8
    packed = pack_layout(q.reshape(N, K).astype(np.uint8), layout)
    scales = np.ascontiguousarray(scale16.T)
    return packed, scales


def dequantize_int4(w_packed: np.ndarray, scales: np.ndarray,
                    layout: int = LAYOUT_SPLIT_HALF) -> np.ndarray:
    """``(unpack - 8).float() * scales.float().t()`` per group, fp32 [N, K].

    Follows ``dequantize_int4`` (w4a16_matmul_triton.py:173-178).
    """
    q = unpack_layout(w_packed, layout).astype(np.float32) - np.float32(8.0)
    N, K = q.shape
    s = np.asarray(scales).astype(np.float32).T.reshape(N, K // GROUP_SIZE, 1)
    return (q.reshape(N, K // GROUP_SIZE, GROUP_SIZE) * s).reshape(N, K)


def w4a16_reference_f32(x, w_packed, scales, bias=None, layout=LAYOUT_SPLIT_HALF):
    """``w4a16_reference`` (w4a16_matmul_triton.py:181-187) without the cast."""
    K = w_packed.shape[1] * 2
    x2 = np.asarray(x).reshape(-1, K)
    return linear_f32(x2, dequantize_int4(w_packed, scales, layout), bias)


def w4a16_reference(x, w_packed, scales, bias=None, layout=LAYOUT_SPLIT_HALF):
    x = np.asarray(x)
    y = w4a16_reference_f32(x, w_packed, scales, bias, layout)
    return y.astype(np.float16).reshape(*x.shape[:-1], w_packed.shape[0])


# ---------------------------------------------------------------- tolerance
def parity_bounds(x: np.ndarray, w_deq: np.ndarray):
    """The output tolerance the north star states for this path.

    max-abs error <= 1e-2 * ||x||_inf * ||w||_inf * sqrt(K) / 64 and
    rel-L2 error <= 2e-3, both against the fp32-accumulated reference
    computed before the fp16 cast.  Returns (max_abs_bound, rel_l2_bound).
    """
    K = w_deq.shape[1]
    xin = float(np.abs(np.asarray(x, np.float32)).max()) if x.size else 0.0
    win = float(np.abs(w_deq).max()) if w_deq.size else 0.0
    return 1e-2 * xin * win * np.sqrt(max(K, 1)) / 64.0, 2e-3


def check_parity(y_gpu: np.ndarray, y_ref_f32: np.ndarray, x: np.ndarray, w_deq: np.ndarray):
    """Returns (ok, max_abs_err, rel_l2_err, max_abs_bound, rel_bound)."""
    y = np.asarray(y_gpu, np.float32).reshape(y_ref_f32.shape)
    err = y - y_ref_f32
    max_abs = float(np.abs(err).max()) if err.size else 0.0
    denom = float(np.linalg.norm(y_ref_f32))
    rel = float(np.linalg.norm(err) / denom) if denom > 0 else float(np.linalg.norm(err))
    b_abs, b_rel = parity_bounds(x, w_deq)
    ok = (max_abs <= b_abs + 1e-6) and (rel <= b_rel)
    return ok, max_abs, rel, b_abs, b_rel
