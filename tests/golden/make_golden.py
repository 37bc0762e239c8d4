"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once, in a checkout that has the reference repository available
(SriramL1/LLM-inference-optimizer), with:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <path>

It imports the reference's own quantizers, packers and ``*_reference``
functions (src/quantization/int8.py, src/quantization/int4.py,
src/kernels/w8a16_matmul_triton.py, src/kernels/w4a16_matmul_triton.py),
runs them on CPU on seeded inputs and writes their outputs as ``.npz`` files
next to this script.  Nothing at test time reads the reference itself: the
fixtures travel, the reference does not.

Inputs are drawn from CPU ``torch.Generator``s so every machine sees the same
bits.  Weight draws mirror the reference tests (randn * 0.05, bias randn * 0.1;
tests/test_w8a16_kernel.py:48-55) plus hand-built rows that hit the rounding
edge cases: exact half-step ties (round-half-to-even), all-zero rows (scale
clamp), and the +-127 / +-7 extremes.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _linear(K, N, bias, seed, std=0.05):
    g = torch.Generator().manual_seed(seed)
    lin = torch.nn.Linear(K, N, bias=bias).half()
    with torch.no_grad():
        lin.weight.copy_((torch.randn(N, K, generator=g) * std).half())
        if bias:
            lin.bias.copy_((torch.randn(N, generator=g) * 0.1).half())
    return lin


def _x(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(M, K, generator=g).half()


def _tie_rows_int8(K):
    """Rows whose values land exactly on half steps of scale = 2^-6."""
    s = 2.0 ** -6
    base = np.array([127, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -126.5, 126.5, 0, -127], np.float32)
    row0 = np.resize(base, K) * s
    row1 = np.zeros(K, np.float32)                       # all-zero row -> clamp(1e-8)
    row2 = -np.resize(base, K) * s
    return np.stack([row0, row1, row2]).astype(np.float16)


def _tie_rows_int4(K):
    """Group-wise rows with scale = 7*2^-4 / 7 = 2^-4 and half-step ties."""
    s = 2.0 ** -4
    base = np.array([7, 0.5, 1.5, 2.5, 3.5, -0.5, -1.5, -2.5, -3.5, 6.5, -6.5, 0, -7, 4.5, -4.5, 5.5], np.float32)
    row0 = np.resize(base, K) * s
    row1 = np.zeros(K, np.float32)
    row2 = -np.resize(base, K) * s
    return np.stack([row0, row1, row2]).astype(np.float16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.path.insert(0, str(Path(args.reference).resolve()))

    from src.kernels.w8a16_matmul_triton import w8a16_reference
    from src.kernels.w4a16_matmul_triton import (
        pack_int4, unpack_int4, dequantize_int4, w4a16_reference,
    )
    from src.quantization.int8 import QuantizedLinearInt8
    from src.quantization.int4 import QuantizedLinearInt4

    torch.set_num_threads(1)

    # ---------------------------------------------------------- INT8 cases
    int8 = {}
    cases8 = [
        ("k100_n37_m7_bias", 100, 37, 7, True),
        ("k384_n100_m5", 384, 100, 5, False),
        ("k256_n64_m1_bias", 256, 64, 1, True),
        ("k1536_n48_m3_bias", 1536, 48, 3, True),
    ]
    for i, (name, K, N, M, bias) in enumerate(cases8):
        lin = _linear(K, N, bias, seed=100 + i)
        q = QuantizedLinearInt8.from_linear(lin)
        x = _x(M, K, seed=200 + i)
        int8[f"{name}/w"] = lin.weight.detach().numpy()
        if bias:
            int8[f"{name}/bias"] = lin.bias.detach().numpy()
        int8[f"{name}/x"] = x.numpy()
        int8[f"{name}/wq"] = q.weight_q.numpy()
        int8[f"{name}/scale"] = q.scale.numpy()
        int8[f"{name}/deq"] = q.dequantized_weight(torch.float32).numpy()
        int8[f"{name}/y16"] = w8a16_reference(x, q.weight_q, q.scale, q.bias).numpy()
        b = q.bias.float() if q.bias is not None else None
        int8[f"{name}/y32"] = torch.nn.functional.linear(
            x.float(), q.dequantized_weight(torch.float32), b).numpy()
        # fp16-scale variant (benchmark config 0 stores fp16 scales); the
        # reference's oracle accepts it via scale.float().
        int8[f"{name}/y16_scale16"] = w8a16_reference(x, q.weight_q, q.scale.half(), q.bias).numpy()
    # edge rows: ties, zero row, extremes
    K = 128
    w = torch.from_numpy(_tie_rows_int8(K))
    lin = torch.nn.Linear(K, 3, bias=False).half()
    with torch.no_grad():
        lin.weight.copy_(w)
    q = QuantizedLinearInt8.from_linear(lin)
    int8["ties/w"] = w.numpy()
    int8["ties/wq"] = q.weight_q.numpy()
    int8["ties/scale"] = q.scale.numpy()
    int8["ties/deq"] = q.dequantized_weight(torch.float32).numpy()
    np.savez_compressed(HERE / "int8_cases.npz", **int8)

    # ---------------------------------------------------------- INT4 cases
    int4 = {}
    cases4 = [
        ("k384_n100_m7_bias", 384, 100, 7, True),
        ("k256_n64_m3", 256, 64, 3, False),
        ("k1536_n40_m2_bias", 1536, 40, 2, True),
    ]
    for i, (name, K, N, M, bias) in enumerate(cases4):
        lin = _linear(K, N, bias, seed=300 + i)
        q = QuantizedLinearInt4.from_linear(lin)
        x = _x(M, K, seed=400 + i)
        int4[f"{name}/w"] = lin.weight.detach().numpy()
        if bias:
            int4[f"{name}/bias"] = lin.bias.detach().numpy()
        int4[f"{name}/x"] = x.numpy()
        int4[f"{name}/packed"] = q.weight_packed.numpy()
        int4[f"{name}/scales"] = q.scales.numpy()
        int4[f"{name}/unpacked"] = unpack_int4(q.weight_packed).numpy()
        int4[f"{name}/deq"] = dequantize_int4(q.weight_packed, q.scales).numpy()
        int4[f"{name}/y16"] = w4a16_reference(x, q.weight_packed, q.scales, q.bias).numpy()
        b = q.bias.float() if q.bias is not None else None
        int4[f"{name}/y32"] = torch.nn.functional.linear(
            x.float(), dequantize_int4(q.weight_packed, q.scales), b).numpy()
    K = 256
    w = torch.from_numpy(_tie_rows_int4(K))
    lin = torch.nn.Linear(K, 3, bias=False).half()
    with torch.no_grad():
        lin.weight.copy_(w)
    q = QuantizedLinearInt4.from_linear(lin)
    int4["ties/w"] = w.numpy()
    int4["ties/packed"] = q.weight_packed.numpy()
    int4["ties/scales"] = q.scales.numpy()
    int4["ties/deq"] = dequantize_int4(q.weight_packed, q.scales).numpy()
    # every nibble value (0..15, including 0 = -8 that the quantizer never
    # emits) through the reference dequantizer, in both nibble positions
    qall = torch.arange(16, dtype=torch.uint8).repeat(4, 16)          # (4, 256)
    qall[2:] = qall[2:].flip(1)
    packed_all = pack_int4(qall)
    scales_all = torch.tensor([[0.5, 1.0, -2.0, 0.0999755859375],
                               [3.0, 0.25, 1.5, 65504.0]], dtype=torch.float16)  # (G=2, N=4)
    int4["allnibbles/q"] = qall.numpy()
    int4["allnibbles/packed"] = packed_all.numpy()
    int4["allnibbles/scales"] = scales_all.numpy()
    int4["allnibbles/deq"] = dequantize_int4(packed_all, scales_all).numpy()
    np.savez_compressed(HERE / "int4_cases.npz", **int4)

    # ------------------------------------------------- pack/unpack KAT
    # the reference's own known-answer test inputs (tests/test_w4a16_kernel.py:52-59)
    torch.manual_seed(0)
    q1 = torch.randint(0, 16, (37, 384), dtype=torch.uint8)
    q2 = torch.arange(16, dtype=torch.uint8).repeat(2, 8)
    kat = {
        "q1": q1.numpy(), "packed1": pack_int4(q1).numpy(), "unpacked1": unpack_int4(pack_int4(q1)).numpy(),
        "q2": q2.numpy(), "packed2": pack_int4(q2).numpy(), "unpacked2": unpack_int4(pack_int4(q2)).numpy(),
    }
    np.savez_compressed(HERE / "pack_kat.npz", **kat)
    for f in ("int8_cases.npz", "int4_cases.npz", "pack_kat.npz"):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
