"""qlinear — B200-native weight-only quantized linear layer (W8A16, W4A16).

Host-side mirror of the quantized-linear interface of
SriramL1/LLM-inference-optimizer:

    qlinear.kernels.w8a16_matmul   <-> src/kernels/w8a16_matmul_triton.py
    qlinear.kernels.w4a16_matmul   <-> src/kernels/w4a16_matmul_triton.py
    qlinear.quantization.int8      <-> src/quantization/int8.py
    qlinear.quantization.int4      <-> src/quantization/int4.py
    qlinear.sharded                 column-sharded large-N layers (new)

The compute runs in libqlinear.so (hand-written CUDA for sm_100a, C ABI in
include/qlinear.h), bound through ctypes in ``qlinear._lib``.
"""
__version__ = "0.1.0"
