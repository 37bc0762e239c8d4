"""Shared test helpers: seeded inputs (CPU generators, so the GPU kernels and
the CPU oracle see identical bits) and the north-star parity check."""
from __future__ import annotations

import numpy as np
import torch

from oracle import qlinear_oracle as orc


def make_linear(K, N, bias, seed=0, std=0.05, device="cpu"):
    """Mirrors the reference tests' _make_linear (tests/test_w8a16_kernel.py:48-55)
    with a CPU generator: W = randn*std fp16, bias = randn*0.1."""
    g = torch.Generator().manual_seed(seed)
    lin = torch.nn.Linear(K, N, bias=bias).half()
    with torch.no_grad():
        lin.weight.copy_((torch.randn(N, K, generator=g) * std).half())
        if bias:
            lin.bias.copy_((torch.randn(N, generator=g) * 0.1).half())
    return lin.to(device)


def make_x(M, K, seed=1, device="cpu", lead=None):
    g = torch.Generator().manual_seed(seed)
    shape = (M, K) if lead is None else (*lead, K)
    return torch.randn(*shape, generator=g).half().to(device)


def assert_parity(y_gpu: torch.Tensor, y_ref_f32: np.ndarray, x: np.ndarray, w_deq: np.ndarray, what=""):
    """North-star tolerance against the fp32-accumulated reference before the
    fp16 cast: max-abs <= 1e-2*|x|inf*|w|inf*sqrt(K)/64 and rel-L2 <= 2e-3."""
    y = y_gpu.detach().float().cpu().numpy()
    assert np.isfinite(y).all(), f"{what}: non-finite output"
    ok, max_abs, rel, b_abs, b_rel = orc.check_parity(y, y_ref_f32, x, w_deq)
    assert ok, f"{what}: max_abs {max_abs:.3e} (bound {b_abs:.3e}) rel_l2 {rel:.3e} (bound {b_rel:.1e})"
    return max_abs, rel


def linear_unsplit(q, x):
    """q(x) through the decode kernel planned without a workspace (no
    K-split): the plan the fused greedy-head launch uses, so its fp16
    outputs are bit-identical to what that launch reduces."""
    from qlinear import _lib
    from qlinear.quantization.int8 import QuantizedLinearInt8
    lib = _lib.load()
    M, K = x.shape
    N = q.out_features
    out = torch.empty(M, N, dtype=torch.float16, device=x.device)
    flags = _lib.QL_FLAG_FORCE_GEMV | _lib.QL_FLAG_PDL
    stream = torch.cuda.current_stream().cuda_stream
    bias = q.bias.data_ptr() if q.bias is not None else None
    if isinstance(q, QuantizedLinearInt8):
        st = lib.ql_w8a16_linear(x.data_ptr(), 0, q.weight_q.data_ptr(), q.scale.data_ptr(), _lib.QL_DTYPE_F32,
                                 bias, 0, out.data_ptr(), M, N, K, K, K, N, None, 0, flags, stream)
    else:
        st = lib.ql_w4a16_linear(x.data_ptr(), 0, q.weight_packed.data_ptr(), q.layout, q.scales.data_ptr(), bias,
                                 0, out.data_ptr(), M, N, K, K, K // 2, N, N, None, 0, flags, stream)
    _lib.check(st)
    return out
