"""W8A16 kernel parity on the GPU, through the reference-facing API and the C ABI.

Mirrors the reference's tests/test_w8a16_kernel.py (same shapes, M values,
bias on/off, 3-D input, quantization-error and byte bounds) and adds:
  * the north-star tolerance against the CPU oracle's fp32 result
    (max-abs <= 1e-2*|x|inf*|w|inf*sqrt(K)/64, rel-L2 <= 2e-3);
  * the benchmark config-0 case (fp16 scales);
  * ragged / tiny shapes, both kernel paths, determinism, workspace hygiene,
    PDL on/off, CUDA-graph capture, device quantizer/dequantizer bit-exact.
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import qlinear_oracle as orc
from qlinear import _lib
from qlinear.kernels import _launch
from qlinear.kernels.w8a16_matmul import (
    w8a16_linear, w8a16_reference, w8a16_dequantize_cuda, w8a16_quantize_cuda,
)
from qlinear.quantization.int8 import QuantizedLinearInt8

from helpers import assert_parity, make_linear, make_x

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="requires a CUDA GPU")]

GOLDEN = Path(__file__).resolve().parent / "golden"

LAYER_SHAPES = [
    (1536, 1536),   # q_proj / o_proj
    (1536, 256),    # k_proj / v_proj
    (1536, 8960),   # gate_proj / up_proj
    (8960, 1536),   # down_proj
    (100, 37),      # awkward: K not a multiple of 16 -> portable kernel
]
M_VALUES = [1, 7, 16, 100, 300]


def _run_oracle(x, q):
    wq = q.weight_q.cpu().numpy()
    scale = q.scale.cpu().numpy()
    deq = orc.dequantize_int8(wq, scale)
    b = q.bias.cpu().numpy() if q.bias is not None else None
    return orc.linear_f32(x.cpu().numpy().reshape(-1, wq.shape[1]), deq, b), deq


def _raw_call(x, q, flags, ws=None):
    """Calls the C ABI directly with explicit flags (test hook)."""
    lib = _lib.load()
    N, K = q.weight_q.shape
    x2 = x.reshape(-1, K).contiguous()
    out = torch.empty((x2.shape[0], N), dtype=torch.float16, device=x.device)
    st = lib.ql_w8a16_linear(
        x2.data_ptr(), 0, q.weight_q.data_ptr(), q.scale.data_ptr(),
        _launch.dtype_code(q.scale.dtype),
        q.bias.data_ptr() if q.bias is not None else None,
        _launch.dtype_code(q.bias.dtype) if q.bias is not None else 0,
        out.data_ptr(), x2.shape[0], N, K, x2.stride(0), q.weight_q.stride(0), out.stride(0),
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        flags, torch.cuda.current_stream().cuda_stream)
    _lib.check(st)
    return out


@pytest.mark.parametrize("K,N", LAYER_SHAPES)
@pytest.mark.parametrize("M", M_VALUES)
@pytest.mark.parametrize("bias", [False, True])
def test_kernel_matches_dequantized_reference(K, N, M, bias):
    lin = make_linear(K, N, bias)
    q = QuantizedLinearInt8.from_linear(lin)
    x = make_x(M, K, seed=1)
    y32, deq = _run_oracle(x, q)
    q = q.cuda()
    xd = x.cuda()
    out = w8a16_linear(xd, q.weight_q, q.scale, q.bias)
    assert out.shape == (M, N) and out.dtype == torch.float16
    assert_parity(out, y32, x.numpy(), deq, f"w8 K{K} N{N} M{M} bias{bias}")
    ref = w8a16_reference(xd, q.weight_q, q.scale, q.bias)
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=2e-2)


def test_kernel_handles_3d_input():
    lin = make_linear(1536, 256, bias=True)
    q = QuantizedLinearInt8.from_linear(lin).cuda()
    x = make_x(None, 1536, seed=7, lead=(2, 5)).cuda()
    out = q(x)
    assert out.shape == (2, 5, 256)
    ref = w8a16_reference(x, q.weight_q, q.scale, q.bias)
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=2e-2)


def test_baseline_config0_fp16_scales():
    """benchmark config 0: x [1,1536] N(0,1); W [8960,1536] N(0,0.02);
    per-row int8 with fp16 scales."""
    lin = make_linear(1536, 8960, bias=False, std=0.02, seed=0)
    q = QuantizedLinearInt8.from_linear(lin)
    s16 = q.scale.half()
    x = make_x(1, 1536, seed=1)
    deq = orc.dequantize_int8(q.weight_q.numpy(), s16.numpy())
    y32 = orc.linear_f32(x.numpy(), deq)
    out = w8a16_linear(x.cuda(), q.weight_q.cuda(), s16.cuda())
    assert_parity(out, y32, x.numpy(), deq, "config0")


@pytest.mark.parametrize("K,N,M", [(16, 5, 1), (48, 33, 3), (1552, 40, 9), (128, 1, 2),
                                   (4096, 17, 8), (2048, 300, 64), (256, 64, 17)])
def test_ragged_shapes(K, N, M):
    lin = make_linear(K, N, bias=True, seed=K + N)
    q = QuantizedLinearInt8.from_linear(lin)
    x = make_x(M, K, seed=M)
    y32, deq = _run_oracle(x, q)
    out = w8a16_linear(x.cuda(), q.weight_q.cuda(), q.scale.cuda(), q.bias.cuda())
    assert_parity(out, y32, x.numpy(), deq, f"ragged K{K} N{N} M{M}")


def test_empty_batch_and_noncontiguous_input():
    lin = make_linear(256, 64, bias=True)
    q = QuantizedLinearInt8.from_linear(lin).cuda()
    x0 = torch.empty((0, 256), dtype=torch.float16, device="cuda")
    assert q(x0).shape == (0, 64)
    big = make_x(6, 512, seed=3).cuda()
    xs = big[:, ::2]                     # non-contiguous view
    y32, deq = _run_oracle(xs.contiguous(), q)
    assert_parity(q(xs), y32, xs.cpu().numpy(), deq, "non-contiguous")


@pytest.mark.parametrize("K,N,M", [(1536, 8960, 1), (8960, 1536, 4), (1536, 256, 16)])
def test_portable_kernel_matches(K, N, M):
    lin = make_linear(K, N, bias=True, seed=11)
    q = QuantizedLinearInt8.from_linear(lin)
    x = make_x(M, K, seed=12)
    y32, deq = _run_oracle(x, q)
    out = _raw_call(x.cuda(), q.cuda(), _lib.QL_FLAG_FORCE_GENERIC)
    assert_parity(out, y32, x.numpy(), deq, "generic")


@pytest.mark.parametrize("K,N,M", [(8960, 1536, 1), (1536, 8960, 8), (8960, 1536, 16)])
def test_deterministic_pdl_and_workspace_clean(K, N, M):
    lin = make_linear(K, N, bias=True, seed=21)
    q = QuantizedLinearInt8.from_linear(lin).cuda()
    x = make_x(M, K, seed=22).cuda()
    a = w8a16_linear(x, q.weight_q, q.scale, q.bias)
    b = w8a16_linear(x, q.weight_q, q.scale, q.bias)
    assert torch.equal(a, b)
    need = _lib.load().ql_w8a16_workspace_size(M, N, K)
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    c = _raw_call(x, q, 0, ws)                       # no PDL
    d = _raw_call(x, q, _lib.QL_FLAG_PDL, ws)       # PDL
    e = _raw_call(x, q, 0, None)                     # no workspace -> no split-K plan
    torch.cuda.synchronize()
    assert torch.equal(a, c) and torch.equal(a, d)
    y32, deq = _run_oracle(x, q)
    assert_parity(e, y32, x.cpu().numpy(), deq, "no-ws")
    assert int(ws.count_nonzero()) == 0, "workspace not left zeroed"
    for buf in _launch._workspaces.values():
        assert int(buf.count_nonzero()) == 0


def test_cuda_graph_capture_matches_eager():
    """The graphed decode engine captures projections in a CUDA graph
    (graphed_decode_engine.py:163-175): capture after one eager call."""
    shapes = [(1536, 1536), (1536, 256), (1536, 8960), (8960, 1536)]
    mods = [QuantizedLinearInt8.from_linear(make_linear(K, N, bias=(N == 256), seed=K + N)).cuda()
            for K, N in shapes]
    xs = [make_x(1, K, seed=K).cuda() for K, _ in shapes]
    eager = [m(x) for m, x in zip(mods, xs)]
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for m, x in zip(mods, xs):
            m(x)                           # warm the side stream's workspace
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            outs = [m(x) for m, x in zip(mods, xs)]
    torch.cuda.current_stream().wait_stream(s)
    for o in outs:
        o.zero_()
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, outs):
        assert torch.equal(a, b)


def test_quantization_error_is_small_vs_fp16():
    """Reference bound (test_w8a16_kernel.py:86-100)."""
    lin = make_linear(1536, 8960, bias=False).cuda()
    q = QuantizedLinearInt8.from_linear(lin)
    x = make_x(64, 1536, seed=2).cuda()
    fp16_out = lin(x).float()
    int8_out = q(x).float()
    rel_err = (fp16_out - int8_out).norm() / fp16_out.norm()
    assert rel_err < 0.03


def test_roundtrip_error_within_half_a_quantization_step():
    lin = make_linear(1536, 1536, bias=False).cuda()
    q = QuantizedLinearInt8.from_linear(lin)
    original = lin.weight.float()
    dequantized = q.dequantized_weight(torch.float32)
    max_allowed = (q.scale[:, None] / 2) * 1.001 + 1e-6
    assert ((original - dequantized).abs() <= max_allowed).all()


def test_device_quantizer_and_dequantizer_bitexact():
    z = np.load(GOLDEN / "int8_cases.npz")
    for name in ("k100_n37_m7_bias", "k384_n100_m5", "k256_n64_m1_bias", "k1536_n48_m3_bias", "ties"):
        w = torch.from_numpy(z[f"{name}/w"]).cuda()
        wq, scale = w8a16_quantize_cuda(w)
        assert np.array_equal(wq.cpu().numpy(), z[f"{name}/wq"]), name
        assert np.array_equal(scale.cpu().numpy().view(np.uint32), z[f"{name}/scale"].view(np.uint32)), name
        deq = w8a16_dequantize_cuda(wq, scale)
        assert np.array_equal(deq.cpu().numpy().view(np.uint32), z[f"{name}/deq"].view(np.uint32)), name
    # a large random matrix and from_linear on CUDA (device quantizer path)
    lin = make_linear(8960, 1536, bias=True, std=0.02, seed=9)
    wq_ref, sc_ref = orc.quantize_int8_rows(lin.weight.detach().numpy())
    q = QuantizedLinearInt8.from_linear(lin.cuda())
    assert np.array_equal(q.weight_q.cpu().numpy(), wq_ref)
    assert np.array_equal(q.scale.cpu().numpy().view(np.uint32), sc_ref.view(np.uint32))
    deq = w8a16_dequantize_cuda(q.weight_q, q.scale.half())
    assert np.array_equal(deq.cpu().numpy().view(np.uint32),
                          orc.dequantize_int8(wq_ref, sc_ref.astype(np.float16)).view(np.uint32))


def test_no_device_error_recorded():
    assert _lib.device_error() == 0


@pytest.mark.parametrize("K,N,M", [(4096, 128256, 4), (1536, 151936, 8)])
def test_multiwave_ring_reuse_repeated(K, N, M):
    """Multi-wave grids whose per-tile weight rings wrap: 40 graph replays
    give bit-identical outputs, column slices match the oracle, no bounded
    wait gives up and the split-K workspace is left zeroed."""
    g = torch.Generator(device="cuda").manual_seed(K + M + 8)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).half()
    w_q, scale = w8a16_quantize_cuda(w)
    del w
    plan = _lib.gemv_plan(8, M, N, K)
    # the per-tile rings wrap: fewer slots than the stages a CTA streams
    blocks = -(-(-(-N // 16)) // plan["tiles_per_cta"])
    per_cta = -(-blocks // (plan["ctas"] // (plan["k_splits"] * plan["batch_chunks"])))
    stages_per_tile = -(-plan["kblocks_per_split"] // plan["kblocks_per_stage"]) * per_cta
    assert plan["stages"] < plan["tiles_per_cta"] * stages_per_tile
    x = make_x(M, K, seed=K + 1).cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ref = w8a16_linear(x, w_q, scale)
        torch.cuda.synchronize()
        out = torch.empty_like(ref)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for _ in range(3):
                w8a16_linear(x, w_q, scale, out=out)
        for _ in range(40):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
    assert _lib.device_error() == 0
    xn = x.cpu().numpy()
    for a, b in ((0, 512), (N - 512, N)):
        deq = orc.dequantize_int8(w_q[a:b].cpu().numpy(), scale[a:b].cpu().numpy())
        assert_parity(ref[:, a:b], orc.linear_f32(xn, deq, None), xn, deq, f"cols {a}:{b}")
    for buf in _launch._workspaces.values():
        assert int(buf.count_nonzero()) == 0
