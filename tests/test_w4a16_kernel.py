"""W4A16 kernel parity on the GPU, through the reference-facing API and the C ABI.

Mirrors the reference's tests/test_w4a16_kernel.py (shapes incl. the awkward
(384, 100), M in {1, 7, 16, 100, 300}, bias on/off, leading dims, error and
byte bounds, half-step round trip) and adds the north-star tolerance against
the CPU oracle, both nibble layouts, benchmark configs 1/4 shapes, the device
nibble decoder / dequantizer / quantizer bit-exact against the oracle and
the reference's fixtures (every nibble value, incl. 0 = -8), determinism,
workspace hygiene and CUDA-graph capture.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import qlinear_oracle as orc
from qlinear import _lib
from qlinear.kernels import _launch
from qlinear.kernels.w4a16_matmul import (
    GROUP_SIZE, LAYOUT_ADJACENT, LAYOUT_SPLIT_HALF, dequantize_int4_cuda, unpack_int4_cuda,
    w4a16_linear, w4a16_quantize_cuda, w4a16_reference,
)
from qlinear.quantization.int4 import QuantizedLinearInt4

from helpers import assert_parity, make_linear, make_x

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="requires a CUDA GPU")]

GOLDEN = Path(__file__).resolve().parent / "golden"

LAYER_SHAPES = [
    (1536, 1536),
    (1536, 256),
    (1536, 8960),
    (8960, 1536),
    (384, 100),
]
M_VALUES = [1, 7, 16, 100, 300]


def _oracle(x, q):
    packed = q.weight_packed.cpu().numpy()
    scales = q.scales.cpu().numpy()
    deq = orc.dequantize_int4(packed, scales, q.layout)
    b = q.bias.cpu().numpy() if q.bias is not None else None
    K = packed.shape[1] * 2
    return orc.linear_f32(x.cpu().numpy().reshape(-1, K), deq, b), deq


def _raw_call(x, q, flags, ws=None):
    lib = _lib.load()
    N, half_k = q.weight_packed.shape
    K = half_k * 2
    x2 = x.reshape(-1, K).contiguous()
    out = torch.empty((x2.shape[0], N), dtype=torch.float16, device=x.device)
    st = lib.ql_w4a16_linear(
        x2.data_ptr(), 0, q.weight_packed.data_ptr(), q.layout, q.scales.data_ptr(),
        q.bias.data_ptr() if q.bias is not None else None,
        _launch.dtype_code(q.bias.dtype) if q.bias is not None else 0,
        out.data_ptr(), x2.shape[0], N, K, x2.stride(0), q.weight_packed.stride(0), q.scales.stride(0),
        out.stride(0), ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        flags, torch.cuda.current_stream().cuda_stream)
    _lib.check(st)
    return out


@pytest.mark.parametrize("K,N", LAYER_SHAPES)
@pytest.mark.parametrize("M", M_VALUES)
@pytest.mark.parametrize("bias", [False, True])
def test_kernel_matches_dequantized_reference(K, N, M, bias):
    lin = make_linear(K, N, bias)
    q = QuantizedLinearInt4.from_linear(lin)
    x = make_x(M, K, seed=1)
    y32, deq = _oracle(x, q)
    q = q.cuda()
    xd = x.cuda()
    out = w4a16_linear(xd, q.weight_packed, q.scales, q.bias)
    assert out.shape == (M, N) and out.dtype == torch.float16
    assert not torch.isnan(out).any()
    assert_parity(out, y32, x.numpy(), deq, f"w4 K{K} N{N} M{M} bias{bias}")
    ref = w4a16_reference(xd, q.weight_packed, q.scales, q.bias)
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("K,N", [(1536, 8960), (8960, 1536)])
@pytest.mark.parametrize("M", [1, 8, 32])
@pytest.mark.parametrize("layout", [LAYOUT_SPLIT_HALF, LAYOUT_ADJACENT])
def test_baseline_config1(K, N, M, layout):
    """benchmark config 1: x [M,K] N(0,1), W N(0,0.02), group-128 int4; the
    reference format and the [-8,7] / low-nibble-even variant."""
    lin = make_linear(K, N, bias=False, std=0.02, seed=0)
    qmin = -7 if layout == LAYOUT_SPLIT_HALF else -8
    q = QuantizedLinearInt4.from_linear(lin, qmin=qmin, layout=layout)
    x = make_x(M, K, seed=1)
    y32, deq = _oracle(x, q)
    q = q.cuda()
    out = q(x.cuda())
    assert_parity(out, y32, x.numpy(), deq, f"config1 K{K} N{N} M{M} layout{layout}")


def test_leading_dims_preserved():
    lin = make_linear(1536, 256, bias=False)
    q = QuantizedLinearInt4.from_linear(lin).cuda()
    x = make_x(None, 1536, seed=5, lead=(2, 5)).cuda()
    out = q(x)
    assert out.shape == (2, 5, 256)
    ref = w4a16_reference(x.reshape(-1, 1536), q.weight_packed, q.scales).reshape(2, 5, 256)
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("K,N,M", [(128, 1, 1), (128, 17, 3), (384, 33, 9), (640, 48, 64),
                                   (4096, 14336, 2), (14336, 4096, 1), (256, 5, 17)])
@pytest.mark.parametrize("layout", [LAYOUT_SPLIT_HALF, LAYOUT_ADJACENT])
def test_ragged_shapes(K, N, M, layout):
    lin = make_linear(K, N, bias=True, seed=K + N, std=0.02)
    q = QuantizedLinearInt4.from_linear(lin, layout=layout)
    x = make_x(M, K, seed=M)
    y32, deq = _oracle(x, q)
    out = q.cuda()(x.cuda())
    assert_parity(out, y32, x.numpy(), deq, f"ragged K{K} N{N} M{M} layout{layout}")


@pytest.mark.parametrize("K,N,M", [(1536, 8960, 1), (8960, 1536, 4), (384, 100, 16)])
@pytest.mark.parametrize("layout", [LAYOUT_SPLIT_HALF, LAYOUT_ADJACENT])
def test_portable_kernel_matches(K, N, M, layout):
    lin = make_linear(K, N, bias=True, seed=11)
    q = QuantizedLinearInt4.from_linear(lin, layout=layout)
    x = make_x(M, K, seed=12)
    y32, deq = _oracle(x, q)
    out = _raw_call(x.cuda(), q.cuda(), _lib.QL_FLAG_FORCE_GENERIC)
    assert_parity(out, y32, x.numpy(), deq, "generic")


@pytest.mark.parametrize("K,N,M", [(8960, 1536, 1), (1536, 8960, 8), (8960, 1536, 32)])
def test_deterministic_pdl_and_workspace_clean(K, N, M):
    lin = make_linear(K, N, bias=True, seed=21)
    q = QuantizedLinearInt4.from_linear(lin).cuda()
    x = make_x(M, K, seed=22).cuda()
    a = q(x)
    b = q(x)
    assert torch.equal(a, b)
    need = _lib.load().ql_w4a16_workspace_size(M, N, K)
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    c = _raw_call(x, q, 0, ws)
    d = _raw_call(x, q, _lib.QL_FLAG_PDL, ws)
    e = _raw_call(x, q, 0, None)
    torch.cuda.synchronize()
    assert torch.equal(a, c) and torch.equal(a, d)
    y32, deq = _oracle(x, q)
    assert_parity(e, y32, x.cpu().numpy(), deq, "no-ws")
    assert int(ws.count_nonzero()) == 0
    for buf in _launch._workspaces.values():
        assert int(buf.count_nonzero()) == 0


def test_lm_head_shape_config4():
    """benchmark config 4 lm_head 1536 -> 151936, M = 1 and 16 (one GPU)."""
    K, N = 1536, 151936
    lin = make_linear(K, N, bias=False, std=0.02, seed=4)
    q = QuantizedLinearInt4.from_linear(lin)
    qd = q.cuda()
    for M in (1, 16):
        x = make_x(M, K, seed=M)
        y32, deq = _oracle(x, q)
        assert_parity(qd(x.cuda()), y32, x.numpy(), deq, f"lm_head M{M}")


def test_cuda_graph_capture_matches_eager():
    shapes = [(1536, 1536), (1536, 256), (1536, 8960), (8960, 1536)]
    mods = [QuantizedLinearInt4.from_linear(make_linear(K, N, bias=(N == 256), seed=K + N)).cuda()
            for K, N in shapes]
    xs = [make_x(4, K, seed=K).cuda() for K, _ in shapes]
    eager = [m(x) for m, x in zip(mods, xs)]
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for m, x in zip(mods, xs):
            m(x)
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


def test_quantization_error_bounded_vs_fp16():
    lin = make_linear(1536, 1536, bias=False).cuda()
    q = QuantizedLinearInt4.from_linear(lin)
    x = make_x(64, 1536, seed=2).cuda()
    exact = torch.nn.functional.linear(x, lin.weight).float()
    approx = q(x).float()
    rel = (approx - exact).norm() / exact.norm()
    assert rel.item() < 0.2


def test_weight_roundtrip_within_half_step():
    lin = make_linear(1536, 300, bias=False).cuda()
    q = QuantizedLinearInt4.from_linear(lin)
    dq = q.dequantized_weight(torch.float32)
    step = q.scales.float().t().repeat_interleave(GROUP_SIZE, dim=1)
    err = (dq - lin.weight.float()).abs()
    assert (err <= 0.51 * step + 1e-6).all()


def test_device_decoder_bitexact_all_nibbles():
    """The GEMV's register decoder (via ql_w4a16_dequantize / unpack) against
    the reference's dequantize_int4 on every nibble value in both positions."""
    z = np.load(GOLDEN / "int4_cases.npz")
    for name in ("allnibbles", "k384_n100_m7_bias", "k256_n64_m3", "k1536_n40_m2_bias", "ties"):
        packed = torch.from_numpy(z[f"{name}/packed"]).cuda()
        scales = torch.from_numpy(z[f"{name}/scales"]).cuda()
        deq = dequantize_int4_cuda(packed, scales)
        assert np.array_equal(deq.cpu().numpy().view(np.uint32), z[f"{name}/deq"].view(np.uint32)), name
        un = unpack_int4_cuda(packed)
        assert np.array_equal(un.cpu().numpy(), orc.unpack_int4(z[f"{name}/packed"])), name
    # adjacent layout: same nibbles re-packed
    q = z["allnibbles/q"]
    adj = torch.from_numpy(orc.pack_int4_adjacent(q)).cuda()
    scales = torch.from_numpy(z["allnibbles/scales"]).cuda()
    deq = dequantize_int4_cuda(adj, scales, LAYOUT_ADJACENT)
    assert np.array_equal(deq.cpu().numpy().view(np.uint32), z["allnibbles/deq"].view(np.uint32))
    assert np.array_equal(unpack_int4_cuda(adj, LAYOUT_ADJACENT).cpu().numpy(), q)


def test_device_quantizer_bitexact():
    z = np.load(GOLDEN / "int4_cases.npz")
    for name in ("k384_n100_m7_bias", "k256_n64_m3", "k1536_n40_m2_bias", "ties"):
        w = torch.from_numpy(z[f"{name}/w"]).cuda()
        packed, scales = w4a16_quantize_cuda(w)
        assert np.array_equal(packed.cpu().numpy(), z[f"{name}/packed"]), name
        assert np.array_equal(scales.cpu().numpy().view(np.uint16), z[f"{name}/scales"].view(np.uint16)), name
    lin = make_linear(8960, 1536, bias=False, std=0.02, seed=3)
    for layout, qmin in ((LAYOUT_SPLIT_HALF, -7), (LAYOUT_ADJACENT, -8)):
        pr, sr = orc.quantize_int4_groups(lin.weight.detach().numpy(), qmin=qmin, layout=layout)
        q = QuantizedLinearInt4.from_linear(lin.cuda(), qmin=qmin, layout=layout)
        assert np.array_equal(q.weight_packed.cpu().numpy(), pr)
        assert np.array_equal(q.scales.cpu().numpy().view(np.uint16), sr.view(np.uint16))
        lin = lin.cpu()


def test_no_device_error_recorded():
    assert _lib.device_error() == 0


def test_device_quantizer_more_rows_than_grid_y():
    """lm_head-sized row counts (> 65535) go through the grid-stride row loop."""
    g = torch.Generator().manual_seed(13)
    w = (torch.randn(70001, 128, generator=g) * 0.02).half()
    pr, sr = orc.quantize_int4_groups(w.numpy())
    packed, scales = w4a16_quantize_cuda(w.cuda())
    assert np.array_equal(packed.cpu().numpy(), pr)
    assert np.array_equal(scales.cpu().numpy().view(np.uint16), sr.view(np.uint16))


@pytest.mark.parametrize("K,N,M", [(4096, 128256, 6), (1536, 151936, 8), (1536, 151936, 12)])
def test_multiwave_ring_reuse_repeated(K, N, M):
    """Multi-wave grids whose per-tile weight rings wrap (single-k-block
    stages, split-K for K=4096): 40 graph replays give bit-identical
    outputs, column slices match the oracle, no bounded wait gives up and
    the split-K workspace is left zeroed."""
    g = torch.Generator(device="cuda").manual_seed(K + M)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).half()
    packed, scales = w4a16_quantize_cuda(w)
    del w
    plan = _lib.gemv_plan(4, M, N, K)
    # the per-tile rings wrap: fewer slots than the stages a CTA streams
    blocks = -(-(-(-N // 16)) // plan["tiles_per_cta"])
    per_cta = -(-blocks // (plan["ctas"] // (plan["k_splits"] * plan["batch_chunks"])))
    stages_per_tile = -(-plan["kblocks_per_split"] // plan["kblocks_per_stage"]) * per_cta
    assert plan["stages"] < plan["tiles_per_cta"] * stages_per_tile
    x = make_x(M, K, seed=K).cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ref = w4a16_linear(x, packed, scales)
        torch.cuda.synchronize()
        out = torch.empty_like(ref)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for _ in range(3):
                w4a16_linear(x, packed, scales, out=out)
        for _ in range(40):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
    assert _lib.device_error() == 0
    xn = x.cpu().numpy()
    for a, b in ((0, 512), (N - 512, N)):
        p_np = packed[a:b].cpu().numpy()
        s_np = scales[:, a:b].cpu().numpy()
        deq = orc.dequantize_int4(p_np, s_np, 0)
        assert_parity(ref[:, a:b], orc.linear_f32(xn, deq, None), xn, deq, f"cols {a}:{b}")
    for buf in _launch._workspaces.values():
        assert int(buf.count_nonzero()) == 0
