"""Tensor-core (tcgen05) GEMM path parity on the GPU.

The path is forced with QL_FLAG_FORCE_GEMM so every batch size exercises it,
and compared with the CPU oracle under the north-star tolerance.  int4
weights enter the MMA as fp16((q-8)*scale) (one rounding per weight), int8
weights exactly with the row scale applied in fp32 in the epilogue.
"""
import numpy as np
import pytest
import torch

from oracle import qlinear_oracle as orc
from qlinear import _lib
from qlinear.kernels import _launch
from qlinear.kernels.w4a16_matmul import LAYOUT_ADJACENT, LAYOUT_SPLIT_HALF
from qlinear.quantization.int4 import QuantizedLinearInt4
from qlinear.quantization.int8 import QuantizedLinearInt8

from helpers import assert_parity, make_linear, make_x

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="requires a CUDA GPU")]


def _call(x, q, flags, ws=None):
    lib = _lib.load()
    wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    dev = x.device
    stream = torch.cuda.current_stream(dev).cuda_stream
    if isinstance(q, QuantizedLinearInt4):
        N, half_k = q.weight_packed.shape
        K = half_k * 2
        out = torch.empty((x.shape[0], N), dtype=torch.float16, device=dev)
        st = lib.ql_w4a16_linear(
            x.data_ptr(), 0, q.weight_packed.data_ptr(), q.layout, q.scales.data_ptr(),
            q.bias.data_ptr() if q.bias is not None else None, 0,
            out.data_ptr(), x.shape[0], N, K, _launch.ld(x, K), _launch.ld(q.weight_packed, K // 2),
            _launch.ld(q.scales, N), _launch.ld(out, N), wsp, wsn, flags, stream)
    else:
        N, K = q.weight_q.shape
        out = torch.empty((x.shape[0], N), dtype=torch.float16, device=dev)
        st = lib.ql_w8a16_linear(
            x.data_ptr(), 0, q.weight_q.data_ptr(), q.scale.data_ptr(), _launch.dtype_code(q.scale.dtype),
            q.bias.data_ptr() if q.bias is not None else None, 0,
            out.data_ptr(), x.shape[0], N, K, _launch.ld(x, K), _launch.ld(q.weight_q, K), _launch.ld(out, N),
            wsp, wsn, flags, stream)
    _lib.check(st)
    return out


def _oracle4(x, q):
    deq = orc.dequantize_int4(q.weight_packed.cpu().numpy(), q.scales.cpu().numpy(), q.layout)
    b = q.bias.cpu().numpy() if q.bias is not None else None
    return orc.linear_f32(x.cpu().numpy(), deq, b), deq


def _oracle8(x, q):
    deq = orc.dequantize_int8(q.weight_q.cpu().numpy(), q.scale.cpu().numpy())
    b = q.bias.cpu().numpy() if q.bias is not None else None
    return orc.linear_f32(x.cpu().numpy(), deq, b), deq


@pytest.mark.parametrize("K,N", [(128, 128), (256, 100), (1536, 256), (1536, 8960), (8960, 1536)])
@pytest.mark.parametrize("M", [1, 16, 33, 64, 100, 300])
@pytest.mark.parametrize("layout", [LAYOUT_SPLIT_HALF, LAYOUT_ADJACENT])
def test_w4_gemm_forced(K, N, M, layout):
    lin = make_linear(K, N, bias=True, std=0.02, seed=K + N + M)
    q = QuantizedLinearInt4.from_linear(lin, layout=layout)
    x = make_x(M, K, seed=M + 3)
    y32, deq = _oracle4(x, q)
    out = _call(x.cuda(), q.cuda(), _lib.QL_FLAG_FORCE_GEMM)
    assert_parity(out, y32, x.numpy(), deq, f"gemm w4 K{K} N{N} M{M} layout{layout}")


@pytest.mark.parametrize("K,N", [(128, 128), (384, 100), (1536, 256), (1536, 8960), (8960, 1536)])
@pytest.mark.parametrize("M", [1, 16, 33, 64, 100, 300])
def test_w8_gemm_forced(K, N, M):
    lin = make_linear(K, N, bias=True, std=0.02, seed=K + N + M)
    q = QuantizedLinearInt8.from_linear(lin)
    x = make_x(M, K, seed=M + 5)
    y32, deq = _oracle8(x, q)
    out = _call(x.cuda(), q.cuda(), _lib.QL_FLAG_FORCE_GEMM)
    assert_parity(out, y32, x.numpy(), deq, f"gemm w8 K{K} N{N} M{M}")


@pytest.mark.parametrize("wbits", [4, 8])
def test_gemm_prefill_shapes(wbits):
    """benchmark config 3 shape class at a size the oracle finishes quickly."""
    for K, N, M in ((4096, 1024, 512), (2048, 4096, 256)):
        lin = make_linear(K, N, bias=False, std=0.02, seed=K ^ N)
        x = make_x(M, K, seed=M)
        if wbits == 4:
            q = QuantizedLinearInt4.from_linear(lin)
            y32, deq = _oracle4(x, q)
        else:
            q = QuantizedLinearInt8.from_linear(lin)
            y32, deq = _oracle8(x, q)
        out = q.cuda()(x.cuda())          # default dispatch: M >= 48 takes the tensor-core path
        assert_parity(out, y32, x.numpy(), deq, f"prefill w{wbits} K{K} N{N} M{M}")


@pytest.mark.parametrize("wbits", [4, 8])
@pytest.mark.parametrize("M,K,N", [(2048, 14336, 4096), (8192, 4096, 14336), (8192, 14336, 4096),
                                   (2048, 1536, 8960)])
def test_prefill_full_size(M, K, N, wbits):
    """Benchmark config 3 at its real sizes (the 192-row int8 tile from M =
    1024, multi-wave grids): weights quantized on the device, the whole
    product on the GPU through the default dispatch, the oracle on row and
    column slices at both ends (cheap on the CPU), bit-identical on a second
    run."""
    g = torch.Generator(device="cuda").manual_seed(M + K + N + wbits)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).half()
    lin = torch.nn.Linear(K, N, bias=False, device="cuda", dtype=torch.float16)
    with torch.no_grad():
        lin.weight.copy_(w)
    del w
    q = QuantizedLinearInt4.from_linear(lin) if wbits == 4 else QuantizedLinearInt8.from_linear(lin)
    del lin
    x = torch.randn(M, K, generator=g, device="cuda").half()
    y = q(x)
    y2 = q(x)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    assert bool(torch.isfinite(y).all())
    rows = np.r_[0:48, M - 48:M]
    xs = x[rows].cpu().numpy()
    for a, b in ((0, 384), (N - 384, N)):
        if wbits == 4:
            deq = orc.dequantize_int4(q.weight_packed[a:b].cpu().numpy(), q.scales[:, a:b].cpu().numpy())
        else:
            deq = orc.dequantize_int8(q.weight_q[a:b].cpu().numpy(), q.scale[a:b].cpu().numpy())
        y32 = orc.linear_f32(xs, deq, None)
        assert_parity(y[rows][:, a:b], y32, xs, deq, f"prefill w{wbits} M{M} K{K} N{N} cols {a}:{b}")
    assert _lib.device_error() == 0


def test_gemm_unsupported_shape_is_reported():
    """int8 with K % 128 != 0 cannot take the tensor-core path; forcing it is
    an error status, not a fallback."""
    lin = make_linear(144, 32, bias=False)
    q = QuantizedLinearInt8.from_linear(lin).cuda()
    x = make_x(70, 144).cuda()
    with pytest.raises(_lib.QLinearError):
        _call(x, q, _lib.QL_FLAG_FORCE_GEMM)
    # the default dispatch handles it (decode kernel), correctly
    y32, deq = _oracle8(x, q)
    assert_parity(q(x), y32, x.cpu().numpy(), deq, "k144 default")


@pytest.mark.parametrize("K,N", [(8960, 1536), (1536, 8960), (4096, 256), (2048, 1000)])
@pytest.mark.parametrize("M", [1, 16, 32, 33, 64, 200])
@pytest.mark.parametrize("wbits", [4, 8])
def test_gemm_split_k(K, N, M, wbits):
    """Grids with fewer tiles than SMs split K across the CTAs of a cluster
    (reduced through distributed shared memory: pushed into the summing
    member for 16/32-row tiles, pulled for wider ones): parity,
    bit-identical repeat, a caller's workspace left untouched and none
    requested."""
    lin = make_linear(K, N, bias=True, std=0.02, seed=K + N + M + wbits)
    x = make_x(M, K, seed=M + 11)
    if wbits == 4:
        q = QuantizedLinearInt4.from_linear(lin)
        y32, deq = _oracle4(x, q)
    else:
        q = QuantizedLinearInt8.from_linear(lin)
        y32, deq = _oracle8(x, q)
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")   # room for any split
    qd, xd = q.cuda(), x.cuda()
    a = _call(xd, qd, _lib.QL_FLAG_FORCE_GEMM, ws)
    b = _call(xd, qd, _lib.QL_FLAG_FORCE_GEMM | _lib.QL_FLAG_PDL, ws)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert int(ws.count_nonzero()) == 0
    c = _call(xd, qd, _lib.QL_FLAG_FORCE_GEMM)                     # no workspace: same plan, same bits
    assert torch.equal(a, c)
    assert_parity(a, y32, x.numpy(), deq, f"split-K w{wbits} K{K} N{N} M{M}")


def test_gemm_dispatch_needs_no_workspace():
    lib = _lib.load()
    for M, N, K in ((64, 8960, 1536), (64, 1536, 8960), (512, 4096, 14336), (32, 151936, 1536), (16, 1536, 8960)):
        assert lib.ql_w4a16_workspace_size(M, N, K) == 0
        assert lib.ql_w8a16_workspace_size(M, N, K) == 0


def test_gemm_no_device_error():
    assert _lib.device_error() == 0
