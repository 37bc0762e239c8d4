"""Small-batch tensor-core kernel (qdec_kernel, tcgen05 with the decoded
weights in TMEM) parity on the GPU.

The path is forced with QL_FLAG_FORCE_TCDEC so every supported shape runs
it, and compared with the CPU oracle (the reference's dequantize-then-fp32
linear) under the north-star tolerance.  The kernel decodes int4 codes to
1024 + q (low nibbles) and 1024 + 16 q (high nibbles, activations staged
times 1/16) and subtracts the offset through per-group activation sums,
int8 to 1152 + b with one correction per row of the batch; these tests pin
that arithmetic against the oracle on seeded inputs, both int4 nibble
layouts, fp16 and fp32 scales / biases, K-splits across a cluster, ragged N
and M, strided operands, determinism and CUDA-graph replay.
"""
import numpy as np
import pytest
import torch

from qlinear import _lib
from qlinear.kernels.w4a16_matmul import LAYOUT_ADJACENT, LAYOUT_SPLIT_HALF
from qlinear.quantization.int4 import QuantizedLinearInt4
from qlinear.quantization.int8 import QuantizedLinearInt8

from helpers import assert_parity, make_linear, make_x
from test_gemm_path import _call, _oracle4, _oracle8

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="requires a CUDA GPU")]

FORCE = _lib.QL_FLAG_FORCE_TCDEC | _lib.QL_FLAG_PDL

SHAPES = [(128, 128), (256, 100), (1536, 256), (1536, 1536), (1536, 8960), (8960, 1536), (4096, 1000),
          (14336, 512)]


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 3, 8, 16, 17, 32])
@pytest.mark.parametrize("layout", [LAYOUT_SPLIT_HALF, LAYOUT_ADJACENT])
def test_w4_tcdec_forced(K, N, M, layout):
    lin = make_linear(K, N, bias=True, std=0.02, seed=K + N + M)
    q = QuantizedLinearInt4.from_linear(lin, layout=layout)
    x = make_x(M, K, seed=M + 5)
    y32, deq = _oracle4(x, q)
    out = _call(x.cuda(), q.cuda(), FORCE)
    assert_parity(out, y32, x.numpy(), deq, f"tcdec w4 K{K} N{N} M{M} layout{layout}")
    assert _lib.device_error() == 0


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 5, 16, 32])
@pytest.mark.parametrize("scale_dtype", [torch.float32, torch.float16])
def test_w8_tcdec_forced(K, N, M, scale_dtype):
    lin = make_linear(K, N, bias=True, std=0.02, seed=K + N + 2 * M)
    q = QuantizedLinearInt8.from_linear(lin)
    q.scale = q.scale.to(scale_dtype)
    x = make_x(M, K, seed=M + 9)
    y32, deq = _oracle8(x, q)
    out = _call(x.cuda(), q.cuda(), FORCE)
    assert_parity(out, y32, x.numpy(), deq, f"tcdec w8 K{K} N{N} M{M} scale {scale_dtype}")
    assert _lib.device_error() == 0


def test_tcdec_plan_splits_k_over_a_cluster():
    """Narrow layers split K across a cluster (reduced through distributed
    shared memory); wide ones do not."""
    down = _lib.tcdec_plan(4, 1, 1536, 8960)
    assert down is not None and down["k_splits"] > 1 and down["tiles"] == 12
    head = _lib.tcdec_plan(4, 1, 151936, 1536)
    assert head is not None and head["k_splits"] == 1
    assert _lib.tcdec_plan(4, 33, 1536, 1536) is None          # more than 32 rows: not this kernel
    assert _lib.tcdec_plan(8, 4, 1536, 1000) is None            # K not a multiple of 128


@pytest.mark.parametrize("wbits", [4, 8])
def test_tcdec_fp32_bias_and_strides(wbits):
    """fp32 bias, x and out with row strides larger than their rows."""
    K, N, M = 1536, 640, 6
    lin = make_linear(K, N, bias=True, std=0.02, seed=wbits)
    q = (QuantizedLinearInt4.from_linear(lin) if wbits == 4 else QuantizedLinearInt8.from_linear(lin)).cuda()
    xs = make_x(M, K + 64, seed=4).cuda()
    x = xs[:, 32:32 + K]
    bias32 = q.bias.float()
    out_big = torch.full((M, N + 40), 3.0, dtype=torch.float16, device="cuda")
    out = out_big[:, 8:8 + N]
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    if wbits == 4:
        st = lib.ql_w4a16_linear(x.data_ptr(), 0, q.weight_packed.data_ptr(), q.layout, q.scales.data_ptr(),
                                 bias32.data_ptr(), _lib.QL_DTYPE_F32, out.data_ptr(), M, N, K, x.stride(0),
                                 K // 2, N, out.stride(0), None, 0, FORCE, stream)
        y32, deq = _oracle4(x.cpu(), q.cpu())
    else:
        st = lib.ql_w8a16_linear(x.data_ptr(), 0, q.weight_q.data_ptr(), q.scale.data_ptr(), _lib.QL_DTYPE_F32,
                                 bias32.data_ptr(), _lib.QL_DTYPE_F32, out.data_ptr(), M, N, K, x.stride(0), K,
                                 out.stride(0), None, 0, FORCE, stream)
        y32, deq = _oracle8(x.cpu(), q.cpu())
    _lib.check(st)
    torch.cuda.synchronize()
    assert_parity(out, y32, x.cpu().numpy(), deq, f"tcdec w{wbits} strided")
    assert bool((out_big[:, :8] == 3.0).all()) and bool((out_big[:, 8 + N:] == 3.0).all())


@pytest.mark.parametrize("wbits,M,N,K", [(4, 1, 8960, 1536), (4, 8, 1536, 8960), (8, 1, 151936 // 4, 1536),
                                         (4, 16, 28672 // 8, 4096)])
def test_tcdec_deterministic_and_graph_replay(wbits, M, N, K):
    """Bit-identical outputs run to run and from 20 CUDA-graph replays; the
    K-split reduction sums in a fixed order."""
    g = torch.Generator(device="cuda").manual_seed(N + K)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).half()
    lin = torch.nn.Linear(K, N, bias=False, device="cuda", dtype=torch.float16)
    with torch.no_grad():
        lin.weight.copy_(w)
    q = QuantizedLinearInt4.from_linear(lin) if wbits == 4 else QuantizedLinearInt8.from_linear(lin)
    x = torch.randn(M, K, generator=g, device="cuda").half()
    ref = _call(x, q, FORCE)
    torch.cuda.synchronize()
    assert torch.equal(_call(x, q, FORCE), ref)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _call(x, q, FORCE)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            outs = [_call(x, q, FORCE) for _ in range(3)]
        for _ in range(20):
            for o in outs:
                o.zero_()
            graph.replay()
            torch.cuda.synchronize()
            for o in outs:
                assert torch.equal(o, ref)
    assert _lib.device_error() == 0
    # oracle on a column slice at each end
    from oracle import qlinear_oracle as orc
    xn = x.cpu().numpy()
    for a, b in ((0, 256), (N - 256, N)):
        if wbits == 4:
            deq = orc.dequantize_int4(q.weight_packed[a:b].cpu().numpy(), q.scales[:, a:b].cpu().numpy())
        else:
            deq = orc.dequantize_int8(q.weight_q[a:b].cpu().numpy(), q.scale[a:b].cpu().numpy())
        assert_parity(ref[:, a:b], orc.linear_f32(xn, deq, None), xn, deq, f"cols {a}:{b}")


def test_tcdec_every_nibble_value():
    """Codes 0..15 in every position (0 = -8 is never produced by the
    reference's quantizer but decodes exactly): weights with known codes and
    scales against the oracle."""
    K, N, M = 256, 256, 4
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 16, size=(N, K), dtype=np.uint8)
    codes[:16, :16] = np.arange(16, dtype=np.uint8)[None, :]
    from qlinear.kernels.w4a16_matmul import pack_int4
    for layout in (LAYOUT_SPLIT_HALF, LAYOUT_ADJACENT):
        cq = torch.from_numpy(codes)
        packed = pack_int4(cq) if layout == LAYOUT_SPLIT_HALF else (cq[:, 0::2] | (cq[:, 1::2] << 4)).contiguous()
        scales = torch.from_numpy((rng.random((K // 128, N)) * 0.01 + 0.001).astype(np.float16))
        q = QuantizedLinearInt4(packed, scales, None, layout=layout)
        x = make_x(M, K, seed=7)
        y32, deq = _oracle4(x, q)
        out = _call(x.cuda(), q.cuda(), FORCE)
        assert_parity(out, y32, x.numpy(), deq, f"nibbles layout {layout}")
