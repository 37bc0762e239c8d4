"""Row argmax through packed keys (ql_argmax_rows_f16) on the GPU.

Must equal torch.argmax on the same fp16 logits (first index among equal
maxima), for vectorised and unaligned rows, with column offsets, and after
combining the keys of column shards.
"""
import pytest
import torch

from qlinear.kernels.argmax import argmax_f16, argmax_keys, combine_keys, key_columns, key_values
from qlinear.quantization.int4 import QuantizedLinearInt4
from qlinear.sharded import ShardedQuantizedLinear

from helpers import linear_unsplit, make_linear, make_x

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="requires a CUDA GPU")]


@pytest.mark.parametrize("M,N", [(1, 151936), (16, 18992), (64, 16032), (3, 37), (5, 8), (2, 100001)])
def test_argmax_matches_torch(M, N):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    y = (torch.randn(M, N, generator=g, device="cuda") * 4).half()
    # plant exact ties of the row maximum at two columns
    for m in range(M):
        a, b = (m * 13) % N, (m * 29 + N // 2) % N
        y[m, a] = y[m, b] = 60000.0
    assert torch.equal(argmax_f16(y), torch.argmax(y, dim=-1))
    keys = argmax_keys(y)
    assert torch.equal(key_values(keys), y.max(dim=-1).values)


def test_argmax_special_values():
    y = torch.tensor([[-1.0, -0.0, 0.0, -2.0], [float("-inf"), -65504.0, float("-inf"), -7.0],
                      [1.0, float("nan"), 3.0, float("nan")]], dtype=torch.float16, device="cuda")
    assert key_columns(argmax_keys(y)).tolist() == [1, 3, 1]          # -0 == +0 (first), NaN is maximal


def test_sharded_keys_combine_to_full_argmax():
    g = torch.Generator(device="cuda").manual_seed(3)
    y = torch.randn(8, 10000, generator=g, device="cuda").half()
    y[:, 4000] = y[:, 9000] = 100.0                                     # tie across shards
    edges = [0, 2500, 5000, 7500, 10000]
    parts = torch.stack([argmax_keys(y[:, a:b], a) for a, b in zip(edges[:-1], edges[1:])])
    assert torch.equal(key_columns(combine_keys(parts, 0)), torch.argmax(y, dim=-1))


def test_sharded_module_argmax_single_rank():
    lin = make_linear(1536, 4099, bias=True, std=0.02, seed=9)
    q = QuantizedLinearInt4.from_linear(lin).cuda()
    sh = ShardedQuantizedLinear.from_quantized(q, 0, 1)
    x = make_x(5, 1536, seed=4).cuda()
    assert torch.equal(sh.argmax(x), torch.argmax(q(x), dim=-1))


def test_exchange_single_rank_matches_torch_and_replays():
    """World of one: the fused kernel's own push/flag/combine path, eagerly
    and from a CUDA graph replayed several times (epochs advance)."""
    from qlinear.p2p import PeerExchange
    px = PeerExchange(0, 1, max_m=16)
    try:
        g = torch.Generator(device="cuda").manual_seed(1)
        y = torch.randn(16, 30000, generator=g, device="cuda").half()
        y[:, 123] = y[:, 29000] = 50.0
        want = torch.argmax(y, dim=-1)
        assert torch.equal(px.argmax(y, 0), want)
        assert torch.equal(px.argmax(y[:5], 0), want[:5])
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                out = px.argmax(y, 0)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(5):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, want)
        del graph
        from qlinear import _lib
        assert _lib.device_error() == 0
    finally:
        px.close()


@pytest.mark.parametrize("wbits,M,K,N,bias,off", [(4, 1, 1536, 18992, False, 0), (4, 3, 1536, 4099, True, 77),
                                                    (8, 1, 1536, 18992, False, 5), (8, 8, 4096, 16032, True, 0),
                                                    (4, 8, 4096, 16032, False, 112224)])
def test_linear_argmax_fused_single_rank(wbits, M, K, N, bias, off):
    """The decode kernel's greedy-head epilogue (one launch: linear, keys,
    exchange) equals torch.argmax over the same kernel's fp16 outputs, for
    both formats, masked tail tiles, bias and column offsets; mixed with the
    unfused exchange and replayed from a CUDA graph (epochs advance)."""
    from qlinear import _lib
    from qlinear.p2p import PeerExchange
    from qlinear.quantization.int8 import QuantizedLinearInt8
    lin = make_linear(K, N, bias=bias, std=0.02, seed=N + M)
    q = (QuantizedLinearInt4 if wbits == 4 else QuantizedLinearInt8).from_linear(lin).cuda()
    x = make_x(M, K, seed=M + 1).cuda()
    px = PeerExchange(0, 1, max_m=8)
    try:
        assert _lib.load().ql_linear_argmax_supported(wbits, M, N, K) == 1
        want = torch.argmax(linear_unsplit(q, x), dim=-1) + off
        got = px.linear_argmax(x, q, off)
        assert got is not None and torch.equal(got, want)
        assert torch.equal(px.argmax(linear_unsplit(q, x), off), want)   # unfused exchange in between
        assert torch.equal(px.linear_argmax(x, q, off), want)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                out = px.linear_argmax(x, q, off)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(4):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, want)
        del graph
        assert _lib.device_error() == 0
    finally:
        px.close()


def test_linear_argmax_declines_unfused_shapes():
    """More than 8 rows (two batch tiles), more rows than the exchange
    holds, or a tensor-core shape: nothing is launched and None comes back."""
    from qlinear import _lib
    from qlinear.p2p import PeerExchange
    lin = make_linear(1536, 4096, bias=False, std=0.02, seed=2)
    q = QuantizedLinearInt4.from_linear(lin).cuda()
    px = PeerExchange(0, 1, max_m=64)
    try:
        assert _lib.load().ql_linear_argmax_supported(4, 12, 4096, 1536) == 0
        assert _lib.load().ql_linear_argmax_supported(4, 64, 4096, 1536) == 0
        assert px.linear_argmax(make_x(12, 1536, seed=3).cuda(), q, 0) is None
        assert px.linear_argmax(make_x(64, 1536, seed=3).cuda(), q, 0) is None
        x = make_x(12, 1536, seed=3).cuda()
        assert torch.equal(px.argmax(q(x), 0), torch.argmax(q(x), dim=-1))   # the exchange is still in step
    finally:
        px.close()


def test_exchange_peer_wait_is_bounded():
    """A peer that never signals: the kernel gives up after its wait budget
    (about 2 s), records QL_DEVICE_ERROR_PEER_WAIT and returns; the context
    stays usable.  The "peer" is a second local buffer nobody writes flags to."""
    import ctypes
    from qlinear import _lib
    lib = _lib.load()
    nbytes = lib.ql_xchg_buffer_bytes(2, 4)
    bufs = []
    for _ in range(2):
        p, h = ctypes.c_void_p(), (ctypes.c_char * 64)()
        _lib.check(lib.ql_xchg_alloc(nbytes, ctypes.byref(p), h))
        bufs.append(p.value)
    try:
        _lib.clear_device_error()
        peers = (ctypes.c_void_p * 2)(*bufs)
        y = torch.randn(4, 1000, device="cuda").half()
        out = torch.empty(4, dtype=torch.int64, device="cuda")
        _lib.check(lib.ql_argmax_exchange_f16(y.data_ptr(), 4, 1000, 1000, 0, 0, 2, 4, peers, out.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert _lib.device_error() == _lib.QL_DEVICE_ERROR_PEER_WAIT
        _lib.clear_device_error()
        assert torch.equal(argmax_f16(y), torch.argmax(y, dim=-1))     # context still fine
    finally:
        for b in bufs:
            lib.ql_xchg_free(b)


@pytest.mark.parametrize("wbits", [4, 8])
@pytest.mark.parametrize("K,N", [(1536, 151936), (4096, 128256)])
def test_greedy_head_against_oracle_on_lm_heads(wbits, K, N):
    """The greedy head (one launch: the decode kernel makes the keys and its
    last CTA combines them) on the real lm_head shapes, against the CPU
    oracle's fp32 product: every chosen column holds its row's maximum of
    the oracle's logits to within the north-star bound (two columns closer
    than that are a tie either path may break either way), and equals the
    argmax of the same plan's fp16 logits exactly."""
    import numpy as np
    from oracle import qlinear_oracle as orc
    from qlinear.p2p import PeerExchange
    from qlinear.quantization.int8 import QuantizedLinearInt8
    g = torch.Generator(device="cuda").manual_seed(K + wbits)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).half()
    lin = torch.nn.Linear(K, N, bias=False, device="cuda", dtype=torch.float16)
    with torch.no_grad():
        lin.weight.copy_(w)
    del w
    q = QuantizedLinearInt4.from_linear(lin) if wbits == 4 else QuantizedLinearInt8.from_linear(lin)
    del lin
    M = 4
    x = torch.randn(M, K, generator=g, device="cuda").half()
    px = PeerExchange(0, 1, max_m=8)
    ids = px.linear_argmax(x, q, 0)
    assert ids is not None, "a one-rank greedy head takes these shapes in one launch"
    same_plan = torch.argmax(linear_unsplit(q, x), dim=-1)
    torch.cuda.synchronize()
    px.close()
    assert torch.equal(ids, same_plan)
    if wbits == 4:
        deq = orc.dequantize_int4(q.weight_packed.cpu().numpy(), q.scales.cpu().numpy())
    else:
        deq = orc.dequantize_int8(q.weight_q.cpu().numpy(), q.scale.cpu().numpy())
    xn = x.cpu().numpy()
    y32 = orc.linear_f32(xn, deq, None)
    bound = orc.parity_bounds(xn, deq)[0]
    picked = y32[np.arange(M), ids.cpu().numpy()]
    assert (picked >= y32.max(axis=1) - 2 * bound).all(), (picked, y32.max(axis=1), bound)
