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

from helpers import make_linear, make_x

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
