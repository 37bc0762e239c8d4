"""The no-allocation W4A16 entry point (ql_w4a16_linear_static_ws).

Some callers cannot allocate device memory when they call in — a framework
or host program that owns every device allocation, or a request path where a
cudaMalloc (which can synchronise the device) is not allowed — and have no
scratch buffer to pass.  This entry point takes its split-K scratch from a
fixed array inside the library instead.  These tests call it through the C
ABI, twice in a row on the same shape, and check it against the regular
entry point (which gets a zeroed torch workspace) and the CPU oracle.

The file is named to be collected last, and it does not depend on earlier
tests: the first call on the device sets the array up.
"""
import numpy as np
import pytest
import torch

from oracle import qlinear_oracle as orc
from qlinear import _lib
from qlinear.kernels import _launch
from qlinear.quantization.int4 import QuantizedLinearInt4

from helpers import assert_parity, make_linear, make_x

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="requires a CUDA GPU")]


def _args(x, q, out):
    N, half_k = q.weight_packed.shape
    K = half_k * 2
    return (x.data_ptr(), _lib.QL_DTYPE_F16, q.weight_packed.data_ptr(), q.layout, q.scales.data_ptr(),
            q.bias.data_ptr() if q.bias is not None else None, _lib.QL_DTYPE_F16, out.data_ptr(),
            x.shape[0], N, K, _launch.ld(x, K), _launch.ld(q.weight_packed, K // 2), _launch.ld(q.scales, N),
            _launch.ld(out, N))


@pytest.mark.parametrize("M,N,K", [(6, 1536, 8960), (7, 1536, 8960), (5, 1024, 14336), (1, 512, 14336)])
def test_static_scratch_matches_workspace_entry_point(M, N, K):
    """Decode-kernel shapes whose plan splits K (3 to 5 ways on a 148-SM
    B200, ql_gemv_plan) and so uses the scratch; the tensor-core kernel
    needs none (its splits reduce inside a cluster)."""
    lib = _lib.load()
    need = lib.ql_w4a16_workspace_size(M, N, K)
    assert 0 < need <= _lib.QL_STATIC_WS_BYTES, "shape must exercise the split-K scratch"
    lin = make_linear(K, N, bias=True, std=0.02, seed=M + N)
    q = QuantizedLinearInt4.from_linear(lin).cuda()
    x = make_x(M, K, seed=M).cuda()
    stream = torch.cuda.current_stream().cuda_stream

    ref = torch.empty((M, N), dtype=torch.float16, device="cuda")
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    _lib.check(lib.ql_w4a16_linear(*_args(x, q, ref), ws.data_ptr(), ws.numel(), 0, stream))

    outs = []
    for _ in range(2):                      # two calls in a row share the static scratch
        o = torch.empty((M, N), dtype=torch.float16, device="cuda")
        _lib.check(lib.ql_w4a16_linear_static_ws(*_args(x, q, o), 0, stream))
        outs.append(o)
    torch.cuda.synchronize()

    deq = orc.dequantize_int4(q.weight_packed.cpu().numpy(), q.scales.cpu().numpy())
    y32 = orc.linear_f32(x.cpu().numpy(), deq, q.bias.cpu().numpy())
    assert_parity(ref, y32, x.cpu().numpy(), deq, "workspace entry point")
    for o in outs:
        torch.testing.assert_close(o, ref, atol=2e-2, rtol=2e-2)
        assert_parity(o, y32, x.cpu().numpy(), deq, "static-scratch entry point")
    assert _lib.device_error() == 0


def test_static_scratch_rejects_oversized_plans():
    """A decode-kernel shape (fewer than 8 rows) whose K-split needs more
    scratch than the static array holds is refused before any launch.  The
    candidates' plans need 2.5 to 6.6 MiB on a 148-SM B200 (ql_gemv_plan);
    weights and scales are placeholders, since nothing may run."""
    lib = _lib.load()
    cands = [(7, 16384, 16384), (4, 8192, 57344), (7, 14336, 57344)]
    big = [c for c in cands if lib.ql_w4a16_workspace_size(*c) > _lib.QL_STATIC_WS_BYTES]
    assert big, "on a B200 these shapes plan a K-split larger than the static scratch"
    M, N, K = big[0]
    packed = torch.zeros((N, K // 2), dtype=torch.uint8, device="cuda")
    scales = torch.ones((K // 128, N), dtype=torch.float16, device="cuda")
    x = make_x(M, K).cuda()
    o = torch.full((M, N), 7.0, dtype=torch.float16, device="cuda")
    st = lib.ql_w4a16_linear_static_ws(x.data_ptr(), _lib.QL_DTYPE_F16, packed.data_ptr(), 0, scales.data_ptr(),
                                       None, _lib.QL_DTYPE_F16, o.data_ptr(), M, N, K, K, K // 2, N, N, 0,
                                       torch.cuda.current_stream().cuda_stream)
    assert st == _lib.QL_ERR_WORKSPACE
    assert b"workspace" in lib.ql_strerror(st)
    torch.cuda.synchronize()
    assert bool((o == 7.0).all()), "nothing may be launched for a rejected call"
