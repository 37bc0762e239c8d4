"""The NVLink all-gather kernel (ql_allgather_f16) on one GPU.

With one rank there are no peers to wait for, so these cases run the
kernel's own-column path alone: the staged [gate | up] columns of `src` must
land at their global positions of `out`, on the 16-byte path (aligned
shapes) and the 2-byte path (odd widths, unaligned output rows), call after
call (the epoch advances, the banks alternate).  The multi-rank exchange is
covered on 2 GPUs in test_sharded_nccl.py.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("M,ng,groups,pad", [(1, 4096, 1, 0), (3, 1001, 2, 0), (64, 1792, 2, 8), (16, 8229, 1, 0),
                                             (5, 512, 2, 1)])
def test_single_rank_gather_places_staged_columns(M, ng, groups, pad):
    from qlinear import _lib
    from qlinear.p2p import PeerGather
    dev = _dev()
    N = ng * groups
    px = PeerGather(0, 1, max_m=64, n_cols=N)
    g = torch.Generator(device=dev).manual_seed(M + ng)
    try:
        for it in range(3):
            src = torch.randn(M, N, generator=g, device=dev).half()
            # out with a row pitch of N + pad (pad 1: rows not 16-byte aligned)
            big = torch.full((M, N + pad), float("nan"), dtype=torch.float16, device=dev)
            out = big[:, :N]
            px.gather(out, block=ng, groups=groups, src=src)
            torch.cuda.synchronize()
            assert torch.equal(out, src), it
            if pad:
                assert torch.isnan(big[:, N:]).all()
        assert _lib.device_error() == 0
    finally:
        px.close()


def test_single_rank_sharded_forward_with_gatherer():
    """ShardedQuantizedLinear at world 1 with a PeerGather attached: the
    shard's kernel writes straight into the output; equals the plain layer."""
    from qlinear.p2p import PeerGather
    from qlinear.quantization.int4 import QuantizedLinearInt4
    from qlinear.sharded import ShardedQuantizedLinear
    dev = _dev()
    K, N = 1536, 4096 + 24
    g = torch.Generator().manual_seed(3)
    lin = torch.nn.Linear(K, N, bias=True).half()
    with torch.no_grad():
        lin.weight.copy_((torch.randn(N, K, generator=g) * 0.02).half())
        lin.bias.copy_((torch.randn(N, generator=g) * 0.1).half())
    q = QuantizedLinearInt4.from_linear(lin)
    sh = ShardedQuantizedLinear.from_quantized(q, 0, 1).to(dev)
    qd = q.to(dev)
    sh.gatherer = PeerGather(0, 1, max_m=32, n_cols=N)
    try:
        for M in (1, 7, 32):
            x = torch.randn(M, K, generator=g).half().to(dev)
            assert torch.equal(sh(x), qd(x)), M
    finally:
        sh.gatherer.close()
