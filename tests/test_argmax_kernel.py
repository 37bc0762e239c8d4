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
