"""Fused gate+up projection with SwiGLU (ql_w{4,8}a16_gate_up_silu) on the GPU.

Checked against the CPU oracle: y = x @ W_deq^T in fp32 for the stacked
[2N, K] weight, ref = silu(y[:, :N]) * y[:, N:].  Bound (derived from the
north-star bound e of each projection, e = 1e-2*|x|inf*|w|inf*sqrt(K)/64):
|out - ref| <= (max|up| + max|silu(gate)|) * e + fp16 rounding of the
output, and rel-L2 <= 4e-3 (two projections' errors compound).  Covers the
fused decode-kernel epilogue (small M) and the workspace + elementwise path
(tensor-core M), both int4 layouts and int8, with and without bias, and
the model patch (fuse_mlp_gate_up) on a random-init Qwen2.
"""
import numpy as np
import pytest
import torch

from oracle import qlinear_oracle as orc
from qlinear.kernels.fused_mlp import QuantizedGateUpSiLU, fuse_mlp_gate_up, gate_up_silu, stack_gate_up
from qlinear.quantization.int4 import QuantizedLinearInt4, quantize_model_int4
from qlinear.quantization.int8 import QuantizedLinearInt8, quantize_model_int8

from helpers import make_linear, make_x

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="requires a CUDA GPU")]


def _stacked(K, N, wbits, bias, layout=0, seed=0):
    g = make_linear(K, N, bias=bias, std=0.02, seed=seed)
    u = make_linear(K, N, bias=bias, std=0.02, seed=seed + 1)
    if wbits == 4:
        qg, qu = QuantizedLinearInt4.from_linear(g, layout=layout), QuantizedLinearInt4.from_linear(u, layout=layout)
    else:
        qg, qu = QuantizedLinearInt8.from_linear(g), QuantizedLinearInt8.from_linear(u)
    return stack_gate_up(qg, qu)


def _deq(q):
    if isinstance(q, QuantizedLinearInt4):
        return orc.dequantize_int4(q.weight_packed.cpu().numpy(), q.scales.cpu().numpy(), q.layout)
    return orc.dequantize_int8(q.weight_q.cpu().numpy(), q.scale.cpu().numpy())


@pytest.mark.parametrize("K,N", [(1536, 8960), (4096, 1000), (1536, 256)])
@pytest.mark.parametrize("M", [1, 4, 8, 16, 24, 32, 64, 256])
@pytest.mark.parametrize("wbits,layout", [(4, 0), (4, 1), (8, 0)])
def test_gate_up_silu_matches_oracle(K, N, M, wbits, layout):
    bias = (N == 256)
    q = _stacked(K, N, wbits, bias, layout, seed=K + N + M)
    x = make_x(M, K, seed=M + 2)
    deq = _deq(q)
    b = q.bias.cpu().numpy() if q.bias is not None else None
    y = orc.linear_f32(x.numpy(), deq, b)
    gate, up = y[:, :N], y[:, N:]
    silu = gate / (1.0 + np.exp(-gate))
    ref = silu * up
    out = gate_up_silu(x.cuda(), q.cuda()).float().cpu().numpy()
    assert np.isfinite(out).all()
    e = 1e-2 * np.abs(x.numpy()).max() * np.abs(deq).max() * np.sqrt(K) / 64
    bound = (np.abs(up).max() + np.abs(silu).max()) * e + np.abs(ref).max() * 2.0 ** -10
    assert np.abs(out - ref).max() <= bound, (np.abs(out - ref).max(), bound)
    rel = np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-30)
    assert rel <= 4e-3, rel
    from qlinear.kernels import _launch
    for buf in _launch._workspaces.values():              # the workspace is left zero-filled
        assert int(buf.count_nonzero()) == 0


def test_module_and_bit_identical_repeat():
    q = _stacked(1536, 8960, 4, False, seed=3).cuda()
    mod = QuantizedGateUpSiLU(q)
    x = make_x(2, 1536, seed=5, lead=(1, 2)).cuda()
    a, b = mod(x), mod(x)
    assert a.shape == (1, 2, 8960) and torch.equal(a, b)


@pytest.mark.parametrize("wbits", [8, 4])
def test_fused_mlp_in_model(wbits):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=4096, hidden_size=1536, intermediate_size=8960, num_hidden_layers=2,
                      num_attention_heads=12, num_key_value_heads=2, max_position_embeddings=256,
                      tie_word_embeddings=False)
    torch.manual_seed(0)
    model = Qwen2ForCausalLM(cfg)
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0.0, 0.02)
    model = model.half().cuda().eval()
    (quantize_model_int8 if wbits == 8 else quantize_model_int4)(model)
    ids = torch.randint(0, 4096, (1, 32), generator=torch.Generator().manual_seed(2)).cuda()
    with torch.no_grad():
        ref = model(ids).logits.float()
        assert fuse_mlp_gate_up(model) == 2
        ours = model(ids).logits.float()
        out = model.generate(ids[:, :8], max_new_tokens=6, do_sample=False)
    cos = torch.nn.functional.cosine_similarity(ours.flatten(), ref.flatten(), dim=0).item()
    assert cos > 0.9999, cos
    assert (ours.argmax(-1) == ref.argmax(-1)).float().mean().item() >= 0.98
    assert out.shape == (1, 14)
    from qlinear import _lib
    assert _lib.device_error() == 0


def test_qkv_stacked_matches_oracle():
    """q/k/v from one stacked launch, each within the north-star bound of its projection."""
    from qlinear.kernels.fused_qkv import QuantizedQKV
    from helpers import assert_parity
    mods = [QuantizedLinearInt4.from_linear(make_linear(1536, n, bias=True, std=0.02, seed=n)) for n in (1536, 256, 256)]
    qkv = QuantizedQKV.from_quantized(*[m.cuda() for m in mods])
    x = make_x(3, 1536, seed=9)
    outs = qkv(x.cuda())
    for m, o in zip(mods, outs):
        deq = _deq(m)
        y = orc.linear_f32(x.numpy(), deq, m.bias.cpu().numpy())
        assert_parity(o, y, x.numpy(), deq, f"qkv part {m.out_features}")


@pytest.mark.parametrize("wbits", [8, 4])
def test_fused_qkv_and_mlp_in_model(wbits):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    from qlinear.kernels.fused_qkv import fuse_attention_qkv
    cfg = Qwen2Config(vocab_size=4096, hidden_size=1536, intermediate_size=8960, num_hidden_layers=2,
                      num_attention_heads=12, num_key_value_heads=2, max_position_embeddings=256,
                      tie_word_embeddings=False)
    torch.manual_seed(1)
    model = Qwen2ForCausalLM(cfg)
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0.0, 0.02)
    model = model.half().cuda().eval()
    (quantize_model_int8 if wbits == 8 else quantize_model_int4)(model)
    ids = torch.randint(0, 4096, (1, 32), generator=torch.Generator().manual_seed(3)).cuda()
    with torch.no_grad():
        ref = model(ids).logits.float()
        ref_gen = model.generate(ids[:, :8], max_new_tokens=6, do_sample=False)
        assert fuse_attention_qkv(model) == 2
        assert fuse_mlp_gate_up(model) == 2
        ours = model(ids).logits.float()
        gen = model.generate(ids[:, :8], max_new_tokens=6, do_sample=False)
    cos = torch.nn.functional.cosine_similarity(ours.flatten(), ref.flatten(), dim=0).item()
    assert cos > 0.9999, cos
    assert (ours.argmax(-1) == ref.argmax(-1)).float().mean().item() >= 0.98
    assert gen.shape == ref_gen.shape
