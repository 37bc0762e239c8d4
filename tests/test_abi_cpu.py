"""CPU-only checks of the boundary and the host logic (no GPU needed).

* libqlinear.so loads and exports every function include/qlinear.h declares;
* status strings / version;
* the Python mirror of the reference interface: pack/unpack, from_linear on
  CPU (bit-exact against the oracle and the reference's golden fixtures),
  num_bytes, quantize_model_* module replacement, assert messages.
"""
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import qlinear_oracle as orc
from qlinear import _lib
from qlinear.kernels.w4a16_matmul import (
    GROUP_SIZE, pack_int4, unpack_int4, pack_int4_adjacent, unpack_int4_adjacent,
    dequantize_int4, w4a16_linear, w4a16_reference, LAYOUT_ADJACENT,
)
from qlinear.kernels.w8a16_matmul import w8a16_linear, w8a16_reference
from qlinear.quantization.int8 import QuantizedLinearInt8, quantize_model_int8
from qlinear.quantization.int4 import QuantizedLinearInt4, quantize_model_int4

from helpers import make_linear, make_x

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "qlinear.h"
GOLDEN = ROOT / "tests" / "golden"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ql_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 12
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"symbols declared in qlinear.h but not exported: {missing}"
    # and the ctypes signature table covers exactly the header
    assert sorted(_lib.SIGNATURES) == names


def test_status_strings_and_version():
    lib = _lib.load()
    for code in range(0, -9, -1):
        s = lib.ql_strerror(code)
        assert s and s.startswith(b"ok" if code == 0 else b"qlinear:")
    assert lib.ql_strerror(-1234) == b"qlinear: unknown status"
    assert _lib.version() == (0, 1, 0)


def test_host_argument_checks_without_gpu():
    """Shape/stride/dtype errors are caught on the host before any device call."""
    lib = _lib.load()
    # K not a multiple of 128 for int4
    st = lib.ql_w4a16_linear(1, 0, 1, 0, 1, None, 0, 1, 1, 1, 100, 100, 50, 1, 1, None, 0, 0, None)
    assert st == _lib.QL_ERR_BAD_SHAPE
    # leading dimension too small
    st = lib.ql_w8a16_linear(1, 0, 1, 1, 1, None, 0, 1, 2, 4, 64, 32, 64, 4, None, 0, 0, None)
    assert st == _lib.QL_ERR_BAD_STRIDE
    # bf16 activations are not in this build
    st = lib.ql_w8a16_linear(1, 2, 1, 1, 1, None, 0, 1, 2, 4, 64, 64, 64, 4, None, 0, 0, None)
    assert st == _lib.QL_ERR_UNSUPPORTED
    # null pointers with work to do
    st = lib.ql_w8a16_linear(None, 0, 1, 1, 1, None, 0, 1, 2, 4, 64, 64, 64, 4, None, 0, 0, None)
    assert st == _lib.QL_ERR_NULL_POINTER
    # empty problems are a no-op even with null pointers
    assert lib.ql_w8a16_linear(None, 0, None, None, 1, None, 0, None, 0, 4, 64, 64, 64, 4, None, 0, 0, None) == 0
    # unknown layout
    st = lib.ql_w4a16_linear(1, 0, 1, 7, 1, None, 0, 1, 1, 1, 128, 128, 64, 1, 1, None, 0, 0, None)
    assert st == _lib.QL_ERR_UNSUPPORTED


def test_greedy_head_argument_checks_without_gpu():
    """The fused linear + argmax entry points check the exchange arguments
    and shapes on the host; the support query answers 0 without a device."""
    import ctypes
    lib = _lib.load()
    peers = (ctypes.c_void_p * 2)(1, 1)
    # world outside 1..8
    st = lib.ql_w4a16_linear_argmax(1, 0, 1, 0, 1, None, 0, 1, 16, 128, 128, 64, 16, 0, 0, 9, 4, peers, 1, 0, None)
    assert st == _lib.QL_ERR_BAD_SHAPE
    # rows beyond the exchange's max_m
    st = lib.ql_w8a16_linear_argmax(1, 0, 1, 1, 1, None, 0, 5, 16, 128, 128, 128, 0, 0, 2, 4, peers, 1, 0, None)
    assert st == _lib.QL_ERR_BAD_SHAPE
    # missing peer buffer / output
    null_peers = (ctypes.c_void_p * 2)(1, None)
    st = lib.ql_w8a16_linear_argmax(1, 0, 1, 1, 1, None, 0, 1, 16, 128, 128, 128, 0, 0, 2, 4, null_peers, 1, 0,
                                    None)
    assert st == _lib.QL_ERR_NULL_POINTER
    st = lib.ql_w8a16_linear_argmax(1, 0, 1, 1, 1, None, 0, 1, 16, 128, 128, 128, 0, 0, 2, 4, peers, None, 0, None)
    assert st == _lib.QL_ERR_NULL_POINTER
    # columns past 2^32 - 1
    st = lib.ql_w8a16_linear_argmax(1, 0, 1, 1, 1, None, 0, 1, 16, 128, 128, 128, 0xFFFFFFFF, 0, 2, 4, peers, 1,
                                    0, None)
    assert st == _lib.QL_ERR_BAD_SHAPE
    # bf16 activations
    st = lib.ql_w8a16_linear_argmax(1, 2, 1, 1, 1, None, 0, 1, 16, 128, 128, 128, 0, 0, 2, 4, peers, 1, 0, None)
    assert st == _lib.QL_ERR_UNSUPPORTED
    assert lib.ql_linear_argmax_supported(4, 1, 4096, 1536) in (0, 1)
    assert lib.ql_linear_argmax_supported(5, 1, 4096, 1536) == 0
    assert lib.ql_linear_argmax_supported(4, 1, 4096, 100) == 0


def test_gather_argument_checks_without_gpu():
    """The NVLink all-gather checks shapes, strides and peers on the host;
    its buffer size covers two banks of [max_m, N rounded up to 8] fp16."""
    import ctypes
    lib = _lib.load()
    assert lib.ql_gather_buffer_bytes(0, 1024) == 0
    assert lib.ql_gather_buffer_bytes(4, 0) == 0
    assert lib.ql_gather_buffer_bytes(4, 1001) >= 8448 + 2 * 4 * 1008 * 2
    assert lib.ql_gather_buffer_bytes(4, 1001) % 256 == 0
    names = ["src", "lds", "out", "ldo", "M", "N", "groups", "block", "rank", "world", "max_m", "peers",
             "flags", "stream"]
    ok = dict(zip(names, (None, 0, 1, 4096, 2, 4096, 1, 2048, 0, 2, 4, (ctypes.c_void_p * 2)(1, 1), 0, None)))

    def call(**kw):
        args = dict(ok, **kw)
        return lib.ql_allgather_f16(*[args[n] for n in names])

    assert call(out=None) == _lib.QL_ERR_NULL_POINTER
    assert call(peers=(ctypes.c_void_p * 2)(1, None)) == _lib.QL_ERR_NULL_POINTER
    assert call(world=9) == _lib.QL_ERR_BAD_SHAPE
    assert call(rank=2) == _lib.QL_ERR_BAD_SHAPE
    assert call(M=5) == _lib.QL_ERR_BAD_SHAPE                 # beyond max_m
    assert call(block=2000) == _lib.QL_ERR_BAD_SHAPE          # two shards do not cover 4096 columns
    assert call(N=4095, groups=2) == _lib.QL_ERR_BAD_SHAPE    # groups must divide N
    assert call(ldo=4000) == _lib.QL_ERR_BAD_STRIDE
    assert call(src=1, lds=1000) == _lib.QL_ERR_BAD_STRIDE    # this rank's 2048 columns need lds >= 2048
    # one rank with its columns already in place: nothing to launch
    assert call(world=1, block=4096, peers=(ctypes.c_void_p * 1)(1)) == 0


def test_pack_unpack_roundtrip():
    """The reference's KAT (tests/test_w4a16_kernel.py:52-59)."""
    torch.manual_seed(0)
    q = torch.randint(0, 16, (37, 384), dtype=torch.uint8)
    assert torch.equal(unpack_int4(pack_int4(q)), q)
    q2 = torch.arange(16, dtype=torch.uint8).repeat(2, 8)
    assert torch.equal(unpack_int4(pack_int4(q2)), q2)
    assert torch.equal(unpack_int4_adjacent(pack_int4_adjacent(q)), q)
    assert np.array_equal(pack_int4(q).numpy(), orc.pack_int4(q.numpy()))
    assert np.array_equal(pack_int4_adjacent(q).numpy(), orc.pack_int4_adjacent(q.numpy()))


def test_int8_from_linear_cpu_matches_golden():
    z = np.load(GOLDEN / "int8_cases.npz")
    for name in ("k100_n37_m7_bias", "k384_n100_m5", "ties"):
        w = torch.from_numpy(z[f"{name}/w"])
        lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False).half()
        with torch.no_grad():
            lin.weight.copy_(w)
        q = QuantizedLinearInt8.from_linear(lin)
        assert np.array_equal(q.weight_q.numpy(), z[f"{name}/wq"])
        assert np.array_equal(q.scale.numpy().view(np.uint32), z[f"{name}/scale"].view(np.uint32))
        assert np.array_equal(q.dequantized_weight().numpy().view(np.uint32), z[f"{name}/deq"].view(np.uint32))


def test_int4_from_linear_cpu_matches_golden():
    z = np.load(GOLDEN / "int4_cases.npz")
    for name in ("k384_n100_m7_bias", "k256_n64_m3", "ties"):
        w = torch.from_numpy(z[f"{name}/w"])
        lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False).half()
        with torch.no_grad():
            lin.weight.copy_(w)
        q = QuantizedLinearInt4.from_linear(lin)
        assert np.array_equal(q.weight_packed.numpy(), z[f"{name}/packed"])
        assert np.array_equal(q.scales.numpy().view(np.uint16), z[f"{name}/scales"].view(np.uint16))
        assert np.array_equal(q.dequantized_weight().numpy().view(np.uint32), z[f"{name}/deq"].view(np.uint32))


def test_int4_variant_from_linear_cpu_matches_oracle():
    lin = make_linear(256, 24, bias=True, seed=5)
    q = QuantizedLinearInt4.from_linear(lin, qmin=-8, layout=LAYOUT_ADJACENT)
    packed, scales = orc.quantize_int4_groups(lin.weight.detach().numpy(), qmin=-8,
                                              layout=orc.LAYOUT_ADJACENT)
    assert np.array_equal(q.weight_packed.numpy(), packed)
    assert np.array_equal(q.scales.numpy().view(np.uint16), scales.view(np.uint16))
    deq = dequantize_int4(q.weight_packed, q.scales, LAYOUT_ADJACENT).numpy()
    assert np.array_equal(deq.view(np.uint32),
                          orc.dequantize_int4(packed, scales, orc.LAYOUT_ADJACENT).view(np.uint32))


def test_reference_helpers_match_oracle():
    lin = make_linear(384, 100, bias=True, seed=3)
    x = make_x(5, 384, seed=4)
    q8 = QuantizedLinearInt8.from_linear(lin)
    y = w8a16_reference(x, q8.weight_q, q8.scale, q8.bias).numpy()
    yo = orc.w8a16_reference(x.numpy(), q8.weight_q.numpy(), q8.scale.numpy(), q8.bias.numpy())
    assert np.abs(y.astype(np.float32) - yo.astype(np.float32)).max() <= 2e-3
    q4 = QuantizedLinearInt4.from_linear(lin)
    y = w4a16_reference(x, q4.weight_packed, q4.scales, q4.bias).numpy()
    yo = orc.w4a16_reference(x.numpy(), q4.weight_packed.numpy(), q4.scales.numpy(), q4.bias.numpy())
    assert np.abs(y.astype(np.float32) - yo.astype(np.float32)).max() <= 2e-3


def test_num_bytes_and_ratios():
    """Byte ratios of the reference tests (test_w8a16_kernel.py:116-120,
    test_w4a16_kernel.py:120-125)."""
    lin = make_linear(1536, 8960, bias=False)
    fp16_bytes = lin.weight.numel() * lin.weight.element_size()
    q8 = QuantizedLinearInt8.from_linear(lin)
    q4 = QuantizedLinearInt4.from_linear(lin)
    assert q8.num_bytes() == 8960 * 1536 + 8960 * 4
    assert q4.num_bytes() == 8960 * 768 + 12 * 8960 * 2
    assert q8.num_bytes() < 0.55 * fp16_bytes
    assert q4.num_bytes() < 0.28 * fp16_bytes


def test_kernel_entry_asserts_match_reference_messages():
    lin = make_linear(256, 64, bias=False)
    q8 = QuantizedLinearInt8.from_linear(lin)
    x = make_x(2, 256)
    with pytest.raises(AssertionError):        # x.is_cuda is False (reference :110)
        w8a16_linear(x, q8.weight_q, q8.scale)
    q4 = QuantizedLinearInt4.from_linear(lin)
    with pytest.raises(AssertionError):
        w4a16_linear(x, q4.weight_packed, q4.scales)
    with pytest.raises(AssertionError, match="must be a multiple of 128"):
        QuantizedLinearInt4.from_linear(make_linear(100, 8, bias=False))


def _tiny_qwen2():
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(vocab_size=128, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64)
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).half().eval()


def test_quantize_model_replaces_every_layer_linear():
    """7 linears per layer (q,k,v,o,gate,up,down); lm_head untouched
    (reference test_e2e_quantization.py:48-59)."""
    m = _tiny_qwen2()
    stats = quantize_model_int8(m)
    assert stats["layers_quantized"] == 2 * 7
    assert isinstance(m.model.layers[0].self_attn.q_proj, QuantizedLinearInt8)
    assert isinstance(m.lm_head, torch.nn.Linear)
    assert stats["bytes_after"] < 0.6 * stats["bytes_before"]
    m4 = _tiny_qwen2()
    stats4 = quantize_model_int4(m4)
    assert stats4["layers_quantized"] == 2 * 7
    assert isinstance(m4.model.layers[1].mlp.down_proj, QuantizedLinearInt4)
    assert stats4["bytes_after"] < 0.35 * stats4["bytes_before"]
    # buffers keep the reference's names, so state_dict round-trips
    sd = m4.state_dict()
    assert "model.layers.0.self_attn.q_proj.weight_packed" in sd
    assert "model.layers.0.self_attn.q_proj.scales" in sd
    assert "model.layers.0.self_attn.q_proj.bias" in sd


def test_stacked_gate_up_dequantizes_to_the_stacked_weights():
    """stack_gate_up concatenates quantized buffers; row-local quantization
    makes that equal to quantizing the stacked fp16 weight."""
    from qlinear.kernels.fused_mlp import stack_gate_up
    from helpers import make_linear
    g, u = make_linear(256, 40, bias=True, seed=1), make_linear(256, 40, bias=False, seed=2)
    for cls in (QuantizedLinearInt4, QuantizedLinearInt8):
        s = stack_gate_up(cls.from_linear(g), cls.from_linear(u))
        both = torch.nn.Linear(256, 80, bias=True).half()
        with torch.no_grad():
            both.weight.copy_(torch.cat([g.weight, u.weight]))
            both.bias.copy_(torch.cat([g.bias, torch.zeros(40, dtype=torch.float16)]))
        ref = cls.from_linear(both)
        assert torch.equal(s.dequantized_weight(), ref.dequantized_weight())
        assert torch.equal(s.bias, ref.bias)


def test_stacked_qkv_rows_dequantize_to_the_stacked_weights():
    from qlinear.kernels.fused_qkv import stack_rows
    from helpers import make_linear
    lins = [make_linear(256, n, bias=True, seed=n) for n in (64, 16, 16)]
    for cls in (QuantizedLinearInt4, QuantizedLinearInt8):
        s = stack_rows([cls.from_linear(l) for l in lins])
        both = torch.nn.Linear(256, 96, bias=True).half()
        with torch.no_grad():
            both.weight.copy_(torch.cat([l.weight for l in lins]))
            both.bias.copy_(torch.cat([l.bias for l in lins]))
        ref = cls.from_linear(both)
        assert torch.equal(s.dequantized_weight(), ref.dequantized_weight())
        assert torch.equal(s.bias, ref.bias)
