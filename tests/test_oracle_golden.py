"""Pins the CPU oracle (oracle/qlinear_oracle.py) to the reference.

The fixtures in tests/golden/ were produced by the reference's own functions
(tests/golden/make_golden.py).  Integer, packed and dequantized arrays must
match bit-for-bit; fp32 matmul outputs to summation-order rounding; fp16
outputs to one fp16 ulp (the fp32 value can sit on a rounding boundary).
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import qlinear_oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


def _cases(npz):
    names = sorted({k.split("/")[0] for k in npz.files})
    return names


INT8 = np.load(GOLDEN / "int8_cases.npz")
INT4 = np.load(GOLDEN / "int4_cases.npz")
KAT = np.load(GOLDEN / "pack_kat.npz")


def _fp16_ulp_close(a16, b16):
    a = a16.astype(np.float16).view(np.int16).astype(np.int32)
    b = b16.astype(np.float16).view(np.int16).astype(np.int32)
    return np.all(np.abs(a - b) <= 1)


@pytest.mark.parametrize("name", _cases(INT8))
def test_int8_quantize_dequant_bitexact(name):
    w = INT8[f"{name}/w"]
    wq, scale = orc.quantize_int8_rows(w)
    assert np.array_equal(wq, INT8[f"{name}/wq"])
    assert np.array_equal(scale.view(np.uint32), INT8[f"{name}/scale"].view(np.uint32))
    deq = orc.dequantize_int8(wq, scale)
    assert np.array_equal(deq.view(np.uint32), INT8[f"{name}/deq"].view(np.uint32))


@pytest.mark.parametrize("name", [n for n in _cases(INT8) if n != "ties"])
def test_int8_reference_outputs(name):
    x = INT8[f"{name}/x"]
    wq = INT8[f"{name}/wq"]
    scale = INT8[f"{name}/scale"]
    bias = INT8[f"{name}/bias"] if f"{name}/bias" in INT8.files else None
    y32 = orc.w8a16_reference_f32(x, wq, scale, bias)
    np.testing.assert_allclose(y32, INT8[f"{name}/y32"], rtol=1e-5, atol=1e-5)
    assert _fp16_ulp_close(orc.w8a16_reference(x, wq, scale, bias), INT8[f"{name}/y16"])
    assert _fp16_ulp_close(orc.w8a16_reference(x, wq, scale.astype(np.float16), bias),
                           INT8[f"{name}/y16_scale16"])


def test_int8_ties_round_half_even():
    wq = INT8["ties/wq"]
    # row 0 = [127, .5, 1.5, 2.5, -.5, -1.5, -2.5, 3.5, -126.5, 126.5, 0, -127] * 2^-6
    assert list(wq[0, :12]) == [127, 0, 2, 2, 0, -2, -2, 4, -126, 126, 0, -127]
    assert np.all(wq[1] == 0) and INT8["ties/scale"][1] == np.float32(1e-8)


@pytest.mark.parametrize("name", _cases(INT4))
def test_int4_dequant_bitexact(name):
    packed = INT4[f"{name}/packed"]
    scales = INT4[f"{name}/scales"]
    deq = orc.dequantize_int4(packed, scales)
    assert np.array_equal(deq.view(np.uint32), INT4[f"{name}/deq"].view(np.uint32))


@pytest.mark.parametrize("name", [n for n in _cases(INT4) if n != "allnibbles"])
def test_int4_quantize_bitexact(name):
    packed, scales = orc.quantize_int4_groups(INT4[f"{name}/w"])
    assert np.array_equal(packed, INT4[f"{name}/packed"])
    assert np.array_equal(scales.view(np.uint16), INT4[f"{name}/scales"].view(np.uint16))
    if f"{name}/unpacked" in INT4.files:
        assert np.array_equal(orc.unpack_int4(packed), INT4[f"{name}/unpacked"])


@pytest.mark.parametrize("name", [n for n in _cases(INT4) if n not in ("ties", "allnibbles")])
def test_int4_reference_outputs(name):
    x = INT4[f"{name}/x"]
    packed = INT4[f"{name}/packed"]
    scales = INT4[f"{name}/scales"]
    bias = INT4[f"{name}/bias"] if f"{name}/bias" in INT4.files else None
    y32 = orc.w4a16_reference_f32(x, packed, scales, bias)
    np.testing.assert_allclose(y32, INT4[f"{name}/y32"], rtol=1e-5, atol=1e-5)
    assert _fp16_ulp_close(orc.w4a16_reference(x, packed, scales, bias), INT4[f"{name}/y16"])


def test_int4_all_nibbles_pinned():
    q = INT4["allnibbles/q"]
    assert np.array_equal(orc.pack_int4(q), INT4["allnibbles/packed"])
    assert np.array_equal(orc.unpack_int4(INT4["allnibbles/packed"]), q)
    assert set(np.unique(q)) == set(range(16))


def test_pack_unpack_kat():
    """The reference's own KAT inputs (tests/test_w4a16_kernel.py:52-59)."""
    for i in (1, 2):
        q = KAT[f"q{i}"]
        assert np.array_equal(orc.pack_int4(q), KAT[f"packed{i}"])
        assert np.array_equal(orc.unpack_int4(KAT[f"packed{i}"]), KAT[f"unpacked{i}"])
        assert np.array_equal(KAT[f"unpacked{i}"], q)


def test_adjacent_layout_is_a_permutation_of_reference_nibbles():
    """The variant layout holds the same nibble values as the reference's
    split-half layout, only in a different byte position, so its dequant is
    pinned through the reference's fixtures."""
    q = KAT["q1"]
    adj = orc.pack_int4_adjacent(q)
    assert np.array_equal(orc.unpack_int4_adjacent(adj), q)
    for name in ("k384_n100_m7_bias", "k256_n64_m3"):
        packed = INT4[f"{name}/packed"]
        scales = INT4[f"{name}/scales"]
        qq = orc.unpack_int4(packed)
        deq_adj = orc.dequantize_int4(orc.pack_int4_adjacent(qq), scales, orc.LAYOUT_ADJACENT)
        assert np.array_equal(deq_adj.view(np.uint32), INT4[f"{name}/deq"].view(np.uint32))


def test_variant_quantizer_range():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((16, 256)) * 0.02).astype(np.float16)
    packed, scales = orc.quantize_int4_groups(w, qmin=-8, layout=orc.LAYOUT_ADJACENT)
    q = orc.unpack_int4_adjacent(packed).astype(np.int32) - 8
    assert q.min() >= -8 and q.max() <= 7
    deq = orc.dequantize_int4(packed, scales, orc.LAYOUT_ADJACENT)
    step = np.repeat(scales.astype(np.float32).T, 128, axis=1)
    assert np.all(np.abs(deq - w.astype(np.float32)) <= 0.51 * step + 1e-6)


def test_parity_bound_formula():
    x = np.ones((1, 4096), np.float32) * 2.0
    w = np.ones((8, 4096), np.float32) * 0.5
    b_abs, b_rel = orc.parity_bounds(x, w)
    assert b_abs == pytest.approx(1e-2 * 2.0 * 0.5 * 64 / 64)
    assert b_rel == 2e-3
