"""CPU checks of the oracle itself (no GPU).

Pins the oracle to the reference's own known-answer vector
(tests/test_transformer_cache.py:64-95: E4M3 byte 0x38 decodes to 1.0, and
times a weight_scale of 2.0 gives bf16 2.0) and to first-principles
properties of the restated MLX algorithms (exact RNE rounding, packing
order, quantizer error bounds).
"""

from fractions import Fraction

import numpy as np
import pytest

from helpers import normal_bf16, rng
from oracle import quant as oq
from oracle import ref_ops as ro
from oracle.bf16 import (
    bf16_bits_to_f32,
    e4m3_decode,
    e4m3_encode,
    f32_to_bf16_bits,
    rbf16,
    rbf16_exact,
)


def test_e4m3_known_answer_from_reference_test():
    # tests/test_transformer_cache.py:64-95 of the reference
    assert e4m3_decode(np.array([0x38], dtype=np.uint8))[0] == 1.0
    scaled = e4m3_decode(np.array([0x38], dtype=np.uint8)) * 2.0
    assert float(rbf16(scaled.astype(np.float32))[0]) == 2.0


def test_e4m3_extremes_and_round_trip():
    assert e4m3_decode(np.array([0x7E], dtype=np.uint8))[0] == 448.0
    assert e4m3_decode(np.array([0x01], dtype=np.uint8))[0] == 2.0 ** -9
    assert np.isnan(e4m3_decode(np.array([0x7F], dtype=np.uint8))[0])
    codes = np.array([c for c in range(256) if c not in (0x7F, 0xFF)], dtype=np.uint8)
    back = e4m3_encode(e4m3_decode(codes))
    assert np.array_equal(back, codes)
    # saturation and RNE ties to the even code
    assert e4m3_encode(np.array([1000.0]))[0] == 0x7E
    assert e4m3_encode(np.array([-1000.0]))[0] == 0xFE
    assert e4m3_encode(np.array([1.0 + 1 / 16]))[0] == 0x38  # tie between 1.0 (even) and 1.125
    assert e4m3_encode(np.array([1.0 + 3 / 16]))[0] == 0x3A  # tie between 1.125 and 1.25 (even)


def test_bf16_rne():
    assert f32_to_bf16_bits(np.float32(1.0)) == 0x3F80
    # halfway between 1.0 and 1.0078125 rounds to even (1.0)
    assert float(rbf16(np.float32(1.00390625))) == 1.0
    assert float(rbf16(np.float32(1.01171875))) == 1.015625
    assert bf16_bits_to_f32(np.uint16(0xC2F7)) == -123.5


def _exact_rne_bf16(fr: Fraction) -> float:
    if fr == 0:
        return 0.0
    sign = -1 if fr < 0 else 1
    a = abs(fr)
    e = 0
    while a >= 2:
        a /= 2
        e += 1
    while a < 1:
        a *= 2
        e -= 1
    scaled = a * 128  # 8 significant bits
    fl = scaled.numerator // scaled.denominator
    rem = scaled - fl
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and fl % 2 == 1):
        fl += 1
    return sign * float(Fraction(fl, 128) * Fraction(2) ** e)


def test_single_rounding_of_affine_dequant_is_exact():
    g = rng(0)
    s = rbf16(g.standard_normal(2000).astype(np.float32) * 1e-3)
    b = rbf16(g.standard_normal(2000).astype(np.float32) * 5e-2)
    q = g.integers(0, 256, 2000)
    got = rbf16_exact(s.astype(np.float64) * q + b.astype(np.float64))
    for i in range(0, 2000, 7):
        want = _exact_rne_bf16(Fraction(float(s[i])) * int(q[i]) + Fraction(float(b[i])))
        assert float(got[i]) == want


@pytest.mark.parametrize("bits", [4, 8])
def test_pack_order_low_bits_first(bits):
    per = 32 // bits
    q = np.arange(per, dtype=np.uint32)[None, :] % (1 << bits)
    w = oq.pack_bits(q, bits)
    assert w[0, 0] == sum(int(v) << (bits * i) for i, v in enumerate(q[0]))
    assert np.array_equal(oq.unpack_bits(w, bits, per), q)


@pytest.mark.parametrize("bits", [4, 8])
def test_affine_quantizer_error_bound(bits):
    W = normal_bf16(rng(1), (64, 256), 0.02)
    q = oq.quantize(W, "affine", 64, bits)
    deq = oq.dequantize(q, 256)
    s = np.abs(bf16_bits_to_f32(q["scales"])).repeat(64, axis=1)
    # reconstruction error is about half a quantization step, plus the error of
    # storing the scale in bf16 (q * scale * 2**-9 <= 0.5 step for 8 bits);
    # snapping the larger-magnitude edge to an exact code shrinks the step
    # slightly, so the opposite edge can clip by up to one step
    err = np.abs(deq - W)
    assert np.all(err <= 1.6 * s + np.abs(W) * 2 ** -7 + 1e-6)
    assert np.mean(err <= 1.0 * s + np.abs(W) * 2 ** -7) > 0.99


def test_mxfp8_quantizer_properties():
    W = normal_bf16(rng(2), (32, 128), 0.02)
    q = oq.quantize(W, "mxfp8")
    deq = oq.dequantize(q, 128)
    amax = np.abs(W).reshape(32, 4, 32).max(axis=2)
    e = np.floor(np.log2(amax)) - 8
    assert np.array_equal(q["scales"].astype(np.int64) - 127, e.astype(np.int64))
    rel = np.abs(deq - W) / np.maximum(np.abs(W), 1e-12)
    scaled = np.abs(W) / 2.0 ** e.repeat(32, axis=1)
    # OCP MX: amax / 2**e lies in [256, 512); values above 448 saturate
    assert scaled.max() < 512.0
    assert np.all(np.abs(deq[scaled > 448.0]) == 448.0 * 2.0 ** e.repeat(32, axis=1)[scaled > 448.0])
    normal = (scaled >= 2.0 ** -6) & (scaled <= 448.0)  # E4M3 normal range: 3 mantissa bits
    assert rel[normal].max() <= 2 ** -4 + 1e-6


def test_gelu_rounding_points():
    x = rbf16(np.linspace(-6, 6, 1001).astype(np.float32))
    a = ro.gelu_approx(x)
    b = ro.gelu_tanh_f32(x)
    # the reference's per-op bf16 chain stays within a few bf16 ulps of the
    # single-rounding evaluation
    assert np.max(np.abs(a - b)) <= 0.05
    assert ro._C_GELU == 0.044677734375 and ro._C_SQRT == 0.796875


def test_composition_rounding_points():
    g = rng(3)
    x = normal_bf16(g, (4, 64))
    s = (g.standard_normal(64) * 0.1).astype(np.float32)
    t = (g.standard_normal(64) * 0.1).astype(np.float32)
    out = ro.adaln(x, s, t)
    assert np.array_equal(out, rbf16(out))  # bf16-valued
    n = ro.rms_norm(x)
    assert np.array_equal(out, rbf16((n * (np.float32(1) + s)).astype(np.float32) + t))
