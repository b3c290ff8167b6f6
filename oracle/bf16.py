"""bfloat16 / fp8 helpers for the oracle (test infrastructure only).

bf16 values are carried as float32 arrays whose values are exactly
representable in bf16, or as uint16 bit patterns.  All rounding is IEEE
round-to-nearest-even (RNE), the rounding MLX uses for ``astype(bfloat16)``.
"""

from __future__ import annotations

import numpy as np

from . import _par


def f32_to_bf16_bits(x) -> np.ndarray:
    """RNE float32 -> bf16 bit pattern (uint16).  NaN stays a quiet NaN.

    uint32 arithmetic: u + 0x7FFF + lsb cannot wrap for any non-NaN pattern
    (the largest, -inf = 0xFF800000, stays below 2**32); NaN patterns, the
    only ones that could wrap, are rewritten afterwards.  Large arrays are
    processed in row chunks on every host thread (same bits)."""
    x = np.asarray(x, dtype=np.float32, order="C")
    if x.size >= _par.MIN_ELEMS:
        return _par.chunked(_f32_to_bf16_bits, x)
    return _f32_to_bf16_bits(x)


def _f32_to_bf16_bits(x):
    u = x.view(np.uint32)
    r = (u >> 16) & 1
    r += u
    r += 0x7FFF
    r >>= 16
    out = np.asarray(r.astype(np.uint16))
    nan = np.isnan(x)
    if nan.any():
        out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out[()] if out.ndim == 0 else out


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def rbf16(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (result stays float32).
    The same rounding as ``bf16_bits_to_f32(f32_to_bf16_bits(x))``, done in
    place on uint32 patterns."""
    x = np.asarray(x, dtype=np.float32, order="C")
    if x.size >= _par.MIN_ELEMS:
        return _par.chunked(_rbf16, x)
    return _rbf16(x)


def _rbf16(x):
    u = x.view(np.uint32)
    r = np.asarray((u >> 16) & 1)
    r += u
    r += 0x7FFF
    r &= 0xFFFF0000
    nan = np.isnan(x)
    if nan.any():
        r[nan] = (u[nan] & 0xFFFF0000) | 0x400000
    out = r.view(np.float32)
    return out[()] if out.ndim == 0 else out


def f64_to_f32_round_to_odd(x) -> np.ndarray:
    """float64 -> float32 with round-to-odd.

    Rounding to odd first and then RNE to bf16 gives the correctly rounded
    bf16 value of the float64 input (the float32 intermediate keeps 16 more
    significand bits than bf16), so ``rbf16(f64_to_f32_round_to_odd(v))`` is a
    single RNE rounding of ``v``.
    """
    x = np.asarray(x, dtype=np.float64)
    f = x.astype(np.float32)
    back = f.astype(np.float64)
    inexact = back != x
    # step toward zero where RNE rounded away from zero -> truncation
    away = inexact & (np.abs(back) > np.abs(x))
    f = np.where(away, np.nextafter(f, np.float32(0.0)), f)
    u = f.view(np.uint32) | np.where(inexact, np.uint32(1), np.uint32(0))
    return u.view(np.float32)


def rbf16_exact(x64) -> np.ndarray:
    """Single RNE rounding of a float64 value to bf16 (returned as float32)."""
    return rbf16(f64_to_f32_round_to_odd(x64))


def to_bf16_u16(x_f32) -> np.ndarray:
    return f32_to_bf16_bits(x_f32)


# --------------------------------------------------------------------------
# FP8 E4M3 (OCP "e4m3fn": bias 7, no infinities, 0x7F/0xFF = NaN, max 448)


def _e4m3_table() -> np.ndarray:
    vals = np.zeros(256, dtype=np.float64)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            vals[code] = np.nan
        elif e == 0:
            vals[code] = s * (m / 8.0) * 2.0 ** (-6)
        else:
            vals[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3_VALUES = _e4m3_table()


def e4m3_decode(codes) -> np.ndarray:
    """Decode E4M3 bytes to float64 (exact)."""
    return E4M3_VALUES[np.asarray(codes, dtype=np.uint8)]


_POS_CODES = np.arange(0, 0x7F, dtype=np.int64)  # 0x00..0x7E (finite, >= 0)
_POS_VALS = E4M3_VALUES[_POS_CODES]


def e4m3_encode(x) -> np.ndarray:
    """RNE float -> E4M3 with saturation to +-448 (OCP MX 'satfinite').

    Ties go to the even code (even mantissa), as IEEE RNE does; negative
    values that round to zero keep their sign (code 0x80).
    """
    x = np.asarray(x, dtype=np.float64)
    a = np.minimum(np.abs(x), 448.0)
    idx = np.searchsorted(_POS_VALS, a, side="left")  # first value >= a
    idx = np.clip(idx, 0, len(_POS_VALS) - 1)
    hi = idx
    lo = np.maximum(idx - 1, 0)
    d_hi = _POS_VALS[hi] - a
    d_lo = a - _POS_VALS[lo]
    pick_lo = (d_lo < d_hi) | ((d_lo == d_hi) & ((_POS_CODES[lo] & 1) == 0))
    code = np.where(pick_lo, _POS_CODES[lo], _POS_CODES[hi]).astype(np.uint8)
    sign = np.signbit(x).astype(np.uint8) << 7  # IEEE: the sign survives rounding to zero
    code = code | sign
    code = np.where(np.isnan(x), np.uint8(0x7F), code)
    return code.astype(np.uint8)
