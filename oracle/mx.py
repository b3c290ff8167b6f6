"""The activation side of the native block-scaled fp8 path, restated in numpy
(test infrastructure only).

The product's LTXQ_COMPUTE_MX2 / MX1 GEMMs (ltx-2-mlx_b200/csrc/mx.cu) feed
the reference's mxfp8 cache (E4M3 codes, one E8M0 scale per 32 K;
loader/transformer_cache.py:26-33, 840-848) to the tensor cores as is and
quantize the bf16 activations to MXFP8 in one or two terms.  This module
defines that quantization and the resulting linear layer, so that the GPU
splitter is held bit-exact and the GEMM to fp32 summation order:

* MX(v), per group of 32 consecutive K: e = the smallest integer >= -127 with
  max|v| * 2^-e <= 448 (E4M3's largest value; OCP MX v1.0 picks
  floor(log2 max) - 8 and lets values saturate, this choice never
  saturates); codes = RNE_E4M3(v * 2^-e); scale byte e + 127;
* two terms: hi = MX(x), lo = MX(x - decode(hi)); one term: hi only;
* the linear layer: y = bf16(x_eff . W^T) then bf16(y + bias), with
  x_eff = decode(hi) (+ decode(lo)) exactly and W the exactly dequantized
  mxfp8 weight -- the reference's composition with x replaced by x_eff.

Against the reference composition itself (x, not x_eff) the two-term form
differs by about 2^-8 of each group's largest activation; that is checked
with the path's stated tolerance, not bit for bit.
"""

from __future__ import annotations

import numpy as np

from . import ref_ops as ro
from .bf16 import e4m3_decode, e4m3_encode, rbf16

GROUP = 32


def group_exp(amax: np.ndarray) -> np.ndarray:
    """Smallest e >= -127 with amax * 2^-e <= 448 (amax >= 0, float32)."""
    amax = np.asarray(amax, np.float32)
    bits = amax.view(np.uint32)
    ef = (bits >> 23).astype(np.int64)
    mant = bits & np.uint32(0x7FFFFF)
    e = ef - 127 - 8 + (mant > 0x600000).astype(np.int64)
    e = np.where(ef == 0, -127, e)
    return np.maximum(e, -127)


def mx_term(v: np.ndarray):
    """One MX term of v [..., K] (float32): (codes uint8 [..., K], e int
    [..., K/32], residual v - decode(codes) * 2^e as float32)."""
    v = np.asarray(v, np.float32)
    shp = v.shape
    g = v.reshape(shp[:-1] + (shp[-1] // GROUP, GROUP))
    e = group_exp(np.abs(g).max(axis=-1))
    inv = np.ldexp(np.float32(1.0), (-e).astype(np.int32)).astype(np.float32)[..., None]
    codes = e4m3_encode((g * inv).astype(np.float32))
    val = (e4m3_decode(codes) * np.ldexp(1.0, e.astype(np.int32))[..., None]).astype(np.float32)
    resid = (g - val).astype(np.float32)
    return codes.reshape(shp), e, resid.reshape(shp)


def mx_split(x_bf16: np.ndarray, terms: int = 2):
    """[(codes, e), ...] of the terms of x (bf16 values as float32)."""
    out = []
    v = np.asarray(x_bf16, np.float32)
    for _ in range(terms):
        codes, e, v = mx_term(v)
        out.append((codes, e))
    return out


def mx_value(x_bf16: np.ndarray, terms: int = 2) -> np.ndarray:
    """x_eff = the sum of the decoded terms (float64, exact)."""
    x = np.asarray(x_bf16, np.float32)
    acc = np.zeros(x.shape, np.float64)
    for codes, e in mx_split(x, terms):
        k = x.shape[-1]
        scale = np.repeat(np.ldexp(1.0, e.astype(np.int32)), GROUP, axis=-1)[..., :k]
        acc += e4m3_decode(codes) * scale
    return acc


def mx_linear(x_bf16, w_deq_bf16, bias_bf16=None, terms: int = 2):
    """The MX path's linear layer: the reference composition (ro.linear) on
    x_eff (exact in float32: at most 2 x 4 significant bits)."""
    x_eff = mx_value(x_bf16, terms).astype(np.float32)
    return ro.linear(x_eff, w_deq_bf16, bias_bf16)


def scale_atoms(e: np.ndarray, row_tiles: int) -> np.ndarray:
    """The scale bytes e + 127 of [M, K/32] in the GEMM's atom layout (see
    include/ltxq.h ltxq_mx_split): uint8 [K/128, row_tiles, 512]."""
    m, groups = e.shape
    s = np.zeros((row_tiles * 128, groups), np.uint8)
    s[:m] = (e + 127).astype(np.uint8)
    # rows 128 t + 32 m1 + m0, groups 4 j + k1 -> [j, t, m0, m1, k1]
    a = s.reshape(row_tiles, 4, 32, groups // 4, 4).transpose(3, 0, 2, 1, 4)
    return np.ascontiguousarray(a).reshape(groups // 4, row_tiles, 512)
