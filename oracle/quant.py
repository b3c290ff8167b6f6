"""MLX-layout weight quantization, restated in numpy (test infrastructure only).

Layouts follow the reference's cache (LTX_2_MLX/loader/transformer_cache.py:
1238-1267 writes ``mx.quantize`` outputs; :1436-1462 gives the placeholder
dtypes; :797-811 the per-mode defaults affine->(64,4), mxfp8->(32,8)):

* affine (bits 4 or 8, group_size 64 by default):
  ``weight`` uint32 [N, K*bits/32], element k of a row at bit offset
  ``bits*(k % (32/bits))`` of word ``k // (32/bits)`` (little end first);
  ``scales``/``biases`` bf16 [N, K/group_size]; dequant ``w = scale*q + bias``.
* mxfp8 (group_size 32): ``weight`` uint32 [N, K/4] holding E4M3 bytes in k
  order; ``scales`` uint8 [N, K/32] E8M0 (value 2**(s-127)); no biases.

``pretransposed`` caches (transformer_cache.py:1240-1244, mode
``mxfp8-blocks-pretranspose``) quantize ``W.T`` with the same functions, so
their groups run along the output dimension N.

Parity note: the affine quantizer restates MLX's published ``mx.quantize``
algorithm (fp32 min/max per group, the larger-magnitude edge snapped so that
zero is an exact code, RNE rounding, clip to [0, 2**bits-1], scales/biases
cast to the weight dtype).  No reference test pins these numerics, so the
quantizer is "parity unpinned"; the dequantizer below is the definition the
CUDA path is held bit-exact against.
"""

from __future__ import annotations

import numpy as np

from .bf16 import (
    bf16_bits_to_f32,
    e4m3_decode,
    e4m3_encode,
    f32_to_bf16_bits,
    rbf16,
    rbf16_exact,
)


# --------------------------------------------------------------------------
# packing


def pack_bits(q: np.ndarray, bits: int) -> np.ndarray:
    """Pack unsigned codes [N, K] into uint32 [N, K*bits/32] (MLX order)."""
    per = 32 // bits
    n, k = q.shape
    assert k % per == 0
    q = q.astype(np.uint32).reshape(n, k // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    return np.bitwise_or.reduce(q << shifts, axis=2).astype(np.uint32)


def unpack_bits(w: np.ndarray, bits: int, k: int) -> np.ndarray:
    per = 32 // bits
    n = w.shape[0]
    shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    q = (w.astype(np.uint32)[:, :, None] >> shifts) & np.uint32((1 << bits) - 1)
    return q.reshape(n, -1)[:, :k].astype(np.uint32)


# --------------------------------------------------------------------------
# affine


def affine_quantize(w_bf16_f32: np.ndarray, group_size: int = 64, bits: int = 8):
    """MLX affine quantize of a bf16 weight [N, K] (values given as float32).

    Returns (weight_u32 [N, K*bits/32], scales_bf16_u16 [N, K/gs],
    biases_bf16_u16 [N, K/gs]).
    """
    w = np.asarray(w_bf16_f32, dtype=np.float32)
    n, k = w.shape
    assert k % group_size == 0, "K must be a multiple of group_size"
    g = w.reshape(n, k // group_size, group_size)
    n_bins = np.float32((1 << bits) - 1)
    w_max = g.max(axis=2, keepdims=True).astype(np.float32)
    w_min = g.min(axis=2, keepdims=True).astype(np.float32)
    mask = np.abs(w_min) > np.abs(w_max)
    scales = np.maximum((w_max - w_min) / n_bins, np.float32(1e-7)).astype(np.float32)
    scales = np.where(mask, scales, -scales).astype(np.float32)
    edge = np.where(mask, w_min, w_max).astype(np.float32)
    q0 = np.round(edge / scales).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        snapped = (edge / q0).astype(np.float32)
    scales = np.where(q0 != 0, snapped, scales).astype(np.float32)
    biases = np.where(q0 == 0, np.float32(0.0), edge).astype(np.float32)
    q = np.clip(np.round((g - biases) / scales), 0, n_bins).astype(np.uint32)
    q = q.reshape(n, k)
    return (
        pack_bits(q, bits),
        f32_to_bf16_bits(scales.reshape(n, -1)),
        f32_to_bf16_bits(biases.reshape(n, -1)),
    )


def affine_dequantize(weight_u32, scales_u16, biases_u16, k: int, group_size: int = 64, bits: int = 8):
    """Dequantize to bf16 values (float32 array): ``RNE_bf16(scale*q + bias)``.

    The product and sum are evaluated exactly (float64; for bf16 scale/bias and
    q < 2**8 the result is exact whenever the exponents of scale*q and bias
    differ by less than ~37) and rounded once to bf16.
    """
    q = unpack_bits(np.asarray(weight_u32), bits, k).astype(np.float64)
    n = q.shape[0]
    s = bf16_bits_to_f32(scales_u16).astype(np.float64)
    b = bf16_bits_to_f32(biases_u16).astype(np.float64)
    s = np.repeat(s, group_size, axis=1)[:, :k]
    b = np.repeat(b, group_size, axis=1)[:, :k]
    return rbf16_exact(s * q + b).reshape(n, k)


def affine_dequantize_fast(weight_u32, scales_u16, biases_u16, k: int, group_size: int = 64, bits: int = 8):
    """float32 evaluation of the same dequantization for the timed CPU
    baseline: ``rbf16(fp32 fma-free scale*q + bias)``.  It equals
    ``affine_dequantize`` whenever scale*q + bias is exact in fp32 (the
    exponents of the two terms within 2**8 of each other, true for every
    group ``affine_quantize`` produces from finite weights)."""
    q = unpack_bits(np.asarray(weight_u32), bits, k).astype(np.float32)
    n = q.shape[0]
    s = bf16_bits_to_f32(scales_u16)[:, :, None]
    b = bf16_bits_to_f32(biases_u16)[:, :, None]
    g = q.reshape(n, -1, group_size)
    return rbf16((g * s + b).astype(np.float32)).reshape(n, k)


# --------------------------------------------------------------------------
# mxfp8 (OCP MX v1.0: E8M0 shared scale per 32 elements, E4M3 elements)


def mxfp8_quantize(w_f32: np.ndarray, group_size: int = 32):
    """Returns (weight_u32 [N, K/4], scales_u8 [N, K/32])."""
    w = np.asarray(w_f32, dtype=np.float32).astype(np.float64)
    n, k = w.shape
    assert k % group_size == 0
    g = w.reshape(n, k // group_size, group_size)
    amax = np.abs(g).max(axis=2)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(amax > 0, amax, 1.0))) - 8.0  # emax(E4M3) = 8
    e = np.where(amax > 0, e, -127.0)
    e = np.clip(e, -127.0, 127.0)
    s_code = (e + 127.0).astype(np.uint8)
    scale = np.exp2(e)[:, :, None]
    codes = e4m3_encode(g / scale).reshape(n, k)
    return codes.view(np.uint8).reshape(n, k // 4, 4).copy().view(np.uint32).reshape(n, k // 4), s_code


def mxfp8_dequantize(weight_u32, scales_u8, k: int, group_size: int = 32):
    """bf16 values of E4M3 * 2**(s-127), rounded once (exact in range)."""
    w = np.ascontiguousarray(np.asarray(weight_u32, dtype=np.uint32))
    n = w.shape[0]
    codes = w.view(np.uint8).reshape(n, -1)[:, :k]
    v = e4m3_decode(codes)
    s = np.exp2(np.asarray(scales_u8, dtype=np.float64) - 127.0)
    s = np.repeat(s, group_size, axis=1)[:, :k]
    return rbf16_exact(v * s).reshape(n, k)


_E4M3_F32 = e4m3_decode(np.arange(256, dtype=np.uint8)).astype(np.float32)


def mxfp8_dequantize_fast(weight_u32, scales_u8, k: int, group_size: int = 32):
    """float32 evaluation for the timed CPU baseline: an E4M3 value times a
    power of two is exact in fp32 wherever the product is a normal fp32
    number, so this equals ``mxfp8_dequantize`` for every scale an
    ``mxfp8_quantize`` of finite bf16 weights produces."""
    w = np.ascontiguousarray(np.asarray(weight_u32, dtype=np.uint32))
    n = w.shape[0]
    v = _E4M3_F32[w.view(np.uint8).reshape(n, -1)[:, :k]].reshape(n, -1, group_size)
    s = np.ldexp(np.float32(1.0), np.asarray(scales_u8, dtype=np.int32) - 127).astype(np.float32)[:, :, None]
    return rbf16((v * s).astype(np.float32)).reshape(n, k)


def dequantize_fast(q: dict, k: int) -> np.ndarray:
    """float32 dequantization used only by the timed CPU baselines."""
    if q["mode"] == "affine":
        return affine_dequantize_fast(q["weight"], q["scales"], q["biases"], k, q["group_size"], q["bits"])
    return mxfp8_dequantize_fast(q["weight"], q["scales"], k, q["group_size"])


# --------------------------------------------------------------------------
# generic entry points mirroring the reference's (mode, group_size, bits)


def quantize(w, mode: str = "affine", group_size: int | None = None, bits: int | None = None):
    """``mx.quantize`` restatement.  Returns a dict of numpy arrays."""
    if mode == "affine":
        gs, b = group_size or 64, bits or 4
        wq, s, bi = affine_quantize(w, gs, b)
        return {"weight": wq, "scales": s, "biases": bi, "group_size": gs, "bits": b, "mode": mode}
    if mode == "mxfp8":
        gs = group_size or 32
        wq, s = mxfp8_quantize(w, gs)
        return {"weight": wq, "scales": s, "group_size": gs, "bits": 8, "mode": mode}
    raise ValueError(f"unsupported quantization mode {mode!r}")


def dequantize(q: dict, k: int) -> np.ndarray:
    if q["mode"] == "affine":
        return affine_dequantize(q["weight"], q["scales"], q["biases"], k, q["group_size"], q["bits"])
    if q["mode"] == "mxfp8":
        return mxfp8_dequantize(q["weight"], q["scales"], k, q["group_size"])
    raise ValueError(q["mode"])
