"""The reference's MLX op compositions for the hot path, restated in numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Every function keeps the reference's rounding points: an MLX op on bf16
arrays produces a bf16 array (one RNE rounding per op); Python float
constants are weakly typed and take the array dtype; an op mixing a bf16
array with an fp32 array (the AdaLN tables are fp32, transformer.py:225,248)
computes in fp32 and the result is cast back with ``.astype(x.dtype)``.

Values are carried as float32 arrays holding bf16-representable numbers
where the reference has bf16 arrays.
"""

from __future__ import annotations

import math

import numpy as np

from . import _par
from .bf16 import rbf16

EPS = 1e-6


def _f32(a):
    return np.asarray(a, dtype=np.float32)


# --------------------------------------------------------------------------
# norms (mx.fast.rms_norm / mx.fast.layer_norm with no affine weight)


def rms_norm(x, eps: float = EPS):
    """``mx.fast.rms_norm(x, None, eps)`` (attention.py:305-317,
    transformer.py:36): fp32 statistics, output rounded to bf16."""
    x = _f32(x)
    ms = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True).astype(np.float32)
    inv = (1.0 / np.sqrt((ms + np.float32(eps)).astype(np.float64))).astype(np.float32)
    return rbf16(x * inv)


def layer_norm(x, eps: float = EPS):
    """``mx.fast.layer_norm(x, None, None, eps)`` (model.py:655,683): the
    non-affine LayerNorm, fp32 statistics, output rounded to bf16."""
    x = _f32(x)
    x64 = x.astype(np.float64)
    mu = x64.mean(axis=-1, keepdims=True)
    var = ((x64 - mu) ** 2).mean(axis=-1, keepdims=True).astype(np.float32)
    inv = (1.0 / np.sqrt((var + np.float32(eps)).astype(np.float64))).astype(np.float32)
    return rbf16((x - mu.astype(np.float32)) * inv)


def modulate(normed_bf16, scale, shift, vec_bf16: bool = False):
    """``(normed * (1 + scale) + shift).astype(bf16)``.

    fp32 vectors (the reference's production dtype): fp32 product, fp32 sum,
    one bf16 rounding.  bf16 vectors: every op rounds to bf16.
    """
    n = _f32(normed_bf16)
    s = _f32(scale)
    t = _f32(shift)
    if vec_bf16:
        one_p = rbf16(np.float32(1.0) + s)
        return rbf16(rbf16(n * one_p) + t)
    return rbf16((n * (np.float32(1.0) + s)).astype(np.float32) + t)


def adaln(x, scale, shift, eps: float = EPS, norm: str = "rms", vec_bf16: bool = False):
    """``_adaln_inline`` (transformer.py:21-37) / ``_adaln_norm_mlx``
    (fused_ops.py:192-201): RMSNorm then modulate.  ``norm="layer"`` gives the
    non-affine LayerNorm variant that benchmark config 1 names."""
    nrm = rms_norm(x, eps) if norm == "rms" else layer_norm(x, eps)
    return modulate(nrm, scale, shift, vec_bf16)


def modulate_no_norm(context, scale, shift, vec_bf16: bool = False):
    """Text cross-attention K/V modulation without a norm
    (transformer.py:379): ``(context * (1 + scale_kv) + shift_kv).astype``."""
    return modulate(context, scale, shift, vec_bf16)


def gated_add(residual, branch, gate, gate_bf16: bool = False):
    """``_residual_gate_inline(x, residual, gate)`` (transformer.py:40-50) /
    ``_gated_add_mlx`` (fused_ops.py:362-366): ``(x + branch * gate)``,
    fp32 math for an fp32 gate, cast to bf16."""
    r = _f32(residual)
    b = _f32(branch)
    g = _f32(gate)
    if gate_bf16:
        return rbf16(r + rbf16(b * g))
    return rbf16((b * g).astype(np.float32) + r)


def gate_then_add(residual, branch, gate, gate_bf16: bool = False):
    """Text cross-attention residual (transformer.py:387,484):
    ``cross = (out * gate).astype(bf16)``; ``vx = vx + cross`` (bf16 add)."""
    r = _f32(residual)
    b = _f32(branch)
    g = _f32(gate)
    cross = rbf16(b * g)
    return rbf16(r + cross)


# --------------------------------------------------------------------------
# GELU (nn.gelu_approx, feed_forward.py:8-14,102)

_C_GELU = float(rbf16(np.float32(0.044715)))
_C_SQRT = float(rbf16(np.float32(math.sqrt(2.0 / math.pi))))


def gelu_approx(x_bf16):
    """``0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 * x**3)))`` on a bf16
    array: each op rounds to bf16 and the constants are bf16.  (Large arrays
    run in row chunks on every host thread; element-wise, so the same bits.)"""
    x = _f32(x_bf16)
    if x.size >= _par.MIN_ELEMS:
        return _par.chunked(_gelu_approx, x)
    return _gelu_approx(x)


def _gelu_approx(x):
    x64 = x.astype(np.float64)
    x3 = rbf16(x64 * x64 * x64)  # x**3, exact in float64 for bf16 x
    t = rbf16(np.float32(_C_GELU) * x3)
    t = rbf16(x + t)
    t = rbf16(np.float32(_C_SQRT) * t)
    t = rbf16(np.tanh(t.astype(np.float64)).astype(np.float32))
    t = rbf16(np.float32(1.0) + t)
    h = rbf16(np.float32(0.5) * x)
    return rbf16(h * t)


def gelu_tanh_f32(x):
    """GELU-tanh evaluated in fp32 with a single final rounding (used only to
    bound the difference between the two evaluation orders in tests)."""
    x = _f32(x).astype(np.float64)
    y = 0.5 * x * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))
    return rbf16(y.astype(np.float32))


# --------------------------------------------------------------------------
# linear layers


def linear(x_bf16, w_deq_bf16, bias_bf16=None, threads: int | None = None):
    """``nn.QuantizedLinear`` / ``mx.quantized_matmul(..., transpose=True)``
    then ``+ bias`` (transformer_cache.py:181-193): fp32-accumulated matmul of
    bf16 activations with the bf16-dequantized weight, output rounded to bf16,
    then a bf16 bias add (second rounding)."""
    x = _f32(x_bf16)
    w = _f32(w_deq_bf16)
    y = rbf16(x @ w.T)
    if bias_bf16 is not None:
        y = rbf16(y + _f32(bias_bf16))
    return y


def linear_pretransposed(x_bf16, wT_deq_bf16, bias_bf16=None):
    """``_PretransposedQuantizedLinear`` (transformer_cache.py:177-193):
    ``quantized_matmul(x, Wq_T, transpose=False) + bias``."""
    x = _f32(x_bf16)
    y = rbf16(x @ _f32(wT_deq_bf16))
    if bias_bf16 is not None:
        y = rbf16(y + _f32(bias_bf16))
    return y


def feed_forward(x_bf16, w_in, b_in, w_out, b_out):
    """``FeedForward.__call__`` (feed_forward.py:64-112):
    project_out(gelu_approx(project_in(x)))."""
    h = gelu_approx(linear(x_bf16, w_in, b_in))
    return linear(h, w_out, b_out)


def adaln_linear_gated(x, scale, shift, gate, w_deq, bias, eps: float = EPS,
                       norm: str = "rms", vec_bf16: bool = False):
    """Benchmark config 1: ``out = x + gate * (modulate(norm(x)) @ W^T + b)``
    with the reference's rounding points."""
    a = adaln(x, scale, shift, eps, norm, vec_bf16)
    y = linear(a, w_deq, bias)
    return gated_add(x, y, gate, vec_bf16)


def ff_sublayer(x, scale, shift, gate, w_in, b_in, w_out, b_out, eps: float = EPS,
                norm: str = "rms", vec_bf16: bool = False):
    """Benchmark config 2 / transformer.py:629-650: AdaLN -> FF -> gated add."""
    a = adaln(x, scale, shift, eps, norm, vec_bf16)
    y = feed_forward(a, w_in, b_in, w_out, b_out)
    return gated_add(x, y, gate, vec_bf16)


def head_gate(out_bf16, gate_logits_bf16, heads: int):
    """Per-head attention gate (attention.py:559-601): ``gate =
    2*sigmoid(logits)`` (bf16 ops) and ``out * gate[..., None]`` per head."""
    o = _f32(out_bf16)
    lg = _f32(gate_logits_bf16)
    sig = rbf16((1.0 / (1.0 + np.exp(-lg.astype(np.float64)))).astype(np.float32))
    g = rbf16(np.float32(2.0) * sig)
    rows, width = o.shape
    d = width // heads
    return rbf16(o.reshape(rows, heads, d) * g[:, :, None]).reshape(rows, width)


def cosine(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return float(a @ b / (np.sqrt(a @ a) * np.sqrt(b @ b) + 1e-300))


def max_abs_rel(a, ref) -> float:
    """max|a - ref| / max|ref| (the path's stated tolerance measure: <= 2e-2)."""
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(a - ref).max() / max(np.abs(ref).max(), 1e-30))
