"""GPU parity of the CUDA path against the numpy oracle, through the C ABI.

Bars: dequantized weights and quantizer outputs
bit-exact; elementwise kernels bit-exact (same rounding points, fp64 row
statistics); GEMM outputs within max-abs-rel <= 2e-2 and cosine >= 0.9995 of
the reference composition (in practice within 1 bf16 ulp on almost every
element: the only freedom is the fp32 accumulation order).
"""

import numpy as np
import pytest

from helpers import bf16_bits, from_dev_bf16, normal_bf16, normal_f32, rng, to_dev, to_dev_bf16, ulp_diff_bf16
from oracle import quant as oq
from oracle import ref_ops as ro
from oracle.bf16 import f32_to_bf16_bits

pytestmark = pytest.mark.gpu

MAX_ABS_REL = 2e-2
COS_MIN = 0.9995


def _torch():
    import torch

    return torch


def _ltxq():
    import ltxq

    return ltxq


def _u32(t) -> np.ndarray:
    torch = _torch()
    return t.view(torch.int32).cpu().numpy().view(np.uint32)


def qlinear_from_oracle(q: dict, bias_np=None, n=None, k=None):
    ltxq = _ltxq()
    torch = _torch()
    w = to_dev(q["weight"])
    if q["mode"] == "affine":
        s = to_dev(q["scales"])
        b = to_dev(q["biases"])
    else:
        s = torch.from_numpy(q["scales"].copy()).cuda()
        b = None
    bias = to_dev_bf16(bias_np) if bias_np is not None else None
    return ltxq.QuantizedLinear(w, s, b, bias, group_size=q["group_size"], bits=q["bits"], mode=q["mode"],
                                in_features=k, out_features=n)


def assert_close(out, ref, what=""):
    mar = ro.max_abs_rel(out, ref)
    cos = ro.cosine(out, ref)
    assert mar <= MAX_ABS_REL and cos >= COS_MIN, f"{what}: max_abs_rel={mar:.3e} cos={cos:.6f}"
    return mar, cos


# ----------------------------------------------------------------- quantizer


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("gs", [64, 32, 128])
def test_affine_quantize_bit_exact(cuda, bits, gs):
    torch = _torch()
    ltxq = _ltxq()
    W = normal_bf16(rng(1), (256, 512), 0.02)
    ql = ltxq.QuantizedLinear.from_linear(to_dev_bf16(W), mode="affine", bits=bits, group_size=gs)
    torch.cuda.synchronize()
    wq, s, b = oq.affine_quantize(W, gs, bits)
    assert np.array_equal(_u32(ql.weight), wq)
    assert np.array_equal(bf16_bits(ql.scales), s)
    assert np.array_equal(bf16_bits(ql.biases), b)


def test_mxfp8_quantize_bit_exact(cuda):
    torch = _torch()
    ltxq = _ltxq()
    g = rng(2)
    W = normal_bf16(g, (128, 1024), 0.02)
    W[0, :32] = 0.0  # all-zero group
    W[1, :32] *= 1e-30  # tiny group (E4M3 subnormals / zero codes)
    W[2, 5] = 300.0  # large outlier
    W = ro.rbf16(W)
    ql = ltxq.QuantizedLinear.from_linear(to_dev_bf16(W), mode="mxfp8")
    torch.cuda.synchronize()
    wq, s = oq.mxfp8_quantize(W, 32)
    assert np.array_equal(ql.scales.cpu().numpy(), s)
    assert np.array_equal(_u32(ql.weight), wq)


# ----------------------------------------------------------------- dequantizer


@pytest.mark.parametrize("bits", [8, 4])
def test_affine_dequantize_bit_exact(cuda, bits):
    W = normal_bf16(rng(3), (384, 1024), 0.02)
    q = oq.quantize(W, "affine", 64, bits)
    ql = qlinear_from_oracle(q)
    deq = ql.dequantize()
    ref = oq.dequantize(q, 1024)
    assert np.array_equal(bf16_bits(deq), f32_to_bf16_bits(ref))


def test_mxfp8_dequantize_bit_exact(cuda):
    W = normal_bf16(rng(4), (256, 512), 0.05)
    q = oq.quantize(W, "mxfp8")
    # every E4M3 code, including subnormals and NaN-free extremes
    codes = np.arange(256, dtype=np.uint8)
    codes[0x7F] = 0x7E
    codes[0xFF] = 0xFE
    wb = q["weight"].view(np.uint8).reshape(256, 512)
    wb[0, :256] = codes
    wb[1, :256] = codes
    q["weight"] = wb.reshape(256, 128, 4).copy().view(np.uint32).reshape(256, 128)
    q["scales"][1, :8] = np.array([0, 1, 100, 127, 130, 200, 240, 246], dtype=np.uint8)
    ql = qlinear_from_oracle(q)
    deq = ql.dequantize()
    ref = oq.dequantize(q, 512)
    assert np.array_equal(bf16_bits(deq), f32_to_bf16_bits(ref))


# ----------------------------------------------------------------- elementwise


@pytest.mark.parametrize("C", [4096, 2048])
@pytest.mark.parametrize("norm", ["rms", "layer", "none"])
@pytest.mark.parametrize("vec", ["f32", "bf16"])
def test_adaln_modulate_matches_oracle(cuda, C, norm, vec):
    torch = _torch()
    ltxq = _ltxq()
    g = rng(5)
    x = normal_bf16(g, (1, 257, C))
    s = normal_f32(g, (1, 1, C), 0.1)
    t = normal_f32(g, (1, 1, C), 0.1)
    if vec == "bf16":
        s, t = ro.rbf16(s), ro.rbf16(t)
        sd, td = to_dev_bf16(s), to_dev_bf16(t)
    else:
        sd, td = torch.from_numpy(s).cuda(), torch.from_numpy(t).cuda()
    out = ltxq.adaln_modulate(to_dev_bf16(x), sd, td, 1e-6, norm)
    if norm == "none":
        ref = ro.modulate(x, s, t, vec == "bf16")
    else:
        ref = ro.adaln(x, s, t, 1e-6, norm, vec == "bf16")
    got = from_dev_bf16(out)
    ulps = ulp_diff_bf16(got, ref)
    # identical rounding points; the only freedom is the last fp32 ulp of the
    # row statistic, which can move a value across a bf16 rounding boundary
    assert ulps.max() <= 1 and (ulps > 0).mean() < 1e-3, (ulps.max(), (ulps > 0).mean())


def test_adaln_per_token_and_per_batch_vectors(cuda):
    torch = _torch()
    ltxq = _ltxq()
    g = rng(6)
    B, T, C = 2, 33, 2048
    x = normal_bf16(g, (B, T, C))
    s_tok = normal_f32(g, (B, T, C), 0.1)
    t_tok = normal_f32(g, (B, T, C), 0.1)
    out = from_dev_bf16(ltxq.adaln_norm_fused(to_dev_bf16(x), torch.from_numpy(s_tok).cuda(),
                                              torch.from_numpy(t_tok).cuda(), 1e-6))
    assert ulp_diff_bf16(out, ro.adaln(x, s_tok, t_tok)).max() <= 1
    s_b = normal_f32(g, (B, 1, C), 0.1)
    t_b = normal_f32(g, (B, 1, C), 0.1)
    out = from_dev_bf16(ltxq.adaln_norm_fused(to_dev_bf16(x), torch.from_numpy(s_b).cuda(),
                                              torch.from_numpy(t_b).cuda(), 1e-5))
    assert ulp_diff_bf16(out, ro.adaln(x, s_b, t_b, 1e-5)).max() <= 1


@pytest.mark.parametrize("mode", ["gated", "gate_then_add", "bf16_gate"])
def test_gated_add_bit_exact(cuda, mode):
    torch = _torch()
    ltxq = _ltxq()
    g = rng(7)
    r = normal_bf16(g, (1, 300, 4096))
    b = normal_bf16(g, (1, 300, 4096))
    gate = normal_f32(g, (1, 1, 4096), 0.5)
    if mode == "bf16_gate":
        gate = ro.rbf16(gate)
        gd = to_dev_bf16(gate)
    else:
        gd = torch.from_numpy(gate).cuda()
    out = from_dev_bf16(ltxq.gated_add_fused(to_dev_bf16(r), to_dev_bf16(b), gd, gate_then_add=(mode == "gate_then_add")))
    if mode == "gated":
        ref = ro.gated_add(r, b, gate)
    elif mode == "gate_then_add":
        ref = ro.gate_then_add(r, b, gate)
    else:
        ref = ro.gated_add(r, b, gate, gate_bf16=True)
    assert np.array_equal(f32_to_bf16_bits(out), f32_to_bf16_bits(ref))


def test_head_gate_matches_oracle(cuda):
    ltxq = _ltxq()
    g = rng(8)
    o = normal_bf16(g, (100, 32 * 128))
    lg = normal_bf16(g, (100, 32), 2.0)
    out = from_dev_bf16(ltxq.head_gate(to_dev_bf16(o), to_dev_bf16(lg), 32))
    assert ulp_diff_bf16(out, ro.head_gate(o, lg, 32)).max() <= 1


# ----------------------------------------------------------------- quantized GEMM


def _gemm_case(M, K, N, mode, bits, seed=9, with_bias=True):
    g = rng(seed)
    x = normal_bf16(g, (M, K))
    W = normal_bf16(g, (N, K), 0.02)
    bias = normal_bf16(g, (N,), 0.01) if with_bias else None
    gs = 32 if mode == "mxfp8" else 64
    q = oq.quantize(W, mode, gs, bits)
    deq = oq.dequantize(q, K)
    return x, q, deq, bias


@pytest.mark.parametrize("M", [1, 64, 100, 128, 200, 256, 700])
@pytest.mark.parametrize("qcfg", [("affine", 8), ("affine", 4), ("mxfp8", 8)])
def test_qlinear_matches_oracle(cuda, M, qcfg):
    torch = _torch()
    mode, bits = qcfg
    K, N = 512, 384
    x, q, deq, bias = _gemm_case(M, K, N, mode, bits)
    ql = qlinear_from_oracle(q, bias, N, K)
    out = from_dev_bf16(ql(to_dev_bf16(x)))
    ref = ro.linear(x, deq, bias)
    assert_close(out, ref, f"M={M} {qcfg}")
    # the only freedom is the fp32 summation order: nearly all bits agree (a
    # 1-ulp flip of bf16(acc) can become several ulps after the bias add
    # cancels, so only the fraction of differing elements is bounded)
    ulps = ulp_diff_bf16(out, ref)
    assert (ulps > 0).mean() < 0.01, (ulps.max(), (ulps > 0).mean())
    # and the plain torch fp32 reference of the same op agrees too
    xt = to_dev_bf16(x).float()
    wt = to_dev_bf16(deq).float()
    tref = ((xt @ wt.t()).to(torch.bfloat16).float() + to_dev_bf16(bias).float()).to(torch.bfloat16)
    assert_close(out, from_dev_bf16(tref), "torch fp32 reference")


@pytest.mark.parametrize("epi", ["gelu", "gated", "gate_then_add", "nobias"])
def test_qlinear_epilogues(cuda, epi):
    torch = _torch()
    M, K, N = 300, 512, 512
    x, q, deq, bias = _gemm_case(M, K, N, "affine", 8, seed=10, with_bias=(epi != "nobias"))
    ql = qlinear_from_oracle(q, bias, N, K)
    g = rng(11)
    res = normal_bf16(g, (M, N))
    gate = normal_f32(g, (1, N), 0.5)
    xd = to_dev_bf16(x)
    if epi == "gelu":
        out = ql(xd, gelu=True)
        ref = ro.gelu_approx(ro.linear(x, deq, bias))
    elif epi in ("gated", "gate_then_add"):
        out = ql(xd, residual=to_dev_bf16(res), gate=torch.from_numpy(gate).cuda(), gate_then_add=(epi != "gated"))
        y = ro.linear(x, deq, bias)
        ref = ro.gated_add(res, y, gate) if epi == "gated" else ro.gate_then_add(res, y, gate)
    else:
        out = ql(xd)
        ref = ro.linear(x, deq, None)
    assert_close(from_dev_bf16(out), ref, epi)


def test_adaln_qlinear_gated_config1_small(cuda):
    """BASELINE config 1 structure at a reduced M (full size in test_gpu_configs)."""
    torch = _torch()
    g = rng(0)
    M, C = 256, 1024
    x = normal_bf16(g, (1, M, C))
    shift = ro.rbf16(normal_f32(g, (1, C), 0.1))
    scale = ro.rbf16(normal_f32(g, (1, C), 0.1))
    gate = ro.rbf16(normal_f32(g, (1, C), 0.1))
    W = normal_bf16(g, (C, C), 0.02)
    b = normal_bf16(g, (C,), 0.01)
    q = oq.quantize(W, "affine", 64, 8)
    deq = oq.dequantize(q, C)
    ql = qlinear_from_oracle(q, b, C, C)
    for norm in ("layer", "rms"):
        out = ql(to_dev_bf16(x), residual=to_dev_bf16(x), gate=to_dev_bf16(gate),
                 adaln=(to_dev_bf16(scale), to_dev_bf16(shift), 1e-6, norm))
        ref = ro.adaln_linear_gated(x, scale, shift, gate, deq, b, 1e-6, norm, vec_bf16=True)
        assert_close(from_dev_bf16(out), ref, norm)
    torch.cuda.synchronize()


def test_feed_forward_sublayer_small(cuda):
    torch = _torch()
    ltxq = _ltxq()
    g = rng(12)
    M, D = 200, 512
    x = normal_bf16(g, (1, M, D))
    w_in = normal_bf16(g, (4 * D, D), 0.02)
    b_in = normal_bf16(g, (4 * D,), 0.01)
    w_out = normal_bf16(g, (D, 4 * D), 0.02)
    b_out = normal_bf16(g, (D,), 0.01)
    s = normal_f32(g, (1, 1, D), 0.1)
    t = normal_f32(g, (1, 1, D), 0.1)
    gate = normal_f32(g, (1, 1, D), 0.1)
    qi = oq.quantize(w_in, "affine", 64, 4)
    qo = oq.quantize(w_out, "affine", 64, 4)
    ff = ltxq.FeedForward(qlinear_from_oracle(qi, b_in, 4 * D, D), qlinear_from_oracle(qo, b_out, D, 4 * D))
    out = ff.sublayer(to_dev_bf16(x), torch.from_numpy(s).cuda(), torch.from_numpy(t).cuda(),
                      torch.from_numpy(gate).cuda())
    ref = ro.ff_sublayer(x, s, t, gate, oq.dequantize(qi, D), b_in, oq.dequantize(qo, 4 * D), b_out)
    assert_close(from_dev_bf16(out), ref, "ff sublayer")
    plain = ff(to_dev_bf16(x))
    ref2 = ro.feed_forward(x, oq.dequantize(qi, D), b_in, oq.dequantize(qo, 4 * D), b_out)
    assert_close(from_dev_bf16(plain), ref2, "ff plain")


def test_no_device_error_after_suite(cuda):
    from ltxq import _lib

    assert _lib.device_error() == 0


@pytest.mark.parametrize("gs,K,bits", [(32, 512, 8), (128, 1024, 4), (64, 320, 8), (64, 448, 4)])
def test_qlinear_group_sizes_and_unaligned_group_rows(cuda, gs, K, bits):
    """Group sizes 32/128 and K whose group-parameter rows are not 16-byte
    blocks (the scalar group-load path)."""
    M, N = 300, 256
    g = rng(13)
    x = normal_bf16(g, (M, K))
    W = normal_bf16(g, (N, K), 0.02)
    bias = normal_bf16(g, (N,), 0.01)
    q = oq.quantize(W, "affine", gs, bits)
    deq = oq.dequantize(q, K)
    out = from_dev_bf16(qlinear_from_oracle(q, bias, N, K)(to_dev_bf16(x)))
    assert_close(out, ro.linear(x, deq, bias), f"gs={gs} K={K}")
    assert (ulp_diff_bf16(out, ro.linear(x, deq, bias)) > 0).mean() < 0.01


@pytest.mark.parametrize("heads,d,with_pe,strided", [(32, 128, True, True), (32, 64, True, False), (8, 128, False, True)])
def test_qk_norm_rope_matches_oracle(cuda, heads, d, with_pe, strided):
    """Fused QK RMSNorm + split RoPE against the oracle (attention.py:320-329,
    rope.py:53-90) and against the plain torch fp32 reference."""
    import torch

    import ltxq
    from ltxq.block import apply_split_rope, rms_norm_weighted
    from oracle import block as ob

    g = rng(14)
    T, W = 77, heads * d
    base = normal_bf16(g, (T, W + 40 if strided else W))
    x = base[:, 8:8 + W] if strided else base
    w = (1.0 + normal_f32(g, (W,), 0.1)).astype(np.float32)
    ang = g.uniform(0, 6.28, (heads, T, d // 2)).astype(np.float32)
    cos, sin = np.cos(ang), np.sin(ang)
    xd = to_dev_bf16(base)[None]
    xd = xd[:, :, 8:8 + W] if strided else xd
    pe = (torch.from_numpy(cos)[None].cuda(), torch.from_numpy(sin)[None].cuda()) if with_pe else None
    out = from_dev_bf16(ltxq.kernels.qk_norm_rope(xd, torch.from_numpy(w).cuda(), heads, 1e-6, pe)[0])
    ref = ob.rms_norm_weighted(x, w)
    if with_pe:
        ref = ob.apply_split_rope(ref, cos, sin, heads)
    ulps = ulp_diff_bf16(out, ref)
    assert ulps.max() <= 1 and (ulps > 0).mean() < 1e-3, (ulps.max(), (ulps > 0).mean())
    tref = rms_norm_weighted(xd, torch.from_numpy(w).cuda(), 1e-6)
    if with_pe:
        tref = apply_split_rope(tref, pe, heads)
    assert_close(out, from_dev_bf16(tref[0]), "torch fp32 reference")
