"""GPU parity of the CUDA path against the numpy oracle, through the C ABI.

Bars (the path's stated parity requirements): dequantized weights and quantizer outputs
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
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits

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
    assert ql.data_flags() == 0  # scales above 134: the general conversion
    deq = ql.dequantize()
    ref = oq.dequantize(q, 512)
    assert np.array_equal(bf16_bits(deq), f32_to_bf16_bits(ref))


def test_mxfp8_short_conversion_exhaustive(cuda):
    """Every finite E4M3 code under every E8M0 scale the short conversion
    accepts (0..134, bf16-subnormal results included) dequantizes to the
    oracle's bits; the same data with NaN codes takes the general path."""
    from ltxq import _lib

    rows = 135
    codes = np.tile(np.arange(256, dtype=np.uint8), (rows, 1))
    codes[(codes & 0x7F) == 0x7F] = 0x00
    scales = np.repeat(np.arange(rows, dtype=np.uint8)[:, None], 256 // 32, axis=1)
    q = {"weight": codes.reshape(rows, 64, 4).copy().view(np.uint32).reshape(rows, 64), "scales": scales,
         "group_size": 32, "bits": 8, "mode": "mxfp8"}
    ql = qlinear_from_oracle(q)
    assert ql.data_flags() == _lib.QW_MXFP8_FINITE
    ref = f32_to_bf16_bits(oq.dequantize(q, 256))
    assert np.array_equal(bf16_bits(ql.dequantize()), ref)
    ql.fast_path = False
    assert np.array_equal(bf16_bits(ql.dequantize()), ref)


@pytest.mark.parametrize("plant", ["none", "nan_code_pos", "nan_code_neg", "scale_135", "scale_134"])
def test_qweight_scan_flags(cuda, plant):
    from ltxq import _lib

    W = normal_bf16(rng(5), (64, 1024), 0.05)
    q = oq.quantize(W, "mxfp8")
    wb = q["weight"].view(np.uint8).reshape(64, 1024)
    if plant == "nan_code_pos":
        wb[63, 1023] = 0x7F
    elif plant == "nan_code_neg":
        wb[17, 5] = 0xFF
    elif plant == "scale_135":
        q["scales"][40, 31] = 135
    elif plant == "scale_134":
        q["scales"][40, 31] = 134
    q["weight"] = wb.reshape(64, 256, 4).copy().view(np.uint32).reshape(64, 256)
    ql = qlinear_from_oracle(q)
    want = _lib.QW_MXFP8_FINITE if plant in ("none", "scale_134") else 0
    assert ql.data_flags() == want
    got, ref = bf16_bits(ql.dequantize()), f32_to_bf16_bits(oq.dequantize(q, 1024))
    nan = lambda b: ((b & 0x7F80) == 0x7F80) & ((b & 0x7F) != 0)  # noqa: E731  (any NaN payload)
    assert np.array_equal(nan(got), nan(ref))
    assert np.array_equal(got[~nan(ref)], ref[~nan(ref)])


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


def test_head_gate_reads_strided_logits(cuda):
    """Gate logits as a column slice of a fused Q|K|V|gate output (rows at
    stride 3 * width + heads, batch 2) are read in place: the result equals
    the contiguous call bit for bit, bf16 and MX outputs alike."""
    import torch

    from ltxq import kernels as K

    g = rng(81)
    B, T, heads, d = 2, 150, 32, 128
    W = heads * d
    o = to_dev_bf16(normal_bf16(g, (B * T, W))).view(B, T, W)
    fused = to_dev_bf16(normal_bf16(g, (B * T, 3 * W + heads), 2.0)).view(B, T, 3 * W + heads)
    gl = fused[:, :, 3 * W:]
    assert not gl.is_contiguous()
    ref = K.head_gate(o, gl.contiguous(), heads)
    got = K.head_gate(o, gl, heads)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    assert ulp_diff_bf16(from_dev_bf16(got).reshape(B * T, W),
                         ro.head_gate(from_dev_bf16(o).reshape(B * T, W),
                                      from_dev_bf16(gl.contiguous()).reshape(B * T, heads), heads)).max() <= 1
    from test_gpu_mx_fused import _assert_same_terms

    mx_ref = K.head_gate(o, gl.contiguous(), heads, mx_terms=2)
    mx_got = K.head_gate(o, gl, heads, mx_terms=2)
    torch.cuda.synchronize()
    _assert_same_terms(mx_got, mx_ref, "strided-logit gate, MX out")


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
@pytest.mark.parametrize("split_k", [True, False])
def test_qlinear_matches_oracle(cuda, M, qcfg, split_k):
    """split_k=True: these shapes have few output tiles, so the pair kernel
    splits K and splitk_reduce_kernel sums the partials; split_k=False: the
    single-CTA kernel (M <= 128) or the unsplit pair kernel."""
    torch = _torch()
    mode, bits = qcfg
    K, N = 512, 384
    x, q, deq, bias = _gemm_case(M, K, N, mode, bits)
    ql = qlinear_from_oracle(q, bias, N, K)
    out = from_dev_bf16(ql(to_dev_bf16(x), split_k=split_k))
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
@pytest.mark.parametrize("M,split_k", [(300, True), (300, False), (96, False)])
def test_qlinear_epilogues(cuda, epi, M, split_k):
    torch = _torch()
    K, N = 512, 512
    x, q, deq, bias = _gemm_case(M, K, N, "affine", 8, seed=10, with_bias=(epi != "nobias"))
    ql = qlinear_from_oracle(q, bias, N, K)
    g = rng(11)
    res = normal_bf16(g, (M, N))
    gate = normal_f32(g, (1, N), 0.5)
    xd = to_dev_bf16(x)
    if epi == "gelu":
        out = ql(xd, gelu=True, split_k=split_k)
        ref = ro.gelu_approx(ro.linear(x, deq, bias))
    elif epi in ("gated", "gate_then_add"):
        out = ql(xd, residual=to_dev_bf16(res), gate=torch.from_numpy(gate).cuda(), gate_then_add=(epi != "gated"),
                 split_k=split_k)
        y = ro.linear(x, deq, bias)
        ref = ro.gated_add(res, y, gate) if epi == "gated" else ro.gate_then_add(res, y, gate)
    else:
        out = ql(xd, split_k=split_k)
        ref = ro.linear(x, deq, None)
    assert_close(from_dev_bf16(out), ref, epi)


def _zero_affine_linear(N, K, bias_bits):
    """Affine int8 linear whose weights dequantize to exactly 0, with the
    given bf16 bias bit patterns: its output is bf16(0 + bias) per feature."""
    torch = _torch()
    ltxq = _ltxq()
    w = torch.zeros(N, K // 4, dtype=torch.int32, device="cuda")
    s = torch.zeros(N, K // 64, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(N, K // 64, dtype=torch.bfloat16, device="cuda")
    bias = torch.from_numpy(bias_bits.astype(np.uint16).view(np.int16)).cuda().view(torch.bfloat16)
    return ltxq.QuantizedLinear(w, s, b, bias, group_size=64, bits=8, mode="affine", in_features=K, out_features=N)


def test_gelu_epilogue_exhaustive(cuda):
    """The GELU epilogue on every bf16 input: the pair kernel's table path,
    the single-CTA kernel's direct evaluation and the split-K reduce kernel
    give identical bits, and they match the oracle's gelu_approx."""
    torch = _torch()
    pats = np.arange(0x10000, dtype=np.uint32).astype(np.uint16)
    K = 512
    # pair kernel, unsplit (256 feature tiles > half the clusters)
    pair = from_dev_bf16(_zero_affine_linear(0x10000, K, pats)(torch.ones(256, K, dtype=torch.bfloat16,
                                                                              device="cuda"), gelu=True))
    # single-CTA kernel (M <= 128, no split-K workspace)
    single = from_dev_bf16(_zero_affine_linear(0x10000, K, pats)(torch.ones(64, K, dtype=torch.bfloat16,
                                                                                device="cuda"), gelu=True,
                                                                     split_k=False))
    # split-K reduce kernel: 8192 features per call (32 tiles -> 2 splits)
    parts = []
    for c in range(8):
        ql = _zero_affine_linear(8192, K, pats[c * 8192:(c + 1) * 8192])
        parts.append(from_dev_bf16(ql(torch.ones(64, K, dtype=torch.bfloat16, device="cuda"), gelu=True)))
    split = np.concatenate(parts, axis=1)
    bits = lambda a: f32_to_bf16_bits(a)  # noqa: E731
    for name, got in (("pair", pair), ("split", split)):
        same = (bits(got[0]) == bits(single[0])) | (np.isnan(got[0]) & np.isnan(single[0]))
        assert same.all(), (name, [hex(p) for p in pats[~same][:8]])
    assert (bits(pair) == bits(pair[:1])).all()  # every token row alike
    x = ro.rbf16(np.float32(0.0) + bf16_bits_to_f32(pats))
    with np.errstate(invalid="ignore", over="ignore"):
        ref = ro.gelu_approx(x)
    nan_ok = np.isnan(ref) == np.isnan(single[0])
    assert nan_ok.all(), [hex(p) for p in pats[~nan_ok][:8]]
    fin = ~np.isnan(ref)
    ulps = ulp_diff_bf16(single[0][fin], ref[fin])
    # the GPU evaluates tanh in fp32 (tanhf), the oracle in fp64: a rounding
    # boundary may separate them on a handful of inputs
    assert ulps.max() <= 1 and (ulps > 0).sum() <= 64, ((ulps > 0).sum(), ulps.max())


def test_gelu_epilogue_token_pairs_exhaustive(cuda):
    """The GELU epilogue with a different input on every token: token t's
    accumulator is the bf16 pattern t (x[t, 0] = pattern, the weight's first
    column 1, the rest 0), so every bf16x2 word of consecutive tokens holds
    two neighbouring patterns, and words with one half inside and one
    outside the tabulated range occur at each range edge.  The pair kernel
    (table, paired fast path) and the single-CTA kernel's direct evaluation
    give identical bits."""
    torch = _torch()
    ltxq = _ltxq()
    pats = np.arange(0x10000, dtype=np.uint32).astype(np.uint16)
    K, N = 64, 256
    x = torch.zeros(0x10000, K, dtype=torch.bfloat16, device="cuda")
    x[:, 0] = torch.from_numpy(pats.view(np.int16)).cuda().view(torch.bfloat16)
    w = torch.zeros(N, K // 4, dtype=torch.int32, device="cuda")
    w[:, 0] = 1  # code 1 at k = 0, code 0 elsewhere
    s = torch.ones(N, K // 64, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(N, K // 64, dtype=torch.bfloat16, device="cuda")
    ql = ltxq.QuantizedLinear(w, s, b, None, group_size=64, bits=8, mode="affine", in_features=K, out_features=N)
    pair = from_dev_bf16(ql(x, gelu=True))[:, :8]  # every feature alike; 8 of them
    bits = lambda a: f32_to_bf16_bits(a)  # noqa: E731
    assert (bits(pair) == bits(pair[:, :1])).all()
    pair = pair[:, 0]
    # reference: the single-CTA kernel's direct gelu_ref of every pattern (as bias, weights 0)
    direct = from_dev_bf16(_zero_affine_linear(0x10000, 512, pats)(
        torch.ones(64, 512, dtype=torch.bfloat16, device="cuda"), gelu=True, split_k=False))[0]
    # the accumulator of pattern 0x8000 (-0) is +0 (-0 + 0 products); every other
    # pattern is its own accumulator
    keep = pats != 0x8000
    same = (bits(pair) == bits(direct)) | (np.isnan(pair) & np.isnan(direct))
    assert same[keep].all(), [hex(p) for p in pats[keep & ~same][:8]]


def test_split_k_deterministic(cuda):
    """Split-K partials are summed in split order: repeated calls agree bit
    for bit."""
    torch = _torch()
    x, q, deq, bias = _gemm_case(201, 2048, 2048, "mxfp8", 8, seed=21)
    ql = qlinear_from_oracle(q, bias, 2048, 2048)
    xd = to_dev_bf16(x)
    a = ql(xd)
    b = ql(xd)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert_close(from_dev_bf16(a), ro.linear(x, deq, bias), "split-K 201x2048x2048")


def test_adaln_qlinear_gated_config1_small(cuda):
    """Benchmark config 1 structure (fused AdaLN + int8 linear + gated residual) at a reduced M."""
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


@pytest.mark.parametrize("heads,d,with_pe,strided", [(32, 128, True, True), (32, 64, True, False), (8, 128, False, True),
                                                     (6, 64, True, True)])  # 6 x 64: the warp-per-row form
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


@pytest.mark.parametrize("mode,bits,smax", [("mxfp8", 8, 134), ("mxfp8", 8, 246), ("affine", 8, 0), ("affine", 4, 0)])
@pytest.mark.parametrize("M,split_k", [(256, True), (256, False), (128, False)])
def test_gemm_dequant_exact_through_identity(cuda, mode, bits, smax, M, split_k):
    """x = identity makes y[m, n] = dequant(W)[n, m] with one nonzero product
    per output, so the in-GEMM dequantization is checked bit for bit over
    every code: mxfp8 rows carry all finite E4M3 codes under E8M0 scales
    10..smax (normal bf16 results, no overflow; smax 134 takes the short
    conversion, 246 the general one), affine rows all 2^bits codes under
    varied bf16 scales / biases."""
    torch = _torch()
    ltxq = _ltxq()
    K = N = M
    g = rng(30)
    if mode == "mxfp8":
        # row n holds codes k + 128 (n % 2) (mod 256): every code appears for K >= 128
        codes = ((np.arange(K, dtype=np.uint32)[None, :] + 128 * (np.arange(N, dtype=np.uint32)[:, None] % 2))
                 % 256).astype(np.uint8)
        codes[(codes & 0x7F) == 0x7F] = 0  # NaN codes: 0 * NaN would poison the row sums
        scales = (10 + (np.arange(N * (K // 32)) * 7) % (smax - 9)).astype(np.uint8).reshape(N, K // 32)
        q = {"weight": codes.reshape(N, K // 4, 4).copy().view(np.uint32).reshape(N, K // 4), "scales": scales,
             "group_size": 32, "bits": 8, "mode": "mxfp8"}
    else:
        per = 1 << bits
        qv = np.tile(np.arange(K, dtype=np.uint32) % per, (N, 1))
        qv = (qv + np.arange(N, dtype=np.uint32)[:, None]) % per
        scales = f32_to_bf16_bits(normal_f32(g, (N, K // 64), 0.01))
        biases = f32_to_bf16_bits(normal_f32(g, (N, K // 64), 0.5))
        q = {"weight": oq.pack_bits(qv, bits), "scales": scales, "biases": biases, "group_size": 64, "bits": bits,
             "mode": "affine"}
    deq = oq.dequantize(q, K)
    ql = qlinear_from_oracle(q, None, N, K)
    if mode == "mxfp8":
        assert ql.data_flags() == (1 if smax <= 134 else 0)
    eye = torch.eye(M, K, dtype=torch.bfloat16, device="cuda")
    y = bf16_bits(ql(eye, split_k=split_k))
    want = f32_to_bf16_bits(deq.T)
    # +0 and -0 compare equal (a -0 weight times 1 plus +0 products sums to +0)
    both_zero = ((y & 0x7FFF) == 0) & ((want & 0x7FFF) == 0)
    diff = (y != want) & ~both_zero
    assert not diff.any(), (np.argwhere(diff)[:5], y[diff][:5], want[diff][:5])


@pytest.mark.parametrize("epi", ["none", "gelu", "gated_per_token"])
def test_qlinear_hybrid_schedule(cuda, epi):
    """1152 tokens x 4096 features: 80 output tiles on 74 clusters, so the
    first tiles run whole and the last ones are split along K (the video rows
    of one rank of 8).  Matches the oracle, equals the unsplit run to within
    fp32 summation order, and repeats bit for bit."""
    torch = _torch()
    M, K, N = 1152, 1536, 4096
    x, q, deq, bias = _gemm_case(M, K, N, "mxfp8", 8, seed=40)
    ql = qlinear_from_oracle(q, bias, N, K)
    xd = to_dev_bf16(x)
    kw, ref = {}, ro.linear(x, deq, bias)
    if epi == "gelu":
        kw, ref = {"gelu": True}, ro.gelu_approx(ref)
    elif epi == "gated_per_token":
        g = rng(41)
        res = normal_bf16(g, (M, N))
        gate = normal_f32(g, (M, N), 0.5)
        kw = {"residual": to_dev_bf16(res), "gate": torch.from_numpy(gate).cuda()}
        ref = ro.gated_add(res, ref, gate)
    a = ql(xd, **kw)
    b = ql(xd, **kw)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert_close(from_dev_bf16(a), ref, f"hybrid {epi}")
    whole = from_dev_bf16(ql(xd, split_k=False, **kw))
    assert (ulp_diff_bf16(from_dev_bf16(a), whole) > 0).mean() < 0.02


def _pt_linear(WT_q, bias, n, k):
    """QuantizedLinear over pretransposed mxfp8 arrays (W^T packed along N)."""
    ltxq = _ltxq()
    torch = _torch()
    return ltxq.QuantizedLinear(to_dev(WT_q["weight"]), torch.from_numpy(WT_q["scales"].copy()).cuda(), None,
                                to_dev_bf16(bias) if bias is not None else None, group_size=32, bits=8,
                                mode="mxfp8", pretransposed=True, in_features=k, out_features=n)


@pytest.mark.parametrize("M,split_k,epi", [(700, True, "none"), (201, True, "gelu"), (201, False, "none"),
                                           (1152, True, "gated")])
def test_qlinear_pretransposed_matches_oracle(cuda, M, split_k, epi):
    """The cache's mxfp8-blocks-pretranspose layout (transformer_cache.py:177-193,
    1240-1244): y = x @ dequant(W^T) + b, against _PretransposedQuantizedLinear's
    composition (ref_ops.linear_pretransposed)."""
    torch = _torch()
    K, N = 1024, 768
    g = rng(50)
    x = normal_bf16(g, (M, K))
    W = normal_bf16(g, (N, K), 0.02)
    bias = normal_bf16(g, (N,), 0.01)
    qT = oq.quantize(np.ascontiguousarray(W.T), "mxfp8")
    deqT = oq.dequantize(qT, N)  # [K, N]
    ql = _pt_linear(qT, bias, N, K)
    xd = to_dev_bf16(x)
    ref = ro.linear_pretransposed(x, deqT, bias)
    kw = {"split_k": split_k}
    if epi == "gelu":
        kw["gelu"] = True
        ref = ro.gelu_approx(ref)
    elif epi == "gated":
        res = normal_bf16(g, (M, N))
        gate = normal_f32(g, (1, N), 0.5)
        kw.update(residual=to_dev_bf16(res), gate=torch.from_numpy(gate).cuda())
        ref = ro.gated_add(res, ref, gate)
    out = from_dev_bf16(ql(xd, **kw))
    assert_close(out, ref, f"pretransposed M={M} {epi}")
    assert (ulp_diff_bf16(out, ref) > 0).mean() < 0.02


@pytest.mark.parametrize("smax", [134, 246])
@pytest.mark.parametrize("split_k", [True, False])
def test_pretransposed_dequant_exact_through_identity(cuda, smax, split_k):
    """x = identity: y[k, n] = dequant(W^T)[k, n] bit for bit, every finite
    E4M3 code under scales 10..smax (the short and the general conversion)."""
    torch = _torch()
    K = M = 256
    N = 512
    codes = ((np.arange(N, dtype=np.uint32)[None, :] + 7 * np.arange(K, dtype=np.uint32)[:, None]) % 256).astype(np.uint8)
    codes[(codes & 0x7F) == 0x7F] = 0
    scales = (10 + (np.arange(K * (N // 32)) * 5) % (smax - 9)).astype(np.uint8).reshape(K, N // 32)
    qT = {"weight": codes.reshape(K, N // 4, 4).copy().view(np.uint32).reshape(K, N // 4), "scales": scales,
          "group_size": 32, "bits": 8, "mode": "mxfp8"}
    ql = _pt_linear(qT, None, N, K)
    assert ql.data_flags() == (1 if smax <= 134 else 0)
    y = bf16_bits(ql(torch.eye(M, K, dtype=torch.bfloat16, device="cuda"), split_k=split_k))
    want = f32_to_bf16_bits(oq.dequantize(qT, N))
    both_zero = ((y & 0x7FFF) == 0) & ((want & 0x7FFF) == 0)
    diff = (y != want) & ~both_zero
    assert not diff.any(), (np.argwhere(diff)[:5], y[diff][:5], want[diff][:5])


def test_strided_vector_views_match_contiguous(cuda):
    """AdaLN vectors and gates given as strided views of a (B, 1, 9, C) table
    sum (the block's get_ada_values slices, transformer.py:286-309) give the
    same bits as contiguous copies, per batch entry."""
    torch = _torch()
    ltxq = _ltxq()
    g = torch.Generator(device="cuda")
    g.manual_seed(60)
    B, T, C = 2, 96, 1024
    x = torch.randn(B, T, C, generator=g, device="cuda").to(torch.bfloat16)
    vals = torch.randn(B, 1, 9, C, generator=g, device="cuda") * 0.1
    sc, sh = vals[:, :, 1], vals[:, :, 0]
    assert not sc.is_contiguous()
    a = ltxq.adaln_modulate(x, sc, sh, 1e-6)
    b = ltxq.adaln_modulate(x, sc.contiguous(), sh.contiguous(), 1e-6)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    W = normal_bf16(rng(61), (512, C), 0.02)
    q = oq.quantize(W, "mxfp8")
    ql = qlinear_from_oracle(q, None, 512, C)
    res = torch.randn(B, T, 512, generator=g, device="cuda").to(torch.bfloat16)
    gv = (torch.randn(B, 1, 9, 512, generator=g, device="cuda") * 0.5)[:, :, 2]
    y1 = ql(a, residual=res, gate=gv)
    y2 = ql(a, residual=res, gate=gv.contiguous())
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))


@pytest.mark.parametrize("heads,d,batch", [(32, 128, 1), (32, 64, 2)])
def test_qk_norm_rope_pair_equals_two_calls(cuda, heads, d, batch):
    """ltxq_qk_norm_rope_pair (Q and K in one pass, the tables read once)
    gives the bits of two ltxq_qk_norm_rope calls; Q strided as a column
    slice of a fused projection output."""
    import torch

    import ltxq

    g = torch.Generator(device="cuda")
    g.manual_seed(21)
    T, W = 300, heads * d
    fused = torch.randn(batch, T, 3 * W + 32, generator=g, device="cuda").to(torch.bfloat16)
    q, k = fused[..., :W], fused[..., W:2 * W]
    wq = 1.0 + 0.1 * torch.randn(W, generator=g, device="cuda")
    wk = 1.0 + 0.1 * torch.randn(W, generator=g, device="cuda")
    ang = torch.rand(batch, heads, T, d // 2, generator=g, device="cuda") * 6.28
    pe = (torch.cos(ang), torch.sin(ang))
    oq, ok = ltxq.kernels.qk_norm_rope_pair(q, k, wq, wk, heads, 1e-6, pe)
    rq = ltxq.kernels.qk_norm_rope(q, wq, heads, 1e-6, pe)
    rk = ltxq.kernels.qk_norm_rope(k, wk, heads, 1e-6, pe)
    assert torch.equal(oq.view(torch.int16), rq.view(torch.int16))
    assert torch.equal(ok.view(torch.int16), rk.view(torch.int16))
