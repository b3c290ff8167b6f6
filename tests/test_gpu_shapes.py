"""GPU parity at the shapes the benchmarks run, against the numpy oracle.

The reference pins its fused ops at production shape (T = 14640, C = 4096 in
dmlsrc/LTX-2-MLX tests/test_fused_ops.py:44-72); these tests do the same for
the quantized linears and the block, at BASELINE.json's configurations:

* config 1 exactly: x [1, 1024, 4096], LayerNorm (as the config words it) and
  RMSNorm (the reference's block AdaLN) prologue with bf16 vectors, W 4096 x
  4096 affine int8 g64, gated residual; every output element is compared;
* the config-4 linears at full width for every quantization the cache holds
  (mxfp8 with the short and with the general conversion, affine int8 and int4
  g64): K = 2048 / 4096 / 16384, N up to 16384, on 9216 video rows (one GPU),
  1152 rows (one rank of 8: whole and K-split tiles in one launch), 201 audio
  rows (K-split) and 1024 text-context rows; the pretransposed mxfp8 layout;
* config 2 (the int4 FF sub-layer at 3456 tokens) and the per-rank shapes of
  config 5 (30576 x 2 video rows / 8 = 7644, 751 x 2 audio rows, int4);
* whole blocks at the 22B widths (d 4096 / 2048, 32 heads): mxfp8 with 1024
  video tokens, and config 3 exactly (int8 g64, 3456 video + 126 audio tokens).

The GPU always computes every row and feature.  Where the numpy oracle would
take minutes, the comparison uses a sample of rows and output features spread
over every 256 x 256 output tile (first and last row / feature of each tile
included), each sampled dot product over the full K.  Repeat calls must give
the same bits (the K-split schedules add partials in a fixed order).

Bars, as the path states them: max-abs-rel <= 2e-2 and cosine >= 0.9995; in
addition fewer than 2 % of the compared elements may differ from the oracle at
all (the only freedom in a linear is the fp32 accumulation order).
"""

import numpy as np
import pytest

from helpers import from_dev_bf16, ulp_diff_bf16
from oracle import block as ob
from oracle import quant as oq
from oracle import ref_ops as ro
from oracle.bf16 import f32_to_bf16_bits, rbf16

pytestmark = pytest.mark.gpu

MAX_ABS_REL = 2e-2
COS_MIN = 0.9995
MAX_DIFFERING = 0.02

# quantization name -> (mode, bits, short mxfp8 conversion allowed)
QUANT = {"mxfp8": ("mxfp8", 8, True), "mxfp8_general": ("mxfp8", 8, False), "int8": ("affine", 8, True),
         "int4": ("affine", 4, True)}


def _torch():
    import torch

    return torch


def _gen(seed):
    torch = _torch()
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


def _randn(gen, shape, std, dtype=None):
    torch = _torch()
    return (torch.randn(*shape, generator=gen, device="cuda") * std).to(dtype or torch.bfloat16)


def _bits(t):
    torch = _torch()
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _linear(N, K, quant, seed, pretransposed=False):
    """Random bf16 weight ~N(0, 0.02) and bias ~N(0, 0.01), quantized on the
    GPU (the quantizer is bit-exact against the oracle's)."""
    import ltxq
    from ltxq import _lib

    mode, bits, fast = QUANT[quant]
    gen = _gen(seed)
    w = _randn(gen, (N, K), 0.02)
    b = _randn(gen, (N,), 0.01)
    ql = ltxq.QuantizedLinear.from_linear(w, b, mode=mode, bits=bits, pretransposed=pretransposed)
    del w
    if not fast:
        ql.fast_path = False
    if mode == "mxfp8":
        assert ql.data_flags() == (_lib.QW_MXFP8_FINITE if fast else 0)
    return ql


def _host_packed(ql, rows=None) -> dict:
    """The packed arrays of ``ql`` (standard layout) restricted to output
    features ``rows``, on the host in the oracle's dict form."""
    torch = _torch()
    idx = None if rows is None else torch.as_tensor(np.asarray(rows), device=ql.weight.device)

    def sel(t):
        return (t if idx is None else t[idx]).contiguous()

    w = sel(ql.weight.view(torch.int32)).cpu().numpy().view(np.uint32)
    if ql.mode == "affine":
        return {"weight": w, "scales": _bits(sel(ql.scales)), "biases": _bits(sel(ql.biases)),
                "group_size": ql.group_size, "bits": ql.bits, "mode": "affine"}
    return {"weight": w, "scales": sel(ql.scales).cpu().numpy(), "group_size": 32, "bits": 8, "mode": "mxfp8"}


def _spread(n, count, tile=256):
    """About ``count`` indices of [0, n) spread evenly, plus the first and the
    last index of every ``tile``-wide block."""
    if n <= count:
        return np.arange(n)
    idx = np.concatenate([np.linspace(0, n - 1, count).round().astype(np.int64), np.arange(0, n, tile),
                          np.minimum(np.arange(tile - 1, n + tile - 1, tile), n - 1)])
    return np.unique(idx)


def _assert_parity(got, ref, what):
    mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
    differing = float((ulp_diff_bf16(got, ref) > 0).mean())
    print(f"{what}: max_abs_rel={mar:.2e} cos={cos:.7f} differing={differing:.3%}")
    assert mar <= MAX_ABS_REL and cos >= COS_MIN, f"{what}: max_abs_rel={mar:.3e} cos={cos:.6f}"
    assert differing < MAX_DIFFERING, f"{what}: {differing:.2%} of the elements differ"


def _run_linear(M, K, N, quant, epi, seed, rows=320, cols=1024, pretransposed=False):
    """One GEMM on the GPU at the full shape, compared on a row x feature
    sample (or fully when the sample covers everything)."""
    torch = _torch()
    ql = _linear(N, K, quant, seed, pretransposed)
    gen = _gen(seed + 1)
    x = _randn(gen, (M, K), 1.0)
    kw, res, gate = {}, None, None
    if epi == "gelu":
        kw["gelu"] = True
    elif epi in ("gated", "gate_then_add"):
        res = _randn(gen, (M, N), 1.0)
        gate = _randn(gen, (1, N), 0.5, torch.float32)
        kw.update(residual=res, gate=gate, gate_then_add=(epi == "gate_then_add"))
    out = ql(x, **kw)
    r, c = _spread(M, rows), _spread(N, cols)
    rt, ct = torch.as_tensor(r, device="cuda"), torch.as_tensor(c, device="cuda")
    xs = from_dev_bf16(x[rt])
    bias = from_dev_bf16(ql.bias[ct])
    if pretransposed:
        qT = {"weight": ql.weight.view(torch.int32).cpu().numpy().view(np.uint32), "scales": ql.scales.cpu().numpy(),
              "group_size": 32, "bits": 8, "mode": "mxfp8"}
        ref = ro.linear_pretransposed(xs, oq.dequantize(qT, N)[:, c], bias)
    else:
        ref = ro.linear(xs, oq.dequantize(_host_packed(ql, c), K), bias)
    if epi == "gelu":
        ref = ro.gelu_approx(ref)
    elif epi == "gated":
        ref = ro.gated_add(from_dev_bf16(res[rt][:, ct]), ref, gate[0, ct].cpu().numpy())
    elif epi == "gate_then_add":
        ref = ro.gate_then_add(from_dev_bf16(res[rt][:, ct]), ref, gate[0, ct].cpu().numpy())
    got = from_dev_bf16(out[rt][:, ct])
    _assert_parity(got, ref, f"{M}x{K}->{N} {quant} {epi}{' pretransposed' if pretransposed else ''}")
    again = ql(x, **kw)
    assert torch.equal(out.view(torch.int16), again.view(torch.int16)), "repeat call changed bits"


# ---------------------------------------------------------------- config 1 exactly


@pytest.mark.parametrize("norm", ["layer", "rms"])
def test_config1_exact_shape(cuda, norm):
    """BASELINE config 1 at its stated shape and distributions (seed 0, numpy
    PCG64, fp32 draws rounded to bf16), every output element compared."""
    torch = _torch()
    import ltxq
    from helpers import to_dev, to_dev_bf16

    g = np.random.Generator(np.random.PCG64(0))
    x = rbf16(g.standard_normal((1, 1024, 4096), dtype=np.float32))
    shift, scale, gate = (rbf16(g.standard_normal((1, 4096), dtype=np.float32) * np.float32(0.1)) for _ in range(3))
    W = rbf16(g.standard_normal((4096, 4096), dtype=np.float32) * np.float32(0.02))
    b = rbf16(g.standard_normal(4096, dtype=np.float32) * np.float32(0.01))
    q = oq.quantize(W, "affine", 64, 8)
    # the GPU quantizer writes the same packed arrays
    gq = ltxq.QuantizedLinear.from_linear(to_dev_bf16(W), to_dev_bf16(b), mode="affine", bits=8, group_size=64)
    torch.cuda.synchronize()
    assert np.array_equal(gq.weight.view(torch.int32).cpu().numpy().view(np.uint32), q["weight"])
    assert np.array_equal(_bits(gq.scales), q["scales"]) and np.array_equal(_bits(gq.biases), q["biases"])
    ql = ltxq.QuantizedLinear(to_dev(q["weight"]), to_dev(q["scales"]), to_dev(q["biases"]), to_dev_bf16(b),
                              group_size=64, bits=8, mode="affine", in_features=4096, out_features=4096)
    xd = to_dev_bf16(x)
    out = ql(xd, residual=xd, gate=to_dev_bf16(gate), adaln=(to_dev_bf16(scale), to_dev_bf16(shift), 1e-6, norm))
    ref = ro.adaln_linear_gated(x[0], scale, shift, gate, oq.dequantize(q, 4096), b, 1e-6, norm, vec_bf16=True)
    _assert_parity(from_dev_bf16(out[0]), ref, f"config 1 ({norm})")


# ---------------------------------------------------------------- config-4 linears at full width

VIDEO_T, RANK8_T, AUDIO_T, TEXT_L = 9216, 1152, 201, 1024

# (name, M, K, N, epilogue): every GEMM shape of one config-4 block
VIDEO_SHAPES = [
    ("ff_in", VIDEO_T, 4096, 16384, "gelu"),
    ("ff_out", VIDEO_T, 16384, 4096, "gated"),
    ("attn1_qkv_gate", VIDEO_T, 4096, 3 * 4096 + 32, "none"),
    ("attn1_out", VIDEO_T, 4096, 4096, "gated"),
    ("attn2_out", VIDEO_T, 4096, 4096, "gate_then_add"),
    ("a2v_q_gate", VIDEO_T, 4096, 2048 + 32, "none"),
    ("v2a_kv", VIDEO_T, 4096, 2 * 2048, "none"),
    ("a2v_out", VIDEO_T, 2048, 4096, "gated"),
]


@pytest.mark.parametrize("name,M,K,N,epi", VIDEO_SHAPES, ids=[s[0] for s in VIDEO_SHAPES])
def test_video_linears_mxfp8_full_width(cuda, name, M, K, N, epi):
    _run_linear(M, K, N, "mxfp8", epi, seed=100 + VIDEO_SHAPES.index((name, M, K, N, epi)))


@pytest.mark.parametrize("quant", ["mxfp8_general", "int8", "int4"])
@pytest.mark.parametrize("name,M,K,N,epi", VIDEO_SHAPES[:2], ids=["ff_in", "ff_out"])
def test_video_ff_linears_every_quant(cuda, quant, name, M, K, N, epi):
    _run_linear(M, K, N, quant, epi, seed=200 + list(QUANT).index(quant))


AUDIO_SHAPES = [
    ("audio_ff_in", AUDIO_T, 2048, 8192, "gelu"),
    ("audio_ff_out", AUDIO_T, 8192, 2048, "gated"),
    ("audio_attn1_out", AUDIO_T, 2048, 2048, "gated"),
    ("audio_attn1_qkv_gate", AUDIO_T, 2048, 3 * 2048 + 32, "none"),
    ("a2v_kv", AUDIO_T, 2048, 2 * 2048, "none"),
    ("audio_attn2_out", AUDIO_T, 2048, 2048, "gate_then_add"),
]


@pytest.mark.parametrize("quant", list(QUANT))
@pytest.mark.parametrize("name,M,K,N,epi", AUDIO_SHAPES, ids=[s[0] for s in AUDIO_SHAPES])
def test_audio_linears_split_k(cuda, quant, name, M, K, N, epi):
    """201 rows: few output tiles, so the K range of most tiles is split over
    clusters and the partials are added in split order."""
    _run_linear(M, K, N, quant, epi, seed=300 + AUDIO_SHAPES.index((name, M, K, N, epi)), rows=M, cols=N)


RANK8_SHAPES = [
    ("ff_in", RANK8_T, 4096, 16384, "gelu"),
    ("ff_out", RANK8_T, 16384, 4096, "gated"),
    ("attn1_out", RANK8_T, 4096, 4096, "gated"),
    ("attn1_qkv_gate", RANK8_T, 4096, 3 * 4096 + 32, "none"),
]


@pytest.mark.parametrize("quant", ["mxfp8", "int8"])
@pytest.mark.parametrize("name,M,K,N,epi", RANK8_SHAPES, ids=[s[0] for s in RANK8_SHAPES])
def test_rank_of_8_linears_hybrid_schedule(cuda, quant, name, M, K, N, epi):
    """The video rows of one rank of 8: the last wave of tiles is split along K
    while the first ones run whole, in one launch."""
    _run_linear(M, K, N, quant, epi, seed=400 + RANK8_SHAPES.index((name, M, K, N, epi)), rows=M, cols=1024)


@pytest.mark.parametrize("name,M,K,N", [("video_text_kv", TEXT_L, 4096, 2 * 4096),
                                        ("audio_text_kv", TEXT_L, 2048, 2 * 2048)])
def test_text_context_linears(cuda, name, M, K, N):
    _run_linear(M, K, N, "mxfp8", "none", seed=500 + K, rows=M, cols=1024)


@pytest.mark.parametrize("M,K,N,epi", [(VIDEO_T, 4096, 16384, "gelu"), (AUDIO_T, 2048, 2048, "gated")])
def test_pretransposed_full_width(cuda, M, K, N, epi):
    """The cache's mxfp8-blocks-pretranspose layout at config-4 widths."""
    _run_linear(M, K, N, "mxfp8", epi, seed=600 + K, pretransposed=True, rows=min(M, 320), cols=1024)


# ---------------------------------------------------------------- configs 2 and 5


def test_config2_ff_sublayer_full_shape(cuda):
    """AdaLN -> project_in (int4 g64, GELU) -> project_out
    -> gated residual at 3456 x 4096 (hidden 16384); the sub-layer is
    row-local, so a row sample is compared over all 4096 outputs."""
    torch = _torch()
    import ltxq

    M, D, H = 3456, 4096, 16384
    w_in, w_out = _linear(H, D, "int4", 700), _linear(D, H, "int4", 701)
    ff = ltxq.FeedForward(w_in, w_out)
    gen = _gen(702)
    x = _randn(gen, (1, M, D), 1.0)
    s, t, gate = (_randn(gen, (1, 1, D), 0.1, torch.float32) for _ in range(3))
    out = ff.sublayer(x, s, t, gate)
    r = _spread(M, 256)
    rt = torch.as_tensor(r, device="cuda")
    xs = from_dev_bf16(x[0, rt])
    f = lambda a: a.cpu().numpy().reshape(-1)  # noqa: E731
    ref = ro.ff_sublayer(xs, f(s), f(t), f(gate), oq.dequantize(_host_packed(w_in), D), from_dev_bf16(w_in.bias),
                         oq.dequantize(_host_packed(w_out), H), from_dev_bf16(w_out.bias))
    _assert_parity(from_dev_bf16(out[0, rt]), ref, "config 2 FF sub-layer")


@pytest.mark.parametrize("name,M,K,N,epi", [("video_ff_in", 7644, 4096, 16384, "gelu"),
                                            ("video_ff_out", 7644, 16384, 4096, "gated"),
                                            ("audio_ff_in", 1502, 2048, 8192, "gelu")])
def test_config5_rank_shapes_int4(cuda, name, M, K, N, epi):
    """Config 5 per rank of 8: (30576 x 2) / 8 video rows, the CFG pair's
    751 x 2 audio rows, int4 g64."""
    _run_linear(M, K, N, "int4", epi, seed=800 + K + N)


# ---------------------------------------------------------------- blocks at 22B width


def _oracle_params(lin, tabs):
    """Oracle parameters of a block from its GPU-quantized parts: each packed
    weight dequantized on the host (the fp32 form, checked against the exact
    one on two weights)."""
    p = {}
    for i, (name, ql) in enumerate(lin.items()):
        q = _host_packed(ql)
        p[f"{name}.weight"] = oq.dequantize_fast(q, ql.in_features)
        if i < 2:
            assert np.array_equal(f32_to_bf16_bits(p[f"{name}.weight"]),
                                  f32_to_bf16_bits(oq.dequantize(q, ql.in_features)))
        p[f"{name}.bias"] = from_dev_bf16(ql.bias)
    for name, t in tabs.items():
        p[name] = t.float().cpu().numpy()
    return p


def _block_case(mode, bits, T, A, L, seed, compute="dequant", attention="sdpa"):
    torch = _torch()
    import ltxq
    from ltxq.block import AUDIO_22B, VIDEO_22B, BasicAVTransformerBlock, TransformerArgs

    gen = _gen(seed)
    lin, tabs = BasicAVTransformerBlock.random_parts(gen, "cuda", mode=mode, bits=bits)
    p = _oracle_params(lin, tabs)
    blk = BasicAVTransformerBlock(lin, tabs, VIDEO_22B, AUDIO_22B).set_compute(compute).set_attention(attention)

    def stream(cfg, t):
        ang = torch.rand(1, cfg.heads, t, cfg.d_head // 2, generator=gen, device="cuda") * 6.28
        cang = torch.rand(1, AUDIO_22B.heads, t, AUDIO_22B.d_head // 2, generator=gen, device="cuda") * 6.28
        return TransformerArgs(
            x=_randn(gen, (1, t, cfg.dim), 1.0), context=_randn(gen, (1, L, cfg.context_dim), 1.0),
            timesteps=_randn(gen, (1, 1, 9, cfg.dim), 0.1, torch.float32),
            positional_embeddings=(torch.cos(ang), torch.sin(ang)),
            cross_positional_embeddings=(torch.cos(cang), torch.sin(cang)),
            cross_scale_shift_timestep=_randn(gen, (1, 1, 4, cfg.dim), 0.1, torch.float32),
            cross_gate_timestep=_randn(gen, (1, 1, 1, cfg.dim), 0.1, torch.float32),
            prompt_timestep=_randn(gen, (1, 1, 2, cfg.dim), 0.1, torch.float32))

    v, a = stream(VIDEO_22B, T), stream(AUDIO_22B, A)

    def host(args):
        f = lambda t_: t_.float().cpu().numpy()  # noqa: E731
        return {"x": from_dev_bf16(args.x[0]), "context": from_dev_bf16(args.context[0]),
                "timesteps": f(args.timesteps[0, 0]), "prompt": f(args.prompt_timestep[0, 0]),
                "cross_ss": f(args.cross_scale_shift_timestep[0, 0]), "cross_gate": f(args.cross_gate_timestep[0, 0]),
                "pe": tuple(f(c[0]) for c in args.positional_embeddings),
                "cross_pe": tuple(f(c[0]) for c in args.cross_positional_embeddings)}

    hv, ha = host(v), host(a)
    ov, oa = blk(v, a)
    got_v, got_a = from_dev_bf16(ov.x[0]), from_dev_bf16(oa.x[0])
    assert ltxq._lib.device_error() == 0
    del blk, lin
    ref_v, ref_a = ob.block(p, hv, ha, heads_v=VIDEO_22B.heads, heads_a=AUDIO_22B.heads)
    for got, ref, what in ((got_v, ref_v, "video"), (got_a, ref_a, "audio")):
        mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
        print(f"block {mode}{bits} {compute} T={T} A={A} {what}: max_abs_rel={mar:.2e} cos={cos:.7f}")
        assert mar <= MAX_ABS_REL and cos >= COS_MIN, f"{what}: max_abs_rel={mar:.3e} cos={cos:.6f}"


def test_block_22b_width_mxfp8(cuda):
    """The config-4 block (d 4096 / 2048, 32 heads of 128 / 64, mxfp8 g32) on
    1024 video tokens, 201 audio tokens and 1024 text tokens."""
    _block_case("mxfp8", 8, 1024, AUDIO_T, TEXT_L, seed=900)


def test_block_config3_exact(cuda):
    """one int8 g64 block, 3456 video tokens, 126 audio
    tokens, 1024 text tokens."""
    _block_case("affine", 8, 3456, 126, TEXT_L, seed=901)
