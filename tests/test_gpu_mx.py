"""GPU tests of the native block-scaled fp8 path (LTXQ_COMPUTE_MX2 / MX1).

* the activation splitter (ltxq_mx_split) against oracle/mx.py bit for bit:
  codes of each term and the scale bytes in the MMA's atom layout, including
  groups of zeros, tiny and huge values and the 448-saturation boundary;
* the block-scaled GEMM (tcgen05.mma kind::mxf8f6f4 on the cache's E4M3 codes
  and E8M0 scales) against the oracle's MX linear layer (the reference
  composition on the split activations: only the fp32 summation order
  differs) and, with the path's stated tolerance, against the reference
  composition on the bf16 activations, at the config-4 shapes; ragged token
  and feature tiles; every epilogue; repeat calls bit-identical;
* the one-term form against the oracle's one-term layer;
* GEMMs too small for the native path run the dequantizing kernels.
"""

import ctypes

import numpy as np
import pytest

from helpers import from_dev_bf16, normal_bf16, rng, to_dev_bf16, ulp_diff_bf16
from oracle import mx as omx
from oracle import quant as oq
from oracle import ref_ops as ro

pytestmark = pytest.mark.gpu

MAX_ABS_REL = 2e-2
COS_MIN = 0.9995


def _torch():
    import torch

    return torch


def _split_gpu(x_np, terms):
    torch = _torch()
    from ltxq import _lib

    lib = _lib.load()
    M, K = x_np.shape
    codes, sfb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    row_tiles = lib.ltxq_mx_split_sizes(M, K, ctypes.byref(codes), ctypes.byref(sfb))
    assert row_tiles == (M + 127) // 128 + 1
    bufs = [torch.full((n,), 0xAB, dtype=torch.uint8, device="cuda") for n in (codes.value, codes.value, sfb.value,
                                                                                sfb.value)]
    x = to_dev_bf16(x_np)
    _lib.check(lib.ltxq_mx_split(x.data_ptr(), M, K, terms, bufs[0].data_ptr(), bufs[1].data_ptr(),
                                 bufs[2].data_ptr(), bufs[3].data_ptr(), None), "mx_split")
    torch.cuda.synchronize()
    return [b.cpu().numpy() for b in bufs], row_tiles


@pytest.mark.parametrize("terms", [2, 1])
def test_mx_split_bit_exact(cuda, terms):
    g = rng(81)
    M, K = 300, 1024
    x = normal_bf16(g, (M, K))
    x[0, :32] = 0.0                                   # all-zero group
    x[1, :32] *= np.float32(1e-30)                    # tiny group (fp32-subnormal scaled values)
    x[2, 32:64] *= np.float32(1e30)                   # huge group
    x[3, :32] = ro.rbf16(np.float32(1.75) * np.float32(2.0) ** np.arange(-16, 16, dtype=np.float32))
    x[4, :32] = np.float32(448.0)                     # exactly E4M3's largest value
    x[5, 64:96] = np.float32(-0.0)
    x[6, :32] = ro.rbf16(np.linspace(-3, 3, 32).astype(np.float32))
    x = ro.rbf16(x)
    (hi, lo, sf_hi, sf_lo), row_tiles = _split_gpu(x, terms)
    ref = omx.mx_split(x, terms)
    np.testing.assert_array_equal(hi.reshape(M, K), ref[0][0])
    np.testing.assert_array_equal(sf_hi.reshape(-1, row_tiles, 512), omx.scale_atoms(ref[0][1], row_tiles))
    if terms == 2:
        np.testing.assert_array_equal(lo.reshape(M, K), ref[1][0])
        np.testing.assert_array_equal(sf_lo.reshape(-1, row_tiles, 512), omx.scale_atoms(ref[1][1], row_tiles))


def _spread(n, count, tile):
    if n <= count:
        return np.arange(n)
    return np.unique(np.concatenate([np.linspace(0, n - 1, count).round().astype(np.int64), np.arange(0, n, tile),
                                     np.minimum(np.arange(tile - 1, n + tile - 1, tile), n - 1)]))


def _mx_case(M, K, N, epi, compute, seed, rows=320, cols=1024):
    """One GEMM at full shape through QuantizedLinear with the given compute
    mode; returns (got, mx-oracle ref, reference-composition ref) on a row x
    feature sample, and the number of library launches of the call."""
    torch = _torch()
    import ltxq
    from ltxq import _lib

    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    w = (torch.randn(N, K, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=gen, device="cuda") * 0.01).to(torch.bfloat16)
    ql = ltxq.QuantizedLinear.from_linear(w, b, mode="mxfp8").set_compute(compute)
    del w
    x = (torch.randn(M, K, generator=gen, device="cuda")).to(torch.bfloat16)
    kw = {}
    res = gate = None
    if epi == "gelu":
        kw["gelu"] = True
    elif epi in ("gated", "gate_then_add"):
        res = torch.randn(M, N, generator=gen, device="cuda").to(torch.bfloat16)
        gate = torch.randn(1, N, generator=gen, device="cuda") * 0.5
        kw.update(residual=res, gate=gate, gate_then_add=(epi == "gate_then_add"))
    ql.data_flags()  # the one-time scan of the packed data is a launch of its own
    n0 = _lib.launch_count()
    out = ql(x, **kw)
    launches = _lib.launch_count() - n0
    again = ql(x, **kw)
    assert torch.equal(out.view(torch.int16), again.view(torch.int16)), "repeat call changed bits"
    r, c = _spread(M, rows, 192), _spread(N, cols, 256)
    rt, ct = torch.as_tensor(r, device="cuda"), torch.as_tensor(c, device="cuda")
    wq = ql.weight.view(torch.int32)[ct].cpu().numpy().view(np.uint32)
    q = {"weight": wq, "scales": ql.scales[ct].cpu().numpy(), "group_size": 32, "bits": 8, "mode": "mxfp8"}
    deq = oq.dequantize(q, K)
    xs = from_dev_bf16(x[rt])
    bias = from_dev_bf16(ql.bias[ct])
    terms = 2 if compute == "mx2" else 1
    refs = [omx.mx_linear(xs, deq, bias, terms), ro.linear(xs, deq, bias)]
    for i, y in enumerate(refs):
        if epi == "gelu":
            y = ro.gelu_approx(y)
        elif epi == "gated":
            y = ro.gated_add(from_dev_bf16(res[rt][:, ct]), y, gate[0, ct].cpu().numpy())
        elif epi == "gate_then_add":
            y = ro.gate_then_add(from_dev_bf16(res[rt][:, ct]), y, gate[0, ct].cpu().numpy())
        refs[i] = y
    return from_dev_bf16(out[rt][:, ct]), refs[0], refs[1], launches


MX_SHAPES = [
    ("ff_in", 9216, 4096, 16384, "gelu"),
    ("ff_out", 3456, 16384, 4096, "gate_then_add"),
    ("rank8_out", 1152, 4096, 4096, "gated"),
    ("ragged_qkv", 1000, 2048, 3 * 4096 + 32, "none"),
]


@pytest.mark.parametrize("name,M,K,N,epi", MX_SHAPES, ids=[s[0] for s in MX_SHAPES])
def test_mx2_gemm_matches_oracle(cuda, name, M, K, N, epi):
    got, ref_mx, ref, launches = _mx_case(M, K, N, epi, "mx2", seed=40 + [s[0] for s in MX_SHAPES].index(name))
    assert launches == 2, f"expected the split + block-scaled GEMM launches, got {launches}"
    differing = float((ulp_diff_bf16(got, ref_mx) > 0).mean())
    mar, cos = ro.max_abs_rel(got, ref_mx), ro.cosine(got, ref_mx)
    print(f"mx2 {name} vs MX oracle: max_abs_rel={mar:.2e} cos={cos:.7f} differing={differing:.3%}")
    assert differing < 0.02 and mar <= MAX_ABS_REL and cos >= COS_MIN
    mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
    print(f"mx2 {name} vs reference composition: max_abs_rel={mar:.2e} cos={cos:.7f}")
    assert mar <= MAX_ABS_REL and cos >= COS_MIN


def test_mx1_gemm_matches_one_term_oracle(cuda):
    """The one-term form computes exactly the oracle's one-term layer (to fp32
    summation order); against the reference composition it is coarser (its
    error is reported, not held to the path's tolerance)."""
    got, ref_mx, ref, launches = _mx_case(2304, 4096, 8192, "none", "mx1", seed=7)
    assert launches == 2
    differing = float((ulp_diff_bf16(got, ref_mx) > 0).mean())
    assert differing < 0.02 and ro.cosine(got, ref_mx) >= COS_MIN, differing
    print(f"mx1 vs reference composition: max_abs_rel={ro.max_abs_rel(got, ref):.2e} cos={ro.cosine(got, ref):.6f}")


def test_small_gemms_keep_the_dequantizing_kernels(cuda):
    """201 audio rows give fewer output tiles than clusters: the MX request
    falls back to the dequantizing K-split kernels, with the same result as
    the default mode."""
    torch = _torch()
    import ltxq

    g = rng(91)
    W = normal_bf16(g, (2048, 2048), 0.02)
    x = to_dev_bf16(normal_bf16(g, (201, 2048)))
    ql = ltxq.QuantizedLinear.from_linear(to_dev_bf16(W), mode="mxfp8")
    a = ql(x)
    b = ql.set_compute("mx2")(x)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_block_with_mx2_matches_oracle(cuda):
    """A 22B-width mxfp8 block (1024 video, 201 audio, 1024 text tokens) with
    every GEMM set to mx2 (those with enough tiles run block-scaled) against
    the oracle block."""
    from test_gpu_shapes import _block_case

    _block_case("mxfp8", 8, 1024, 201, 1024, seed=900, compute="mx2")
