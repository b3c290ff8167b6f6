"""GPU tests of the producers that write the block-scaled GEMMs' MX input
form directly (no separate split pass):

* the AdaLN pass (``ltxq_adaln_modulate_mx``, every row-kernel shape, every
  norm, fp32 / bf16 and broadcast / per-batch vectors) and the per-head gate
  (``ltxq_head_gate_mx``): the same codes and scale bytes as
  ``ltxq_mx_split`` of their bf16 results, which in turn match the oracle's
  split; with ``out`` given, the bf16 result alongside;
* the block-scaled GEMM from MX terms: the same bits as the GEMM from bf16
  activations; with MX output (bias + GELU), the same terms as splitting its
  bf16 result;
* the composed C entries (``ltxq_adaln_qlinear``, ``ltxq_feed_forward``)
  over block-scaled weights, which now fuse the split into their producers:
  the same bits as the separate calls, in fewer launches.

The scale bytes of rows past M (the spare row tile) are not written by the
fused producers; the GEMM reads them only for accumulator columns it never
stores, so the comparisons cover the rows < M.
"""

import ctypes

import numpy as np
import pytest

from helpers import from_dev_bf16, normal_bf16, rng, to_dev_bf16
from oracle import mx as omx

pytestmark = pytest.mark.gpu


def _valid_atoms(M, K):
    row_tiles = (M + 127) // 128 + 1
    return omx.scale_atoms(np.full((M, K // 32), -126, np.int32), row_tiles).reshape(-1) != 0


def _assert_same_terms(a, b, what):
    """Two MXActivations hold the same codes and the same scale bytes of
    rows < M."""
    assert (a.M, a.K, a.terms) == (b.M, b.K, b.terms)
    valid = _valid_atoms(a.M, a.K)
    ta, tb = a.tensors(), b.tensors()
    for i, name in enumerate(("hi", "lo", "sf_hi", "sf_lo")):
        if ta[i] is None:
            assert tb[i] is None
            continue
        x, y = ta[i].cpu().numpy(), tb[i].cpu().numpy()
        if name.startswith("sf"):
            x, y = x[valid], y[valid]
        diff = np.flatnonzero(x.reshape(-1) != y.reshape(-1))
        assert diff.size == 0, f"{what}: {name} differs at {diff.size} bytes (first {diff[:5]})"


def _vec(torch, g, shape, dtype, std=0.2):
    return torch.from_numpy((g.standard_normal(shape) * std).astype(np.float32)).to("cuda").to(dtype)


ADALN_CASES = [
    # (batch, tokens, C, norm, vec dtype, per-batch vectors)
    (1, 300, 4096, "rms", "f32", False),     # 2 warps per row, ragged last row tile
    (2, 500, 2048, "rms", "bf16", True),     # 1 warp per row, 8 chunks per lane
    (1, 77, 1024, "layer", "f32", True),     # 4 chunks per lane
    (1, 5, 128, "none", "bf16", False),      # one 128-channel tile
    (1, 1024, 4096, "none", "f32", False),   # the text-context modulation
]


@pytest.mark.parametrize("terms", [2, 1])
@pytest.mark.parametrize("B,T,C,norm,vdt,per_batch", ADALN_CASES)
def test_adaln_mx_output_matches_split(cuda, B, T, C, norm, vdt, per_batch, terms):
    import torch

    from ltxq import kernels as K

    g = rng(1000 + C + T)
    x = to_dev_bf16(normal_bf16(g, (B, T, C))).view(B, T, C)
    dt = torch.float32 if vdt == "f32" else torch.bfloat16
    vshape = (B, 1, C) if per_batch else (1, 1, C)
    sc, sh = _vec(torch, g, vshape, dt), _vec(torch, g, vshape, dt)
    ref_bf16 = K.adaln_modulate(x, sc, sh, 1e-6, norm)
    fused = K.adaln_modulate(x, sc, sh, 1e-6, norm, mx_terms=terms)
    split = K.MXActivation.split(ref_bf16, terms)
    torch.cuda.synchronize()
    _assert_same_terms(fused, split, f"adaln {norm} C={C}")
    # the split of the bf16 result is the oracle's split (codes; first rows)
    rows = min(B * T, 64)
    xo = from_dev_bf16(ref_bf16.reshape(-1, C)[:rows])
    ref_terms = omx.mx_split(xo, terms)
    np.testing.assert_array_equal(fused.tensors()[0][:rows].cpu().numpy(), ref_terms[0][0])


def test_adaln_mx_with_bf16_output_too(cuda):
    """out and out_mx both given: the bf16 rows alongside the terms."""
    import torch

    from ltxq import _lib
    from ltxq import kernels as K

    g = rng(5)
    M, C = 257, 2048
    x = to_dev_bf16(normal_bf16(g, (M, C)))
    sc, sh = _vec(torch, g, (1, C), torch.float32), _vec(torch, g, (1, C), torch.float32)
    keep = []
    pro = K.prologue(_lib.NORM_RMS, 1e-6, sc, sh, (M,), C, keep)
    act = K.MXActivation((M,), C, 2, x.device)
    st = act.struct()
    out = torch.empty_like(x)
    _lib.check(_lib.load().ltxq_adaln_modulate_mx(x.data_ptr(), M, C, ctypes.byref(pro), out.data_ptr(),
                                                  ctypes.byref(st), K._stream()), "adaln_modulate_mx")
    ref = K.adaln_modulate(x, sc, sh, 1e-6)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    _assert_same_terms(act, K.MXActivation.split(ref, 2), "adaln out + out_mx")


@pytest.mark.parametrize("M,heads,d", [(1000, 32, 128), (201, 32, 64), (3, 1, 128)])
def test_head_gate_mx_output_matches_split(cuda, M, heads, d):
    import torch

    from ltxq import kernels as K

    g = rng(77 + M)
    o = to_dev_bf16(normal_bf16(g, (M, heads * d)))
    gl = to_dev_bf16(normal_bf16(g, (M, heads), 2.0))
    ref = K.head_gate(o, gl, heads)
    for terms in (2, 1):
        fused = K.head_gate(o, gl, heads, mx_terms=terms)
        torch.cuda.synchronize()
        _assert_same_terms(fused, K.MXActivation.split(ref, terms), f"head_gate terms={terms}")


def _mx_linear(torch, N, K_, seed, compute="mx2"):
    import ltxq

    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    w = (torch.randn(N, K_, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=gen, device="cuda") * 0.01).to(torch.bfloat16)
    return ltxq.QuantizedLinear.from_linear(w, b, mode="mxfp8").set_compute(compute), gen


@pytest.mark.parametrize("compute", ["mx2", "mx1"])
def test_gemm_from_terms_matches_bf16_input(cuda, compute):
    import torch

    from ltxq import _lib
    from ltxq import kernels as K

    M, K_, N = 1000, 4096, 4096
    ql, gen = _mx_linear(torch, N, K_, 11, compute)
    terms = ql.mx_terms(M)
    assert terms == (2 if compute == "mx2" else 1)
    x = torch.randn(M, K_, generator=gen, device="cuda").to(torch.bfloat16)
    res = torch.randn(M, N, generator=gen, device="cuda").to(torch.bfloat16)
    gate = torch.randn(1, N, generator=gen, device="cuda") * 0.5
    act = K.MXActivation.split(x, terms)
    ql.data_flags()
    for kw in ({}, {"gelu": True}, {"residual": res, "gate": gate}, {"residual": res, "gate": gate,
                                                                     "gate_then_add": True}):
        a = ql(x, **kw)
        n0 = _lib.launch_count()
        b = ql(act, **kw)
        assert _lib.launch_count() - n0 == 1
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), kw


def test_gemm_mx_output_matches_split(cuda):
    """project_in with GELU writing project_out's input terms: the same terms
    as splitting its bf16 output (ragged rows)."""
    import torch

    from ltxq import kernels as K

    M, K_, N = 1000, 4096, 16384
    ql, gen = _mx_linear(torch, N, K_, 12)
    x = torch.randn(M, K_, generator=gen, device="cuda").to(torch.bfloat16)
    act = K.MXActivation.split(x, 2)
    for gelu in (True, False):
        y = ql(act, gelu=gelu)
        for terms in (2, 1):
            h = ql(act, gelu=gelu, mx_out=terms)
            torch.cuda.synchronize()
            _assert_same_terms(h, K.MXActivation.split(y, terms), f"gemm mx_out gelu={gelu} terms={terms}")
    with pytest.raises(ValueError):
        ql(act, residual=y, gate=torch.ones(1, N, device="cuda"), mx_out=2)


def test_composed_entries_fuse_the_split(cuda):
    """ltxq_adaln_qlinear and ltxq_feed_forward over block-scaled weights:
    the same bits as the separate calls, with the split folded into the
    producers (2 and 3 launches)."""
    import torch

    import ltxq
    from ltxq import _lib
    from ltxq import kernels as K

    M, D, H = 1152, 4096, 16384
    ql_in, gen = _mx_linear(torch, H, D, 21)
    ql_out, _ = _mx_linear(torch, D, H, 22)
    x = torch.randn(1, M, D, generator=gen, device="cuda").to(torch.bfloat16)
    sc = torch.randn(1, 1, D, generator=gen, device="cuda") * 0.1
    sh = torch.randn(1, 1, D, generator=gen, device="cuda") * 0.1
    gate = torch.randn(1, 1, D, generator=gen, device="cuda") * 0.5
    ql_in.data_flags(), ql_out.data_flags()

    a_bf16 = K.adaln_modulate(x, sc, sh, 1e-6)
    sep = ql_in(a_bf16, gelu=True)
    n0 = _lib.launch_count()
    fused = ql_in(x, gelu=True, adaln=(sc, sh, 1e-6))
    assert _lib.launch_count() - n0 == 2
    assert torch.equal(sep.view(torch.int16), fused.view(torch.int16))

    ff = ltxq.FeedForward(ql_in, ql_out)
    ref = ql_out(ql_in(a_bf16, gelu=True), residual=x, gate=gate)
    n0 = _lib.launch_count()
    got = ff.sublayer(x, sc, sh, gate)
    assert _lib.launch_count() - n0 == 3
    assert torch.equal(ref.view(torch.int16), got.view(torch.int16))
    # the plain FF (no prologue): split + two GEMMs
    ref2 = ql_out(ql_in(x, gelu=True))
    assert torch.equal(ref2.view(torch.int16), ff(x).view(torch.int16))
