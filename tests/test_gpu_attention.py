"""GPU tests of the native attention core (``ltxq_attention``): softmax(Q K^T
* scale) V per head against the oracle's ``sdpa`` (numpy, fp32 softmax,
bf16 output; the reference's mx.fast.scaled_dot_product_attention).

Shapes: ragged query and key counts (partial 128-row tiles, the masked last
key stage, a second query tile with no rows), batch 2 with rows that must not
leak across batches, strided column slices of a fused projection output,
head_dim 64 and 128, scores spread over a wide range (the running maximum
moves and O is rescaled), one query / one key, and the block's shapes: video
self-attention 9216 x 9216 x 32 heads (sampled rows and heads), the
audio->video (9216 queries, 201 keys) and video->audio (201 queries, 9216
keys) cross attentions.
"""

import math

import numpy as np
import pytest

from helpers import from_dev_bf16, normal_bf16, rng, to_dev_bf16
from oracle import block as ob
from oracle import ref_ops as ro

pytestmark = pytest.mark.gpu

MAX_ABS_REL = 2e-2
COS_MIN = 0.9995


def _check(got, ref, what):
    mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
    print(f"{what}: max_abs_rel={mar:.2e} cos={cos:.7f}")
    assert mar <= MAX_ABS_REL and cos >= COS_MIN, (what, mar, cos)


def _run(q, k, v, heads, scale=None):
    from ltxq import kernels as K

    return K.attention(q, k, v, heads, scale)


CASES = [
    # (B, Tq, Tk, heads, D, spread)
    (1, 300, 300, 4, 128, 1.0),
    (2, 201, 1000, 4, 64, 1.0),
    (1, 129, 77, 2, 128, 1.0),
    (2, 257, 384, 2, 64, 4.0),   # wide score range: the running maximum moves
    (1, 1, 1, 1, 64, 1.0),
    (1, 1000, 129, 3, 128, 3.0),
]


@pytest.mark.parametrize("B,Tq,Tk,heads,D,spread", CASES)
def test_attention_matches_oracle(cuda, B, Tq, Tk, heads, D, spread):
    import torch

    g = rng(Tq * 7 + Tk + D)
    W = heads * D
    q = normal_bf16(g, (B, Tq, W), spread)
    k = normal_bf16(g, (B, Tk, W), spread)
    # v as a column slice of a wider fused projection row (row stride 3 W + 32)
    fused = normal_bf16(g, (B, Tk, 3 * W + 32))
    v = fused[:, :, 2 * W:3 * W]
    vd = to_dev_bf16(fused).view(B, Tk, 3 * W + 32)[:, :, 2 * W:3 * W]
    out = _run(to_dev_bf16(q).view(B, Tq, W), to_dev_bf16(k).view(B, Tk, W), vd, heads)
    torch.cuda.synchronize()
    got = from_dev_bf16(out).reshape(B, Tq, W)
    for b in range(B):
        _check(got[b], ob.sdpa(q[b], k[b], v[b], heads), f"B{b} {Tq}x{Tk} h{heads} d{D}")


def test_attention_repeat_calls_identical(cuda):
    import torch

    g = rng(3)
    q = to_dev_bf16(normal_bf16(g, (1, 640, 512))).view(1, 640, 512)
    k = to_dev_bf16(normal_bf16(g, (1, 700, 512))).view(1, 700, 512)
    v = to_dev_bf16(normal_bf16(g, (1, 700, 512))).view(1, 700, 512)
    a, b = _run(q, k, v, 4), _run(q, k, v, 4)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def _block_shape(Tq, Tk, heads, D, rows, head_ids, seed):
    import torch

    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    W = heads * D
    q = torch.randn(1, Tq, W, generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.randn(1, Tk, W, generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn(1, Tk, W, generator=gen, device="cuda").to(torch.bfloat16)
    out = _run(q, k, v, heads)
    torch.cuda.synchronize()
    r = np.unique(np.concatenate([np.linspace(0, Tq - 1, rows).round().astype(np.int64), [0, Tq - 1]]))
    for h in head_ids:
        cols = slice(h * D, (h + 1) * D)
        qs = from_dev_bf16(q[0, r, cols])
        ks, vs = from_dev_bf16(k[0, :, cols]), from_dev_bf16(v[0, :, cols])
        ref = ob.sdpa(qs, ks, vs, 1)
        _check(from_dev_bf16(out[0, r, cols]), ref, f"{Tq}x{Tk} head {h}")


def test_video_self_attention_shape(cuda):
    _block_shape(9216, 9216, 32, 128, 384, (0, 17, 31), 11)


def test_cross_attention_shapes(cuda):
    _block_shape(9216, 201, 32, 64, 256, (0, 31), 12)   # audio -> video: video queries, audio keys
    _block_shape(201, 9216, 32, 64, 201, (5,), 13)      # video -> audio: audio queries, video keys


def test_attention_against_torch_sdpa(cuda):
    """A second reference: torch's fp32 SDPA on the same bf16 inputs."""
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    B, T, heads, D = 2, 512, 8, 128
    q, k, v = (torch.randn(B, T, heads * D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    out = _run(q, k, v, heads)
    hf = lambda t: t.float().view(B, T, heads, D).transpose(1, 2)
    ref = torch.nn.functional.scaled_dot_product_attention(hf(q), hf(k), hf(v), scale=1.0 / math.sqrt(D))
    ref = ref.transpose(1, 2).reshape(B, T, heads * D).to(torch.bfloat16)
    _check(from_dev_bf16(out).reshape(-1), from_dev_bf16(ref).reshape(-1), "vs torch fp32 sdpa")


def test_attention_rejects_bad_arguments(cuda):
    import torch

    from ltxq import kernels as K

    x = torch.zeros(1, 8, 96, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        K.attention(x, x, x, 1)  # head_dim 96


def test_block_with_native_attention_matches_oracle(cuda):
    """A 22B-width mxfp8 block (1024 video, 201 audio, 1024 text tokens) with
    every attention core on the native kernel, against the oracle block."""
    from test_gpu_shapes import _block_case

    _block_case("mxfp8", 8, 1024, 201, 1024, seed=901, attention="native")
