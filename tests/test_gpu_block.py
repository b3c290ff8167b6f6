"""GPU parity of the full audio-video block (transformer.py:389-674) against
the numpy oracle block, at reduced widths (the structure, sub-layer order,
rounding points and every epilogue/prologue form are those of the 22B block).
"""

import numpy as np
import pytest

from helpers import block_params, from_dev_bf16, gpu_block, normal_bf16, normal_f32, rng, rope_np, to_dev_bf16
from oracle import block as ob
from oracle import ref_ops as ro

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,bits", [("affine", 8), ("mxfp8", 8)])
def test_av_block_matches_oracle(cuda, mode, bits):
    import torch

    import ltxq
    from ltxq.block import StreamConfig, TransformerArgs

    video = StreamConfig(1024, 8, 128, 1024)
    audio = StreamConfig(512, 8, 64, 512)
    T, A, L = 160, 72, 48
    p_oracle, quant, tables = block_params(video, audio, mode, bits)
    g = rng(31)
    blk = gpu_block(quant, tables, video, audio, mode)

    def stream(cfg, tokens, ctx_tokens, heads_cross):
        d = {
            "x": normal_bf16(g, (tokens, cfg.dim)),
            "context": normal_bf16(g, (ctx_tokens, cfg.context_dim)),
            "timesteps": normal_f32(g, (9, cfg.dim), 0.1),
            "prompt": normal_f32(g, (2, cfg.dim), 0.1),
            "cross_ss": normal_f32(g, (4, cfg.dim), 0.1),
            "cross_gate": normal_f32(g, (1, cfg.dim), 0.1),
            "pe": rope_np(g, cfg.heads, tokens, cfg.d_head),
            "cross_pe": rope_np(g, heads_cross, tokens, audio.d_head),
        }
        return d

    vs = stream(video, T, L, audio.heads)
    as_ = stream(audio, A, L, audio.heads)
    ref_v, ref_a = ob.block(p_oracle, vs, as_, heads_v=video.heads, heads_a=audio.heads)

    def args(d):
        f = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        pe = tuple(f(c)[None] for c in d["pe"])
        cpe = tuple(f(c)[None] for c in d["cross_pe"])
        return TransformerArgs(x=to_dev_bf16(d["x"])[None], context=to_dev_bf16(d["context"])[None],
                               timesteps=f(d["timesteps"])[None, None], positional_embeddings=pe,
                               cross_positional_embeddings=cpe,
                               cross_scale_shift_timestep=f(d["cross_ss"])[None, None],
                               cross_gate_timestep=f(d["cross_gate"])[None, None],
                               prompt_timestep=f(d["prompt"])[None, None])

    ov, oa = blk(args(vs), args(as_))
    got_v, got_a = from_dev_bf16(ov.x[0]), from_dev_bf16(oa.x[0])
    for got, ref, what in ((got_v, ref_v, "video"), (got_a, ref_a, "audio")):
        mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
        assert mar <= 2e-2 and cos >= 0.9995, f"{what}: max_abs_rel={mar:.3e} cos={cos:.6f}"
    assert ltxq._lib.device_error() == 0


def test_step_graph_replay_matches_eager(cuda):
    """A two-block step captured by ltxq.graph.StepGraph and replayed on new
    inputs (copied into the captured input tensors) gives the eager step's
    bits."""
    import torch

    import ltxq
    from ltxq.block import BasicAVTransformerBlock, StreamConfig, TransformerArgs
    from ltxq.graph import StepGraph

    video = StreamConfig(1024, 8, 128, 1024)
    audio = StreamConfig(512, 8, 64, 512)
    T, A, L = 96, 40, 32
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    blocks = [BasicAVTransformerBlock.random(gen, "cuda", mode="mxfp8", video=video, audio=audio) for _ in range(2)]

    def rnd(*shape, std=1.0, dtype=torch.float32):
        return (torch.randn(*shape, generator=gen, device="cuda") * std).to(dtype)

    def rope(heads, t, d):
        ang = torch.rand(1, heads, t, d // 2, generator=gen, device="cuda") * 6.28
        return torch.cos(ang), torch.sin(ang)

    def args(cfg, t):
        return TransformerArgs(x=rnd(1, t, cfg.dim, dtype=torch.bfloat16),
                               context=rnd(1, L, cfg.context_dim, dtype=torch.bfloat16),
                               timesteps=rnd(1, 1, 9, cfg.dim, std=0.1), positional_embeddings=rope(cfg.heads, t, cfg.d_head),
                               cross_positional_embeddings=rope(audio.heads, t, audio.d_head),
                               cross_scale_shift_timestep=rnd(1, 1, 4, cfg.dim, std=0.1),
                               cross_gate_timestep=rnd(1, 1, 1, cfg.dim, std=0.1),
                               prompt_timestep=rnd(1, 1, 2, cfg.dim, std=0.1))

    v, a = args(video, T), args(audio, A)

    def step(v, a):
        for b in blocks:
            v, a = b(v, a)
        return v, a

    g = StepGraph(step, v, a)
    assert g.launches > 0
    new_v = rnd(1, T, video.dim, dtype=torch.bfloat16)
    new_a = rnd(1, A, audio.dim, dtype=torch.bfloat16)
    v.x.copy_(new_v)
    a.x.copy_(new_a)
    gv, ga = g.replay()
    gv_x, ga_x = gv.x.clone(), ga.x.clone()
    ev, ea = step(v, a)
    assert torch.equal(gv_x.view(torch.int16), ev.x.view(torch.int16))
    assert torch.equal(ga_x.view(torch.int16), ea.x.view(torch.int16))
    g.release()
    assert ltxq._lib.device_error() == 0


def test_av_block_batch2_matches_oracle_per_entry(cuda):
    """Batch 2 (the cond/uncond pair of classifier-free guidance): per-batch
    AdaLN vectors, RoPE tables and contexts; each batch entry equals the
    oracle block run on that entry alone."""
    import torch

    import ltxq
    from ltxq.block import StreamConfig, TransformerArgs

    video = StreamConfig(1024, 8, 128, 1024)
    audio = StreamConfig(512, 8, 64, 512)
    T, A, L = 96, 40, 32
    mode, bits = "mxfp8", 8
    p_oracle, quant, tables = block_params(video, audio, mode, bits, seed=33)
    g = rng(34)
    blk = gpu_block(quant, tables, video, audio, mode)

    def stream(cfg, tokens):
        return {
            "x": normal_bf16(g, (tokens, cfg.dim)),
            "context": normal_bf16(g, (L, cfg.context_dim)),
            "timesteps": normal_f32(g, (9, cfg.dim), 0.1),
            "prompt": normal_f32(g, (2, cfg.dim), 0.1),
            "cross_ss": normal_f32(g, (4, cfg.dim), 0.1),
            "cross_gate": normal_f32(g, (1, cfg.dim), 0.1),
            "pe": rope_np(g, cfg.heads, tokens, cfg.d_head),
            "cross_pe": rope_np(g, audio.heads, tokens, audio.d_head),
        }

    entries = [(stream(video, T), stream(audio, A)) for _ in range(2)]

    def args(ds):
        f = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
        st = lambda key: torch.stack([f(d[key]) for d in ds])  # noqa: E731
        pe = tuple(torch.stack([f(d["pe"][i]) for d in ds]) for i in range(2))
        cpe = tuple(torch.stack([f(d["cross_pe"][i]) for d in ds]) for i in range(2))
        return TransformerArgs(x=torch.stack([to_dev_bf16(d["x"]) for d in ds]),
                               context=torch.stack([to_dev_bf16(d["context"]) for d in ds]),
                               timesteps=st("timesteps")[:, None], positional_embeddings=pe,
                               cross_positional_embeddings=cpe, cross_scale_shift_timestep=st("cross_ss")[:, None],
                               cross_gate_timestep=st("cross_gate")[:, None], prompt_timestep=st("prompt")[:, None])

    ov, oa = blk(args([e[0] for e in entries]), args([e[1] for e in entries]))
    for bi, (vs, as_) in enumerate(entries):
        ref_v, ref_a = ob.block(p_oracle, vs, as_, heads_v=video.heads, heads_a=audio.heads)
        for got, ref, what in ((from_dev_bf16(ov.x[bi]), ref_v, "video"), (from_dev_bf16(oa.x[bi]), ref_a, "audio")):
            mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
            assert mar <= 2e-2 and cos >= 0.9995, f"entry {bi} {what}: max_abs_rel={mar:.3e} cos={cos:.6f}"
    assert ltxq._lib.device_error() == 0


def test_split_key_merge_matches_full_attention(cuda):
    """The log-sum-exp the video->audio split-key attention merges with (from
    the memory-efficient SDPA, natural log, padded query dimension) gives
    the full attention: two key halves merged vs SDPA over all keys."""
    import math

    import torch
    import torch.nn.functional as F

    from ltxq.block import merge_attention_partials

    g = torch.Generator(device="cuda")
    g.manual_seed(70)
    B, H, Lq, Lk, D = 1, 32, 201, 2304, 64
    q = torch.randn(B, H, Lq, D, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, H, Lk, D, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, H, Lk, D, generator=g, device="cuda").to(torch.bfloat16)
    sc = 1.0 / math.sqrt(D)
    outs, lses = [], []
    for part in range(2):
        ks, vs = k[:, :, part * Lk // 2:(part + 1) * Lk // 2], v[:, :, part * Lk // 2:(part + 1) * Lk // 2]
        o, lse = torch.ops.aten._scaled_dot_product_efficient_attention(q, ks, vs, None, True, 0.0, False,
                                                                        scale=sc)[:2]
        outs.append(o.float())
        lses.append(lse[..., :Lq].float())
    merged = merge_attention_partials(torch.stack(outs), torch.stack(lses))
    full = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=sc)
    err = (merged - full).abs().max().item() / full.abs().max().item()
    assert err < 1e-2, err
