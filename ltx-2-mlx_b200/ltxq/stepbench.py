"""Timing of a whole denoise step of the 22B model on one GPU.

    python -m ltxq.stepbench [--blocks 48] [--iters 3]

Prints one JSON object with, for batch 1 (no guidance) and batch 2 (the
CFG pair as one pass):

* ``blocks_ms``: the 48-block loop alone (what ``bench.py`` times);
* ``model_ms``: ``LTXAVModel.__call__`` (preprocess with the AdaLN MLPs,
  the blocks, the output heads), so ``model_ms - blocks_ms`` is the cost of
  the stages around the block loop;

and the fused ``denoise_update`` kernel on the video latent (1 x 9216 x 128,
CFG: three bf16 reads and one bf16 write per element) against the measured
HBM copy bandwidth.  Each figure is the device time per step from CUDA
events around replays of one captured CUDA graph (synchronized on both
sides, after warm-up replays).  Weights are random (mxfp8 g32), inputs
synthetic; the 19 GB of packed weights stream per step, far above the L2.
"""

from __future__ import annotations

import argparse
import json
import os

import torch


def _time_replays(graph, iters: int, warmup: int = 1) -> float:
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def _hbm_peak() -> float | None:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("--blocks", type=int, default=48)
    ap.add_argument("--video-tokens", type=int, default=9216)
    ap.add_argument("--audio-tokens", type=int, default=201)
    ap.add_argument("--text-tokens", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args(argv)

    from .block import AUDIO_22B, VIDEO_22B
    from .denoise import denoise_update
    from .graph import StepGraph
    from .model import LTXAVModel, Modality

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(2026)
    model = LTXAVModel.random(gen, dev, n_blocks=args.blocks)
    T, A, L = args.video_tokens, args.audio_tokens, args.text_tokens

    def rnd(*shape, std=1.0, dtype=torch.float32):
        return (torch.randn(*shape, generator=gen, device=dev) * std).to(dtype)

    def rope(b, heads, t, d):
        ang = torch.rand(b, heads, t, d // 2, generator=gen, device=dev) * 6.28
        return torch.cos(ang), torch.sin(ang)

    out = {"workload": "22b_denoise_step_mxfp8g32", "blocks": args.blocks, "video_tokens": T, "audio_tokens": A,
           "text_tokens": L, "iters": args.iters, "timing": "CUDA events around CUDA-graph replays"}
    for b in (1, 2):
        sig = torch.full((b,), 0.909375, dtype=torch.float32, device=dev)
        vm = Modality(rnd(b, T, 128, dtype=torch.bfloat16), sig, rnd(b, L, VIDEO_22B.context_dim, dtype=torch.bfloat16),
                      rope(b, VIDEO_22B.heads, T, VIDEO_22B.d_head), rope(b, AUDIO_22B.heads, T, AUDIO_22B.d_head),
                      sigma=sig)
        am = Modality(rnd(b, A, 128, dtype=torch.bfloat16), sig, rnd(b, L, AUDIO_22B.context_dim, dtype=torch.bfloat16),
                      rope(b, AUDIO_22B.heads, A, AUDIO_22B.d_head), rope(b, AUDIO_22B.heads, A, AUDIO_22B.d_head),
                      sigma=sig)
        g_model = StepGraph(model, vm, am)
        model_ms = _time_replays(g_model, args.iters)
        g_model.release()
        va, aa = model._prepare(model.video, vm, am), model._prepare(model.audio, am, vm)

        def blocks(va, aa):
            for blk in model.blocks:
                va, aa = blk(va, aa)
            return va.x, aa.x

        g_blocks = StepGraph(blocks, va, aa)
        blocks_ms = _time_replays(g_blocks, args.iters)
        g_blocks.release()
        out[f"batch{b}"] = {"model_ms": model_ms, "blocks_ms": blocks_ms, "around_blocks_ms": model_ms - blocks_ms}
        del va, aa, vm, am
        torch.cuda.empty_cache()

    x, vc, vu = (rnd(1, T, 128, dtype=torch.bfloat16) for _ in range(3))
    res = torch.empty_like(x)

    def update(x, vc, vu):
        return denoise_update(x, vc, 0.909375, 0.725, v_uncond=vu, cfg_scale=3.0, out=res)

    reps = 50
    g_upd = StepGraph(lambda *a: [update(*a) for _ in range(reps)][-1], x, vc, vu)
    us = _time_replays(g_upd, 5) * 1e3 / reps
    g_upd.release()
    nbytes = 4 * x.numel() * 2
    peak = _hbm_peak()
    out["denoise_update"] = {"shape": [1, T, 128], "us": us, "bytes": nbytes, "gbs": nbytes / (us * 1e-6) / 1e9,
                             "hbm_peak_gbs": peak,
                             "frac_of_measured_hbm": None if peak is None else nbytes / (us * 1e-6) / 1e9 / peak,
                             "note": "9.4 MB per launch (L2-resident between launches): bound by launch latency"}
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    main()
