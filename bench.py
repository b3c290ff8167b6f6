"""Benchmark of the quantized DiT-block hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload step|ff]

Default workload "step" (benchmark config 4, the configuration the
headline metric is quoted on): one 22B-shaped denoise step -- 48 random-init audio-video
blocks, every block linear quantized mxfp8 (group 32, E8M0 scales) on the
GPU from bf16 weights ~N(0, 0.02), 1024x576x121 frames -> 9216 video tokens
(d 4096, 32 heads x 128), 201 audio tokens (d 2048, 32 x 64), 1024 text tokens
per stream, batch 1; AdaLN vectors ~N(0, 0.1) fp32 (the sigma schedule only
changes their values, not the cost); RoPE tables from synthetic positions.
Synthetic, seeded data (the reference uses no dataset).

``value`` is ms per denoise step (lower is better), max over ranks, inputs
resident in HBM; the 19 GB of packed weights streamed every step are far
larger than the L2, so no flush is needed.  Under torchrun (N > 1) the video
tokens are row-sharded over the ranks (9216 / N rows each), weights are
replicated, audio and text streams are replicated, and the K/V of video
self-attention and of video->audio cross-attention are all-gathered with NCCL
(strong scaling: the job is fixed).  ``e2e`` is the same metric through the
public block API with this step's latent rows copied from pinned host memory
and the results copied back inside the timed region.  ``roofline`` describes
the dominant kernel, the video FF project_in GEMM (mxfp8 CTA-pair GEMM,
9216/N x 4096 -> 16384 with the GELU epilogue), timed with CUDA events around
its launches inside the timed steps.

Workload "ff": the video FF sub-layer, int4 g64, 3456 tokens,
reported in quantized-GEMM TFLOP/s.

``--impl reference`` times the reference's composition on the host CPU (the
numpy restatement in oracle/, all host threads) on a bounded sample of the
same workload and prints the same metric.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ltx-2-mlx_b200"))

METRIC = "ms/denoise step (22B shape, 8xB200) + quantized-GEMM TFLOP/s vs peak, 1/2/4/8 GPU"

# ---- config 4: 22B-shaped denoise step
STEP_T, STEP_A, STEP_L, STEP_BLOCKS = 9216, 201, 1024, 48
VD, AD = 4096, 2048


def step_linear_flops(t_video: int, t_audio: int, t_text: int) -> float:
    """2*M*N*K over every block linear (which rows each projection reads:
    transformer.py:447-668, attention.py:560-602)."""
    V, A, L = t_video, t_audio, t_text
    f = 0.0
    f += 2 * V * VD * (3 * VD + 32) + 2 * V * VD * VD                  # attn1 qkv+gate, out
    f += 2 * V * VD * (VD + 32) + 2 * L * VD * 2 * VD + 2 * V * VD * VD  # attn2 q+gate, kv (text), out
    f += 2 * A * AD * (3 * AD + 32) + 2 * A * AD * AD                  # audio_attn1
    f += 2 * A * AD * (AD + 32) + 2 * L * AD * 2 * AD + 2 * A * AD * AD  # audio_attn2
    f += 2 * V * VD * (AD + 32) + 2 * A * AD * 2 * AD + 2 * V * AD * VD  # a2v: q(video) kv(audio) out
    f += 2 * A * AD * (AD + 32) + 2 * V * VD * 2 * AD + 2 * A * AD * AD  # v2a: q(audio) kv(video) out
    f += 2 * V * VD * 4 * VD * 2 + 2 * A * AD * 4 * AD * 2              # feed-forwards
    return f


# ---- config 2: video FF sub-layer
FF_T, FF_D, FF_H = 3456, 4096, 16384
FF_FLOPS = 2.0 * FF_T * FF_D * FF_H * 2

# ---- config 1: one fused AdaLN + quantized linear + gated residual
CFG1_M, CFG1_D = 1024, 4096
CFG1_FLOPS = 2.0 * CFG1_M * CFG1_D * CFG1_D

# ---- step-shaped workloads: --workload -> (blocks, quant, video tokens, audio tokens, batch, workload name)
STEP_PRESETS = {
    "config3": (1, "int8", 3456, 126, 1, "config3_av_block_int8g64_3456video_126audio"),
    "config5": (48, "int4", 30576, 751, 2, "config5_22b_denoise_step_int4g64_batch2_30576video_751audio"),
}


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def _traffic(kernel_key: str):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get(kernel_key)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle-reason sampling while the benchmark runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0"))


# ============================================================================ CPU legs (oracle)


class CpuBlock:
    """One config-4 block (d 4096 / 2048, 32 heads, every linear mxfp8 g32) on
    the host cores through the oracle's numpy restatement of the reference
    composition, at the full token counts: 9216 video, 201 audio and 1024 text
    rows.  The unit of work is one of the block's seven sub-layers, attention
    included; each call dequantizes that sub-layer's packed weights once (the
    reference's quantized matmul works from the packed cache on every call)
    and runs the sub-layer on all of its rows.  A block is the sum of its
    sub-layers; a step is 48 blocks."""

    SUBLAYERS = {  # sub-layer -> the attention / FF modules whose weights it reads
        "video_self_attention": ("attn1",),
        "video_text_cross_attention": ("attn2",),
        "audio_self_attention": ("audio_attn1",),
        "audio_text_cross_attention": ("audio_attn2",),
        "audio_video_cross_attention": ("audio_to_video_attn", "video_to_audio_attn"),
        "video_feed_forward": ("ff",),
        "audio_feed_forward": ("audio_ff",),
    }

    def __init__(self, video_tokens: int = STEP_T, audio_tokens: int = STEP_A, quant: str = "mxfp8", seed: int = 0):
        import numpy as np

        from ltxq.block import AUDIO_22B, VIDEO_22B, linear_specs, table_specs
        from oracle.bf16 import f32_to_bf16_bits, rbf16

        self.video_tokens, self.audio_tokens, self.quant = video_tokens, audio_tokens, quant
        g = np.random.default_rng(seed)
        self.q = {}
        for name, (n, k) in linear_specs().items():
            # packed arrays drawn directly (mxfp8: finite E4M3 codes of either
            # sign, E8M0 scales around 2^-9; affine: random codes, scales and
            # biases): the timed work does not depend on the values
            if quant == "mxfp8":
                codes = (g.integers(0, 0x7F, size=(n, k), dtype=np.uint8)
                         | (g.integers(0, 2, size=(n, k), dtype=np.uint8) << 7))
                qq = {"mode": "mxfp8", "group_size": 32, "bits": 8,
                      "weight": codes.view(np.uint32).reshape(n, k // 4),
                      "scales": g.integers(112, 120, size=(n, k // 32), dtype=np.uint8)}
            else:
                bits = 8 if quant == "int8" else 4
                words = g.integers(0, 2 ** 32, size=(n, k * bits // 32), dtype=np.uint64).astype(np.uint32)
                gp = lambda std: f32_to_bf16_bits(g.standard_normal((n, k // 64), dtype=np.float32) * std)  # noqa: E731
                qq = {"mode": "affine", "group_size": 64, "bits": bits, "weight": words, "scales": gp(1e-3),
                      "biases": gp(0.05)}
            self.q[name] = (qq, rbf16(g.standard_normal(n, dtype=np.float32) * np.float32(0.01)), k)
        self.tabs = {k: (g.standard_normal(s, dtype=np.float32) * np.float32(0.1)
                         + np.float32(1.0 if k.endswith("norm.weight") else 0.0)) for k, s in table_specs().items()}

        def stream(cfg, t):
            ang = g.uniform(0, 6.28, (cfg.heads, t, cfg.d_head // 2)).astype(np.float32)
            cang = g.uniform(0, 6.28, (AUDIO_22B.heads, t, AUDIO_22B.d_head // 2)).astype(np.float32)
            return {"x": rbf16(g.standard_normal((t, cfg.dim), dtype=np.float32)),
                    "context": rbf16(g.standard_normal((STEP_L, cfg.context_dim), dtype=np.float32)),
                    "timesteps": (g.standard_normal((9, cfg.dim)) * 0.1).astype(np.float32),
                    "prompt": (g.standard_normal((2, cfg.dim)) * 0.1).astype(np.float32),
                    "cross_ss": (g.standard_normal((4, cfg.dim)) * 0.1).astype(np.float32),
                    "cross_gate": (g.standard_normal((1, cfg.dim)) * 0.1).astype(np.float32),
                    "pe": (np.cos(ang), np.sin(ang)), "cross_pe": (np.cos(cang), np.sin(cang))}

        self.vs = stream(VIDEO_22B, video_tokens)
        self.as_ = stream(AUDIO_22B, audio_tokens)

    def _weights(self, modules):
        from oracle import quant as oq

        p = dict(self.tabs)
        for name, (qq, b, k) in self.q.items():
            if name.split(".")[0] in modules:
                p[f"{name}.weight"] = oq.dequantize_fast(qq, k)
                p[f"{name}.bias"] = b
        return p

    def run(self, sub: str) -> float:
        """Seconds of one sub-layer (weight dequantization included)."""
        from oracle import block as ob
        from oracle import ref_ops as ro

        vs, as_ = self.vs, self.as_
        vx, ax = vs["x"], as_["x"]
        t0 = time.perf_counter()
        p = self._weights(self.SUBLAYERS[sub])
        if sub in ("video_self_attention", "audio_self_attention"):
            s, x, name, table = ((vs, vx, "attn1", "scale_shift_table") if sub.startswith("video")
                                 else (as_, ax, "audio_attn1", "audio_scale_shift_table"))
            sh, sc, g = ob.ada(p[table], s["timesteps"], 0, 3)
            ro.gated_add(x, ob.attention(p, name, ro.adaln(x, sc, sh), pe=s["pe"]), g)
        elif sub in ("video_text_cross_attention", "audio_text_cross_attention"):
            s, x, name, table, prompt = ((vs, vx, "attn2", "scale_shift_table", "prompt_scale_shift_table")
                                         if sub.startswith("video") else
                                         (as_, ax, "audio_attn2", "audio_scale_shift_table",
                                          "audio_prompt_scale_shift_table"))
            sh_q, sc_q, g = ob.ada(p[table], s["timesteps"], 6, 9)
            kv = ob.ada(p[prompt], s["prompt"], 0, 2)
            enc = ro.modulate(s["context"], kv[1], kv[0])
            ro.gate_then_add(x, ob.attention(p, name, ro.adaln(x, sc_q, sh_q), context=enc), g)
        elif sub == "audio_video_cross_attention":
            vn, an = ro.rms_norm(vx), ro.rms_norm(ax)
            ta, tv = p["scale_shift_table_a2v_ca_audio"], p["scale_shift_table_a2v_ca_video"]
            a_sc_a2v, a_sh_a2v, a_sc_v2a, a_sh_v2a = ob.ada(ta, as_["cross_ss"], 0, 4)
            v_sc_a2v, v_sh_a2v, v_sc_v2a, v_sh_v2a = ob.ada(tv, vs["cross_ss"], 0, 4)
            out = ob.attention(p, "audio_to_video_attn", ro.modulate(vn, v_sc_a2v, v_sh_a2v),
                               context=ro.modulate(an, a_sc_a2v, a_sh_a2v), pe=vs["cross_pe"], k_pe=as_["cross_pe"])
            ro.gated_add(vx, out, tv[4] + vs["cross_gate"][0])
            out = ob.attention(p, "video_to_audio_attn", ro.modulate(an, a_sc_v2a, a_sh_v2a),
                               context=ro.modulate(vn, v_sc_v2a, v_sh_v2a), pe=as_["cross_pe"], k_pe=vs["cross_pe"])
            ro.gated_add(ax, out, ta[4] + as_["cross_gate"][0])
        else:
            s, x, table, base = ((vs, vx, "scale_shift_table", "ff") if sub.startswith("video")
                                 else (as_, ax, "audio_scale_shift_table", "audio_ff"))
            sh, sc, g = ob.ada(p[table], s["timesteps"], 3, 6)
            ro.ff_sublayer(x, sc, sh, g, p[f"{base}.project_in.proj.weight"], p[f"{base}.project_in.proj.bias"],
                           p[f"{base}.project_out.weight"], p[f"{base}.project_out.bias"])
        return time.perf_counter() - t0


def _cpu_threads() -> int:
    """Threads of the CPU legs: the cores this process may use (oracle/_par.py)."""
    from oracle._par import usable_cpus

    return usable_cpus()


def _limit_cpu_threads():
    """Context that sizes the BLAS thread pools to the usable cores."""
    try:
        from threadpoolctl import threadpool_limits

        return threadpool_limits(limits=_cpu_threads())
    except ImportError:  # pragma: no cover - threadpoolctl is in the image
        import contextlib

        return contextlib.nullcontext()


def _cpu_block_rotation(blk: "CpuBlock", n_runs: int, warmup: int = 0) -> dict:
    """Runs the block's sub-layers in turn, ``warmup`` untimed then ``n_runs``
    timed (at least one of each), and returns each sub-layer's mean seconds."""
    subs = list(CpuBlock.SUBLAYERS)
    for i in range(warmup):
        blk.run(subs[i % len(subs)])
    times: dict = {s: [] for s in subs}
    for i in range(max(n_runs, len(subs))):
        s = subs[i % len(subs)]
        times[s].append(blk.run(s))
        print(f"[cpu] {s}: {times[s][-1]:.2f} s on {_cpu_threads()} threads", file=sys.stderr, flush=True)
    return {s: sum(v) / len(v) for s, v in times.items()}


def _cpu_block_line(per_sub: dict, blk: "CpuBlock", blocks: int = STEP_BLOCKS) -> tuple:
    """(ms per step of ``blocks`` blocks, the cpu_baseline description) from
    measured sub-layer seconds."""
    block_s = sum(per_sub.values())
    threads = _cpu_threads()
    extra = f"extrapolated x{blocks} blocks per step" if blocks > 1 else "not extrapolated"
    desc = (f"measured: one full block ({blk.quant}; {blk.video_tokens} video, {blk.audio_tokens} audio, {STEP_L} "
            f"text rows; attention included; weights dequantized once per sub-layer call) = {block_s:.2f} s, as "
            f"the sum of its 7 sub-layers timed separately at full size; {extra}. oracle/ numpy restatement of the "
            f"reference composition (BLAS on {threads} threads, elementwise ops on one)")
    return block_s * blocks * 1e3, desc


def _cpu_config1(norm: str = "layer"):
    """BASELINE config 1 on the host at its full shape (not extrapolated):
    seconds, FLOPs."""
    import numpy as np

    from oracle import quant as oq
    from oracle import ref_ops as ro
    from oracle.bf16 import rbf16

    g = np.random.default_rng(0)
    x = rbf16(g.standard_normal((1024, 4096), dtype=np.float32))
    sc, sh, gt = (rbf16(g.standard_normal((1, 4096), dtype=np.float32) * np.float32(0.1)) for _ in range(3))
    w = rbf16(g.standard_normal((4096, 4096), dtype=np.float32) * np.float32(0.02))
    b = rbf16(g.standard_normal(4096, dtype=np.float32) * np.float32(0.01))
    q = oq.quantize(w, "affine", 64, 8)
    t0 = time.perf_counter()
    ro.adaln_linear_gated(x, sc, sh, gt, oq.dequantize_fast(q, 4096), b, 1e-6, norm, vec_bf16=True)
    return time.perf_counter() - t0, CFG1_FLOPS


def _cpu_ff_sample(sample: int = FF_T, seed: int = 1):
    """The config-2 FF sub-layer on ``sample`` of its rows (all 3456 by
    default: not extrapolated): seconds, FLOPs."""
    import numpy as np

    from oracle import quant as oq
    from oracle import ref_ops as ro
    from oracle.bf16 import rbf16

    g = np.random.default_rng(seed)
    x = rbf16(g.standard_normal((1, sample, FF_D)).astype(np.float32))
    w_in = rbf16((g.standard_normal((FF_H, FF_D)) * 0.02).astype(np.float32))
    w_out = rbf16((g.standard_normal((FF_D, FF_H)) * 0.02).astype(np.float32))
    b_in = rbf16((g.standard_normal(FF_H) * 0.01).astype(np.float32))
    b_out = rbf16((g.standard_normal(FF_D) * 0.01).astype(np.float32))
    v = (g.standard_normal((3, 1, 1, FF_D)) * 0.1).astype(np.float32)
    qi = oq.quantize(w_in, "affine", 64, 4)
    qo = oq.quantize(w_out, "affine", 64, 4)
    t0 = time.perf_counter()
    wi = oq.dequantize_fast(qi, FF_D)
    wo = oq.dequantize_fast(qo, FF_H)
    ro.ff_sublayer(x, v[0], v[1], v[2], wi, b_in, wo, b_out)
    return time.perf_counter() - t0, 2.0 * sample * FF_D * FF_H * 2


def cpu_baseline(workload: str):
    """Bounded CPU measurement for the cpu_baseline field of the GPU line."""
    with _limit_cpu_threads():
        return _cpu_baseline(workload)


def _cpu_baseline(workload: str):
    threads = _cpu_threads()
    if workload in ("step", "config3"):
        blk = CpuBlock() if workload == "step" else CpuBlock(3456, 126, "int8")
        blocks = STEP_BLOCKS if workload == "step" else 1
        ms, desc = _cpu_block_line(_cpu_block_rotation(blk, 7), blk, blocks)
        return {"value": ms, "unit": "ms/step" if blocks > 1 else "ms/block", "cores": threads, "kind": "port",
                "sample": desc}
    if workload == "config5":
        return None  # hours per step on the host cores; the config-4 line carries the CPU figure
    if workload == "config1":
        sec, flops = _cpu_config1()
        return {"value": flops / sec / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": f"the whole config-1 call (1024 x 4096 -> 4096, LayerNorm prologue, gated residual) in "
                          f"{sec:.3f} s, not extrapolated"}
    sec, flops = _cpu_ff_sample()
    return {"value": flops / sec / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"the whole config-2 FF sub-layer ({FF_T} tokens, int4 g64) in {sec:.2f} s, not extrapolated"}


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return
    with _limit_cpu_threads():
        _run_reference(args, world)


def _run_reference(args, world):
    threads = _cpu_threads()
    measured = None
    if args.workload == "config5":
        print(json.dumps({"impl": "reference", "unavailable": "config 5 on the host cores takes hours per step "
                          "(30576 x 2 video rows); the config-4 reference line measures the same composition"}))
        return
    if args.workload in ("step", "config3"):
        blk = CpuBlock() if args.workload == "step" else CpuBlock(3456, 126, "int8")
        blocks = STEP_BLOCKS if args.workload == "step" else 1
        per_sub = _cpu_block_rotation(blk, args.steps, args.warmup)
        value, desc = _cpu_block_line(per_sub, blk, blocks)
        unit, hib, scaling = ("ms/step" if blocks > 1 else "ms/block"), False, "strong"
        cfg = (_step_config(world) if args.workload == "step" else
               _step_config(world, 1, True, "int8", 3456, audio_tokens=126, workload=STEP_PRESETS["config3"][5]))
        ms_step = value
        measured = {"block_s": sum(per_sub.values()), "sublayer_s": per_sub, "blocks_per_step": blocks,
                    "extrapolation": (f"x{blocks} blocks (every block has the same shapes)" if blocks > 1
                                      else "none"),
                    "timed_steps": f"each step times one sub-layer of the block in turn at full size "
                                   f"({max(args.steps, len(CpuBlock.SUBLAYERS))} sub-layer runs)"}
    else:
        run = (lambda i: _cpu_config1()) if args.workload == "config1" else (lambda i: _cpu_ff_sample(FF_T, i))
        for i in range(args.warmup):
            run(100 + i)
        secs, flops = [], 0.0
        for i in range(args.steps):
            s, flops = run(i)
            secs.append(s)
        sec = sum(secs) / len(secs)
        value, unit, hib, scaling = flops / sec / 1e12, "TFLOP/s", True, "weak"
        cfg = _config1_config(world) if args.workload == "config1" else _ff_config(world)
        ms_step = sec * 1e3
        desc = f"the whole {cfg['workload']} workload per step ({sec:.3f} s), not extrapolated"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": hib,
        "scaling": scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if measured is not None:
        line["measured"] = measured
    print(json.dumps(line), flush=True)


# ============================================================================ GPU arm


STEP_QUANT = {  # --quant -> (mode, bits, workload name, description)
    "mxfp8": ("mxfp8", 8, "config4_22b_denoise_step_mxfp8g32", "mxfp8 g32 (E4M3, E8M0 scales), all block linears"),
    "int8": ("affine", 8, "22b_denoise_step_int8g64", "affine int8 g64 (bf16 scales/biases), all block linears"),
    "int4": ("affine", 4, "22b_denoise_step_int4g64", "affine int4 g64 (bf16 scales/biases), all block linears"),
}


def _packed_bytes(quant, n, k):
    """Packed weight + group parameters of an [n, k] linear."""
    if quant == "mxfp8":
        return n * k + n * k // 32
    bits = 8 if quant == "int8" else 4
    return n * k * bits // 8 + 2 * 2 * n * k // 64


_EXCHANGE = {"gather": "video self-attention K/V all-gather", "head_parallel": "video self-attention Q/K/V and "
             "output all-to-all (head-parallel)", "split_keys": "video->audio local keys merged by log-sum-exp"}


def _step_config(world, n_blocks=STEP_BLOCKS, graph=True, quant="mxfp8", video_tokens=STEP_T,
                 self_attention="gather", v2a="gather", audio_tokens=STEP_A, batch=1, workload=None,
                 compute="dequant", attention="sdpa"):
    v2a_text = "video->audio K/V all-gather" if v2a == "gather" else _EXCHANGE[v2a]
    return {"workload": workload or STEP_QUANT[quant][2], "blocks": n_blocks, "video_tokens": video_tokens,
            "execution": "one CUDA graph per step (captured once, replayed)" if graph else "eager launches",
            "audio_tokens": audio_tokens, "text_tokens": STEP_L, "global_batch": batch, "seq_len": video_tokens,
            "quant": STEP_QUANT[quant][3], "compute": compute,
            "attention": ("torch SDPA (cuDNN)" if attention == "sdpa" else "ltxq_attention (native sm_100a)"),
            "parallelism": (f"video rows sharded x{world}, weights replicated, {_EXCHANGE[self_attention]}, "
                            f"{v2a_text} (NCCL)" if world > 1 else "single GPU (no collective)"),
            "l2": "not flushed: 19 GB of packed weights streamed per step >> 126 MB L2"}


def _config1_config(world):
    return {"workload": "config1_adaln_qlinear_gated_int8g64_1024x4096x4096", "tokens": CFG1_M, "d": CFG1_D,
            "quant": "affine int8 g64", "norm": "LayerNorm without affine, eps 1e-6", "global_batch": world,
            "seq_len": CFG1_M, "parallelism": f"replicas{world}",
            "l2": "flushed before every timed step (256 MiB write, outside the events)"}


def _ff_config(world):
    return {"workload": "config2_video_ff_sublayer_int4g64_3456tok", "tokens": FF_T, "d": FF_D, "inner": FF_H,
            "quant": "affine int4 g64", "global_batch": world, "seq_len": FF_T, "parallelism": f"replicas{world}",
            "l2": "flushed before every timed step (256 MiB write, outside the events)"}


def _max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch

    t = torch.tensor([x], device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def exchange_ms(events: list) -> dict:
    """Device ms per kind between each phase-0 and phase-1 event of
    ``RowShard.wait_probe`` records ``(kind, phase, event)``: how long the
    compute stream waited for a side-stream exchange ("wait") or ran one in
    line ("sync")."""
    out = {"wait": 0.0, "sync": 0.0}
    if len(events) % 2:
        raise ValueError("unpaired exchange probe events")
    for (k0, p0, e0), (k1, p1, e1) in zip(events[0::2], events[1::2]):
        if k0 != k1 or (p0, p1) != (0, 1):
            raise ValueError(f"exchange probe events out of order: {(k0, p0)} then {(k1, p1)}")
        out[k0] += e0.elapsed_time(e1)
    return out


def exchange_forms(world: int, self_attention: str = "auto", v2a: str = "auto") -> tuple[str, str]:
    """The row-sharded attention exchanges; "auto" picks by GPU count: at 2 GPUs
    the K/V all-gathers measured fastest (202.6 ms against 221.3 / 205.0), at 8
    the Q/K/V all-to-all and the split-key form (88.5 ms against 93.1)."""
    if self_attention == "auto":
        self_attention = "head_parallel" if world >= 8 else "gather"
    if v2a == "auto":
        v2a = "split_keys" if world >= 8 else "gather"
    return self_attention, v2a


def run_step(args, world, rank, local, dev):
    import torch

    from ltxq import _lib
    from ltxq.block import AUDIO_22B, VIDEO_22B, BasicAVTransformerBlock, RowShard, TransformerArgs
    from ltxq.graph import StepGraph

    T, A, B = args.video_tokens, args.audio_tokens, args.batch
    args.self_attention, args.v2a = exchange_forms(world, args.self_attention, args.v2a)
    if T % world:
        raise SystemExit(f"{T} video tokens do not split over {world} ranks")
    tl = T // world
    shard = RowShard(torch.distributed.group.WORLD if world > 1 else None, world, rank, overlap=not args.no_overlap,
                     self_attention=args.self_attention, v2a=args.v2a)
    gen = torch.Generator(device=dev)
    gen.manual_seed(2026)  # identical on every rank: weights are replicated
    n_blocks = args.blocks
    q_mode, q_bits = STEP_QUANT[args.quant][:2]
    blocks = [BasicAVTransformerBlock.random(gen, dev, mode=q_mode, bits=q_bits).set_compute(args.compute).set_attention(args.attention)
              for _ in range(n_blocks)]
    weight_bytes = sum(b.nbytes() for b in blocks)

    def rnd(*shape, std=1.0, dtype=torch.float32):
        return (torch.randn(*shape, generator=gen, device=dev) * std).to(dtype)

    def rope(heads, t, d):
        # the batch entries (the CFG pair) share token positions; the tables are
        # materialized per entry, as the kernels read them
        ang = torch.rand(1, heads, t, d // 2, generator=gen, device=dev) * 6.2831853
        return tuple(f(ang).expand(B, -1, -1, -1).contiguous() for f in (torch.cos, torch.sin))

    vx_full = rnd(B, T, VD, dtype=torch.bfloat16)
    ax = rnd(B, A, AD, dtype=torch.bfloat16)
    pe_v = rope(VIDEO_22B.heads, T, VIDEO_22B.d_head)
    cpe_v = rope(AUDIO_22B.heads, T, AUDIO_22B.d_head)
    rows = slice(rank * tl, (rank + 1) * tl)
    video = TransformerArgs(
        x=vx_full[:, rows].contiguous(), context=rnd(B, STEP_L, VD, dtype=torch.bfloat16),
        timesteps=rnd(B, 1, 9, VD, std=0.1), positional_embeddings=tuple(c[:, :, rows].contiguous() for c in pe_v),
        cross_positional_embeddings=tuple(c[:, :, rows].contiguous() for c in cpe_v),
        cross_scale_shift_timestep=rnd(B, 1, 4, VD, std=0.1), cross_gate_timestep=rnd(B, 1, 1, VD, std=0.1),
        prompt_timestep=rnd(B, 1, 2, VD, std=0.1))
    audio = TransformerArgs(
        x=ax, context=rnd(B, STEP_L, AD, dtype=torch.bfloat16), timesteps=rnd(B, 1, 9, AD, std=0.1),
        positional_embeddings=rope(AUDIO_22B.heads, A, AUDIO_22B.d_head),
        cross_positional_embeddings=rope(AUDIO_22B.heads, A, AUDIO_22B.d_head),
        cross_scale_shift_timestep=rnd(B, 1, 4, AD, std=0.1), cross_gate_timestep=rnd(B, 1, 1, AD, std=0.1),
        prompt_timestep=rnd(B, 1, 2, AD, std=0.1))
    del vx_full, pe_v, cpe_v
    stream = torch.cuda.current_stream()
    use_graph = not args.eager
    ff_events: list = []

    def probe(tag):
        # external: recorded as event nodes when the step is captured in a graph
        e = torch.cuda.Event(enable_timing=True, external=use_graph)
        e.record(torch.cuda.current_stream())
        ff_events.append(e)

    xchg_events: list = []  # (kind, phase, event) around each exchange the compute stream waits for

    def xprobe(kind, phase):
        e = torch.cuda.Event(enable_timing=True, external=use_graph)
        e.record(torch.cuda.current_stream())
        xchg_events.append((kind, phase, e))

    def xchg_ms() -> dict:
        return exchange_ms(xchg_events)

    def step(v, a):
        for b in blocks:
            v, a = b(v, a, shard)
        return v, a

    clk = ClockSampler(local).start()
    graph = None
    for _ in range(max(args.warmup - (1 if use_graph else 0), 0)):
        step(video, audio)
    torch.cuda.synchronize()
    if use_graph:
        # the last warm-up step runs inside StepGraph (before the capture)
        for b in blocks:
            b.probe = probe
        shard.wait_probe = xprobe if world > 1 else None
        graph = StepGraph(step, video, audio, warmup=1)
        ff_events = ff_events[len(ff_events) - 2 * n_blocks:]  # the captured events
        xchg_events = xchg_events[len(xchg_events) // 2:]  # warm-up pass, then the captured one
        shard.wait_probe = None
        for b in blocks:
            b.probe = None
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    evs, ff_ms, xw = [], [], []
    n_launch0 = _lib.launch_count()
    if args.profile_range:
        torch.cuda.cudart().cudaProfilerStart()
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if use_graph:
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            e1.synchronize()  # read this replay's FF and exchange probes
            ff_ms += [ff_events[i].elapsed_time(ff_events[i + 1]) for i in range(0, len(ff_events), 2)]
            if xchg_events:
                xw.append(xchg_ms())
        else:
            for b in blocks:
                b.probe = probe
            e0.record(stream)
            step(video, audio)
            e1.record(stream)
        evs.append((e0, e1))
    if args.profile_range:
        torch.cuda.cudart().cudaProfilerStop()
    n_launches = (graph.launches * args.steps if use_graph else _lib.launch_count() - n_launch0)
    torch.cuda.synchronize()
    clk.stop()
    for b in blocks:
        b.probe = None
    if world > 1:
        torch.distributed.barrier()
    total_ms = _max_over_ranks(sum(a.elapsed_time(b) for a, b in evs), world, dev)
    ms_step = total_ms / args.steps
    if not use_graph:
        ff_ms = [ff_events[i].elapsed_time(ff_events[i + 1]) for i in range(0, len(ff_events), 2)]
    ff_avg = sum(ff_ms) / len(ff_ms)
    exchange = None
    if world > 1 and use_graph:
        # every rank holds the same probe list (same steps, same block code)
        wait_ms = _max_over_ranks(sum(x["wait"] for x in xw) / max(len(xw), 1), world, dev)
        sync_ms = _max_over_ranks(sum(x["sync"] for x in xw) / max(len(xw), 1), world, dev)
        exchange = {"self_attention": args.self_attention, "v2a": args.v2a,
                    "exposed_wait_ms_per_step": wait_ms, "inline_collective_ms_per_step": sync_ms,
                    "per_block_ms": (wait_ms + sync_ms) / n_blocks,
                    "how": "CUDA events on the compute stream around each join of a side-stream collective "
                           "(time the compute stream waited) and around each collective run in line, in the "
                           "replayed step graph; max over ranks"}

    # ---- e2e through the public block API with host buffers
    vx_host = video.x.cpu().pin_memory()
    ax_host = audio.x.cpu().pin_memory()
    vo_host, ao_host = torch.empty_like(vx_host).pin_memory(), torch.empty_like(ax_host).pin_memory()
    vdev, adev = torch.empty_like(video.x), torch.empty_like(audio.x)
    e2e = []
    for i in range(args.steps + 1):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if use_graph:
            # the graph reads its inputs from the tensors it was captured with
            video.x.copy_(vx_host, non_blocking=True)
            audio.x.copy_(ax_host, non_blocking=True)
            vo, ao = graph.replay()
        else:
            vdev.copy_(vx_host, non_blocking=True)
            adev.copy_(ax_host, non_blocking=True)
            vo, ao = step(video.replace(x=vdev), audio.replace(x=adev))
        vo_host.copy_(vo.x, non_blocking=True)
        ao_host.copy_(ao.x, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        if i:  # the first pass warms the copy path
            e2e.append(e0.elapsed_time(e1))
    e2e_ms = _max_over_ranks(sum(e2e), world, dev) / len(e2e)
    dev_err = _lib.device_error()
    if graph is not None:
        graph.release()  # before the process group that its collectives use goes away

    if rank == 0:
        hbm, tf_burst, tf_sust, peak_kind = _peaks()
        lin_flops = step_linear_flops(B * T, B * A, B * STEP_L) * n_blocks
        ff_flops = 2.0 * B * tl * VD * 4 * VD
        achieved = ff_flops / (ff_avg / 1e3) / 1e12
        h2d = vx_host.numel() * 2 + ax_host.numel() * 2
        line = {
            "metric": METRIC, "value": ms_step, "unit": "ms/block" if n_blocks == 1 else "ms/step",
            "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": _step_config(world, n_blocks, use_graph, args.quant, T, args.self_attention, args.v2a, A, B,
                                   args.workload_name, args.compute, args.attention),
            "quantized_gemm": {"linear_tflop_per_step": lin_flops / 1e12,
                               "step_linear_tflops_per_s": lin_flops / (ms_step / 1e3) / 1e12,
                               "ff_in_gemm_ms": ff_avg, "ff_in_gemm_tflops": achieved,
                               "frac_of_bf16_burst_peak": achieved / tf_burst},
            "roofline": {"bound": "tensor",
                         "kernel": (f"qgemm_pair_kernel<{args.quant}> (video FF project_in, GELU epilogue)"
                                    if args.compute == "dequant" else
                                    f"qgemm_mx_pair_kernel<{2 if args.compute == 'mx2' else 1}> (video FF "
                                    "project_in: MX terms in from the AdaLN pass, GELU, MX terms out)"),
                         "achieved": achieved, "peak": tf_sust, "unit": "TFLOP/s", "frac": achieved / tf_sust,
                         "peak_kind": (f"{peak_kind} bf16 sustained (kernel timed inside a long step)"
                                       if peak_kind == "measured" else "fallback 1400 TFLOP/s sustained"),
                         "traffic": (_traffic(f"qgemm_pair_{args.quant}_ff_in_{B * tl}x16384x4096")
                                     if args.compute == "dequant" else None),
                         "algorithmic_per_launch": {"flops": ff_flops,
                                                    "bytes": B * tl * VD * 2 + _packed_bytes(args.quant, 4 * VD, VD)
                                                    + B * tl * 4 * VD * 2}},
            "e2e": {"value": e2e_ms, "unit": "ms/step", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": h2d,
                    "api": f"ltxq.block.BasicAVTransformerBlock x{n_blocks} (C ABI: ltxq_adaln_modulate, ltxq_qlinear, "
                           "ltxq_qk_norm_rope, ltxq_head_gate"
                           + (", ltxq_adaln_modulate_mx, ltxq_head_gate_mx, ltxq_qlinear_mx)"
                              if args.compute != "dequant" else ")")},
            "gpu_launches": n_launches,
            "weights_gb": weight_bytes / 1e9,
            **({"exchange": exchange} if exchange is not None else {}),
            "clocks": clk.summary(),
            "cpu_baseline": None if (args.no_cpu_baseline or world > 1) else cpu_baseline(args.workload),
            "device_error": dev_err,
        }
        print(json.dumps(line), flush=True)


def run_ff(args, world, rank, local, dev):
    import torch

    import ltxq
    from ltxq import _lib

    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    def randn(*shape, std=1.0, dtype=torch.bfloat16):
        return (torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32) * std).to(dtype)

    x = randn(1, FF_T, FF_D)
    ff = ltxq.FeedForward.from_linear(randn(FF_H, FF_D, std=0.02), randn(FF_H, std=0.01), randn(FF_D, FF_H, std=0.02),
                                      randn(FF_D, std=0.01), mode="affine", group_size=64, bits=4)
    scale, shift, gate = (randn(1, 1, FF_D, std=0.1, dtype=torch.float32) for _ in range(3))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def step_kernels(evs):
        evs[0].record(stream)
        a = ltxq.adaln_modulate(x, scale, shift, 1e-6, "rms")
        evs[1].record(stream)
        h = ff.project_in(a, gelu=True)
        evs[2].record(stream)
        y = ff.project_out(h, residual=x, gate=gate)
        evs[3].record(stream)
        return y

    mk = lambda: [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    clk = ClockSampler(local).start()
    for _ in range(args.warmup):
        flush.fill_(1)
        step_kernels(mk())
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    all_evs = []
    n_launch0 = _lib.launch_count()
    for _ in range(args.steps):
        flush.fill_(1)
        evs = mk()
        step_kernels(evs)
        all_evs.append(evs)
    n_launches = _lib.launch_count() - n_launch0
    torch.cuda.synchronize()
    clk.stop()
    total = _max_over_ranks(sum(e[0].elapsed_time(e[3]) for e in all_evs), world, dev)
    gin = sum(e[1].elapsed_time(e[2]) for e in all_evs) / len(all_evs)
    x_host = x.cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    x_dev = torch.empty_like(x)
    e2e = []
    for i in range(args.steps + 1):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        x_dev.copy_(x_host, non_blocking=True)
        y = ff.sublayer(x_dev, scale, shift, gate)
        out_host.copy_(y, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        if i:
            e2e.append(e0.elapsed_time(e1))
    e2e_total = _max_over_ranks(sum(e2e), world, dev)
    dev_err = _lib.device_error()
    if rank == 0:
        hbm, tf_burst, tf_sust, peak_kind = _peaks()
        achieved = 2.0 * FF_T * FF_D * FF_H / (gin / 1e3) / 1e12
        line = {
            "metric": METRIC, "value": world * FF_FLOPS * args.steps / (total / 1e3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": _ff_config(world),
            "roofline": {"bound": "tensor", "kernel": "qgemm_pair_kernel<affine4> (project_in, GELU epilogue)",
                         "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s", "frac": achieved / tf_burst,
                         "peak_kind": f"{peak_kind} bf16 burst",
                         "traffic": _traffic("qgemm_pair_affine4_ff_in_3456x16384x4096")},
            "e2e": {"value": world * FF_FLOPS * len(e2e) / (e2e_total / 1e3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2,
                    "api": "ltxq.FeedForward.sublayer -> ltxq_feed_forward"},
            "gpu_launches": n_launches, "clocks": clk.summary(),
            "cpu_baseline": None if (args.no_cpu_baseline or world > 1) else cpu_baseline("ff"),
            "device_error": dev_err,
        }
        print(json.dumps(line), flush=True)


def run_config1(args, world, rank, local, dev):
    """out = x + gate * (modulate(LN(x)) @ W^T + b) at
    1024 x 4096 -> 4096, affine int8 g64, bf16 vectors, through the public
    QuantizedLinear call (ltxq_adaln_qlinear: the AdaLN pass, then the GEMM
    with the gated residual in its epilogue).  value = quantized-GEMM TFLOP/s
    of the whole call, summed over the replicas."""
    import torch

    import ltxq
    from ltxq import _lib

    gen = torch.Generator(device=dev)
    gen.manual_seed(4321 + rank)

    def randn(*shape, std=1.0, dtype=torch.bfloat16):
        return (torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32) * std).to(dtype)

    x = randn(1, CFG1_M, CFG1_D)
    scale, shift, gate = (randn(1, CFG1_D, std=0.1) for _ in range(3))
    ql = ltxq.QuantizedLinear.from_linear(randn(CFG1_D, CFG1_D, std=0.02), randn(CFG1_D, std=0.01), mode="affine",
                                          bits=8, group_size=64)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def call():
        return ql(x, residual=x, gate=gate, adaln=(scale, shift, 1e-6, "layer"))

    def split(evs):  # the same two kernels, with an event between them (roofline of the GEMM)
        evs[0].record(stream)
        a = ltxq.adaln_modulate(x, scale, shift, 1e-6, "layer")
        evs[1].record(stream)
        y = ql(a, residual=x, gate=gate)
        evs[2].record(stream)
        return y

    mk = lambda n: [torch.cuda.Event(enable_timing=True) for _ in range(n)]  # noqa: E731
    clk = ClockSampler(local).start()
    for _ in range(args.warmup):
        flush.fill_(1)
        call()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    n_launch0 = _lib.launch_count()
    evs = []
    for _ in range(args.steps):
        flush.fill_(1)
        e = mk(2)
        e[0].record(stream)
        call()
        e[1].record(stream)
        evs.append(e)
    n_launches = _lib.launch_count() - n_launch0
    parts = []
    for _ in range(args.steps):
        flush.fill_(1)
        e = mk(3)
        split(e)
        parts.append(e)
    torch.cuda.synchronize()
    clk.stop()
    total = _max_over_ranks(sum(a.elapsed_time(b) for a, b in evs), world, dev)
    gemm_ms = sum(e[1].elapsed_time(e[2]) for e in parts) / len(parts)
    mod_ms = sum(e[0].elapsed_time(e[1]) for e in parts) / len(parts)
    x_host = x.cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    x_dev = torch.empty_like(x)
    e2e = []
    for i in range(args.steps + 1):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        x_dev.copy_(x_host, non_blocking=True)
        y = ql(x_dev, residual=x_dev, gate=gate, adaln=(scale, shift, 1e-6, "layer"))
        out_host.copy_(y, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        if i:
            e2e.append(e0.elapsed_time(e1))
    e2e_total = _max_over_ranks(sum(e2e), world, dev)
    dev_err = _lib.device_error()
    if rank == 0:
        hbm, tf_burst, tf_sust, peak_kind = _peaks()
        achieved = CFG1_FLOPS / (gemm_ms / 1e3) / 1e12
        w_bytes = _packed_bytes("int8", CFG1_D, CFG1_D) + CFG1_D * 2
        act_bytes = CFG1_M * CFG1_D * 2 * 3  # modulated x in, residual in, out
        line = {
            "metric": METRIC, "value": world * CFG1_FLOPS * args.steps / (total / 1e3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": _config1_config(world),
            "roofline": {"bound": "tensor", "kernel": "qgemm_pair_kernel<affine8> (gated-residual epilogue)",
                         "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s", "frac": achieved / tf_burst,
                         "peak_kind": f"{peak_kind} bf16 burst", "gemm_ms": gemm_ms,
                         "traffic": _traffic("qgemm_pair_affine8_config1_1024x4096x4096"),
                         "algorithmic_per_launch": {"flops": CFG1_FLOPS, "bytes": w_bytes + act_bytes}},
            "adaln_pass": {"ms": mod_ms, "gb_per_s": CFG1_M * CFG1_D * 4 / (mod_ms / 1e3) / 1e9,
                           "frac_of_hbm": CFG1_M * CFG1_D * 4 / (mod_ms / 1e3) / 1e9 / hbm},
            "e2e": {"value": world * CFG1_FLOPS * len(e2e) / (e2e_total / 1e3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2,
                    "api": "ltxq.QuantizedLinear(adaln=...) -> ltxq_adaln_qlinear"},
            "gpu_launches": n_launches, "clocks": clk.summary(),
            "cpu_baseline": None if (args.no_cpu_baseline or world > 1) else cpu_baseline("config1"),
            "device_error": dev_err,
        }
        print(json.dumps(line), flush=True)


def run_ours(args):
    import torch

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    try:
        if args.workload == "ff":
            run_ff(args, world, rank, local, dev)
        elif args.workload == "config1":
            run_config1(args, world, rank, local, dev)
        else:
            run_step(args, world, rank, local, dev)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["step", "config1", "ff", "config3", "config5"], default="step",
                    help="step = config 4 (the headline); config1, ff (config 2), config3 and config5 are the "
                         "other BASELINE configurations")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the timed steps with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    ap.add_argument("--eager", action="store_true",
                    help="launch the step op by op instead of replaying it as one captured CUDA graph")
    ap.add_argument("--no-overlap", action="store_true",
                    help="run the K/V all-gathers on the compute stream instead of a side stream")
    ap.add_argument("--self-attention", choices=["auto", "gather", "head_parallel"], default="auto",
                    help="row-sharded video self-attention: K/V all-gather, or Q/K/V all-to-all over heads; "
                         "auto = head_parallel on 8 or more GPUs (measured faster there), gather below")
    ap.add_argument("--v2a", choices=["auto", "gather", "split_keys"], default="auto",
                    help="row-sharded video->audio attention: K/V all-gather, or local keys merged by log-sum-exp; "
                         "auto = split_keys on 8 or more GPUs, gather below")
    ap.add_argument("--quant", choices=sorted(STEP_QUANT), default="mxfp8",
                    help="block-linear quantization of the step workload (config 4 is mxfp8)")
    ap.add_argument("--video-tokens", type=int, default=STEP_T,
                    help="video tokens of the step (9216 = config 4; fewer only to study per-rank shapes on one GPU)")
    ap.add_argument("--audio-tokens", type=int, default=STEP_A)
    ap.add_argument("--attention", choices=["sdpa", "native"], default="sdpa",
                    help="attention core: torch SDPA (cuDNN) or this library's sm_100a kernel (ltxq_attention)")
    ap.add_argument("--compute", choices=["dequant", "mx2", "mx1"], default="dequant",
                    help="GEMM compute mode (include/ltxq.h LTXQ_COMPUTE_*): dequant = bf16 tensor cores over the "
                         "exactly dequantized weight; mx2 / mx1 = native block-scaled fp8 MMAs on mxfp8 weights with "
                         "the activations in two / one MXFP8 terms")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--blocks", type=int, default=STEP_BLOCKS,
                    help="blocks per step (48 = the 22B model; fewer only for bounded profiler captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    args.workload_name = None
    if args.workload in STEP_PRESETS:
        (args.blocks, args.quant, args.video_tokens, args.audio_tokens, args.batch,
         args.workload_name) = STEP_PRESETS[args.workload]
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
