"""Benchmark of the quantized DiT-block hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload ("config 2"): the video feed-forward
sub-layer of the 22B block -- AdaLN (RMSNorm + modulate) prologue, Linear
4096->16384 with GELU-tanh, Linear 16384->4096, gated residual -- on
3456 tokens x 4096 bf16 (~N(0,1)), weights ~N(0, 0.02) quantized affine int4
group 64 on the GPU, biases ~N(0, 0.01), AdaLN vectors ~N(0, 0.1) fp32.
Synthetic, seeded data (the reference uses no dataset).

A step is one pass of the sub-layer.  ``value`` is whole-job quantized-GEMM
throughput (2*M*N*K of both linears / step time, summed over ranks) with the
inputs resident in HBM; the L2 is flushed (a 256 MiB write) before every
timed step, outside the timed events.  ``e2e`` is the same metric through the
public API (``FeedForward.sublayer`` -> ``ltxq_feed_forward``) with the input
copied from pinned host memory and the output copied back inside the timed
region.  ``roofline`` describes the dominant kernel (the project_in GEMM).
Under torchrun every rank runs its own sub-layer (weak scaling, no
collective on this workload); timings are max over ranks.

``--impl reference`` times the reference composition on the host CPU (the
numpy restatement in oracle/, all host threads) on a bounded sample of the
same workload and prints the same metric.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ltx-2-mlx_b200"))

METRIC = "ms/denoise step (22B shape, 8xB200) + quantized-GEMM TFLOP/s vs peak, 1/2/4/8 GPU"
WORKLOAD = "config2_video_ff_sublayer_int4g64_3456tok"
T, D, H = 3456, 4096, 16384
FLOPS = 2.0 * T * D * H * 2  # both linears (927.7 GFLOP)
BITS, GS = 4, 64


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
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
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
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------- reference arm (CPU)


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return
    import numpy as np

    from oracle import quant as oq
    from oracle import ref_ops as ro
    from oracle.bf16 import rbf16

    cores = os.cpu_count() or 1
    g = np.random.default_rng(0)
    sample = args.cpu_sample
    x = rbf16(g.standard_normal((1, sample, D)).astype(np.float32))
    w_in = rbf16((g.standard_normal((H, D)) * 0.02).astype(np.float32))
    w_out = rbf16((g.standard_normal((D, H)) * 0.02).astype(np.float32))
    b_in = rbf16((g.standard_normal(H) * 0.01).astype(np.float32))
    b_out = rbf16((g.standard_normal(D) * 0.01).astype(np.float32))
    s = (g.standard_normal((1, 1, D)) * 0.1).astype(np.float32)
    t = (g.standard_normal((1, 1, D)) * 0.1).astype(np.float32)
    gate = (g.standard_normal((1, 1, D)) * 0.1).astype(np.float32)
    qi = oq.quantize(w_in, "affine", GS, BITS)
    qo = oq.quantize(w_out, "affine", GS, BITS)

    def step():
        # the reference keeps only the packed weights: the composition
        # dequantizes (inside mx.quantized_matmul) every call
        wi = oq.affine_dequantize_fast(qi["weight"], qi["scales"], qi["biases"], D, GS, BITS)
        wo = oq.affine_dequantize_fast(qo["weight"], qo["scales"], qo["biases"], H, GS, BITS)
        return ro.ff_sublayer(x, s, t, gate, wi, b_in, wo, b_out)

    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    flops = 2.0 * sample * D * H * 2
    val = flops / sec / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3 * (T / sample),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens": T, "d": D, "inner": H, "quant": f"affine int{BITS} g{GS}"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": f"{sample} of {T} tokens per step (oracle/ numpy restatement: dequantize + "
                                   f"fp32 BLAS with bf16 rounding points), ms_per_step scaled by tokens"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample(seconds_budget: float = 20.0):
    """Bounded CPU measurement for the main arm's cpu_baseline field."""
    import numpy as np

    from oracle import quant as oq
    from oracle import ref_ops as ro
    from oracle.bf16 import rbf16

    g = np.random.default_rng(1)
    sample = 256
    x = rbf16(g.standard_normal((1, sample, D)).astype(np.float32))
    w_in = rbf16((g.standard_normal((H, D)) * 0.02).astype(np.float32))
    w_out = rbf16((g.standard_normal((D, H)) * 0.02).astype(np.float32))
    b_in = rbf16((g.standard_normal(H) * 0.01).astype(np.float32))
    b_out = rbf16((g.standard_normal(D) * 0.01).astype(np.float32))
    v = (g.standard_normal((3, 1, 1, D)) * 0.1).astype(np.float32)
    qi = oq.quantize(w_in, "affine", GS, BITS)
    qo = oq.quantize(w_out, "affine", GS, BITS)
    times = []
    t_start = time.perf_counter()
    while not times or (time.perf_counter() - t_start < seconds_budget and len(times) < 5):
        t0 = time.perf_counter()
        wi = oq.affine_dequantize_fast(qi["weight"], qi["scales"], qi["biases"], D, GS, BITS)
        wo = oq.affine_dequantize_fast(qo["weight"], qo["scales"], qo["biases"], H, GS, BITS)
        ro.ff_sublayer(x, v[0], v[1], v[2], wi, b_in, wo, b_out)
        times.append(time.perf_counter() - t0)
    sec = sorted(times)[len(times) // 2]
    return {"value": 2.0 * sample * D * H * 2 / sec / 1e12, "unit": "TFLOP/s", "cores": os.cpu_count() or 1,
            "kind": "port", "sample": f"{sample} tokens of the {T}-token sub-layer, median of {len(times)} "
                                      f"(dequantize + numpy fp32 BLAS with the reference's bf16 rounding points)"}


# ---------------------------------------------------------------------------- our arm (GPU)


def run_ours(args):
    import torch

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    import ltxq
    from ltxq import _lib

    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    def randn(*shape, std=1.0, dtype=torch.bfloat16):
        return (torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32) * std).to(dtype)

    x = randn(1, T, D)
    ff = ltxq.FeedForward.from_linear(randn(H, D, std=0.02), randn(H, std=0.01), randn(D, H, std=0.02),
                                      randn(D, std=0.01), mode="affine", group_size=GS, bits=BITS)
    scale = randn(1, 1, D, std=0.1, dtype=torch.float32)
    shift = randn(1, 1, D, std=0.1, dtype=torch.float32)
    gate = randn(1, 1, D, std=0.1, dtype=torch.float32)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream()

    def step_kernels(evs):
        # the three launches of the sub-layer, events between them
        evs[0].record(stream)
        a = ltxq.adaln_modulate(x, scale, shift, 1e-6, "rms")
        evs[1].record(stream)
        h = ff.project_in(a, gelu=True)
        evs[2].record(stream)
        y = ff.project_out(h, residual=x, gate=gate)
        evs[3].record(stream)
        return y

    def make_evs():
        return [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    clk = ClockSampler(local).__enter__()  # runs from warm-up through the timed region
    for _ in range(args.warmup):
        flush.fill_(1)
        step_kernels(make_evs())
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()

    all_evs = []
    if True:
        for _ in range(args.steps):
            flush.fill_(1)
            evs = make_evs()
            step_kernels(evs)
            all_evs.append(evs)
        torch.cuda.synchronize()
    clk.__exit__(None, None, None)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    step_ms = [e[0].elapsed_time(e[3]) for e in all_evs]
    gin_ms = [e[1].elapsed_time(e[2]) for e in all_evs]
    gout_ms = [e[2].elapsed_time(e[3]) for e in all_evs]
    mod_ms = [e[0].elapsed_time(e[1]) for e in all_evs]
    total_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = world * FLOPS * args.steps / (total_ms / 1e3) / 1e12

    # ---- e2e through the public API with host buffers
    x_host = x.cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    x_dev = torch.empty_like(x)
    for _ in range(max(1, args.warmup)):
        x_dev.copy_(x_host, non_blocking=True)
        y = ff.sublayer(x_dev, scale, shift, gate)
        out_host.copy_(y, non_blocking=True)
    torch.cuda.synchronize()
    e2e_ms = []
    for _ in range(args.steps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        x_dev.copy_(x_host, non_blocking=True)
        y = ff.sublayer(x_dev, scale, shift, gate)
        out_host.copy_(y, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        e2e_ms.append(e0.elapsed_time(e1))
    e2e_total = sum(e2e_ms)
    if world > 1:
        t = torch.tensor([e2e_total], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_total = float(t.item())
    e2e_value = world * FLOPS * args.steps / (e2e_total / 1e3) / 1e12
    dev_err = _lib.device_error()

    if rank == 0:
        hbm, tf_burst, tf_sust, peak_kind = _peaks()
        gin_avg = sum(gin_ms) / len(gin_ms)
        gin_flops = 2.0 * T * D * H
        achieved = gin_flops / (gin_avg / 1e3) / 1e12
        traffic = _traffic("qgemm_affine4_ff_in_3456x16384x4096")
        cpu = None if args.no_cpu_baseline or world > 1 else cpu_baseline_sample()
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens": T, "d": D, "inner": H, "quant": f"affine int{BITS} g{GS}",
                       "global_batch": world, "seq_len": T, "parallelism": f"replicas{world}",
                       "l2": "flushed before every timed step (256 MiB write, outside the events)"},
            "breakdown_ms": {"adaln_modulate": sum(mod_ms) / len(mod_ms), "qgemm_ff_in_gelu": gin_avg,
                             "qgemm_ff_out_gated": sum(gout_ms) / len(gout_ms)},
            "roofline": {"bound": "tensor", "kernel": "qgemm_kernel<affine4,256> (project_in, GELU epilogue)",
                         "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s", "frac": achieved / tf_burst,
                         "peak_kind": f"{peak_kind} bf16 burst (MEASURED_PEAKS.json)" if peak_kind == "measured"
                         else "fallback 1590 TFLOP/s", "traffic": traffic,
                         "algorithmic_per_launch": {"flops": gin_flops,
                                                    "bytes": T * D * 2 + H * D // 2 + H * D // GS * 4 + T * H * 2}},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": x.numel() * 2,
                    "d2h_bytes_per_step": x.numel() * 2, "api": "ltxq.FeedForward.sublayer -> ltxq_feed_forward"},
            "gpu_launches": 3 * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "device_error": dev_err,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-sample", type=int, default=256)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
