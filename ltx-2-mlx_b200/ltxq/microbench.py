"""Quantized-linear microbenchmark (the analogue of the reference's
scripts/bench_ff_microbench.py ``quant_matmul``, :451-551).

    python -m ltxq.microbench --shapes 9216x4096x4096 --modes affine4,mxfp8,mxfp8_mx2
    python -m ltxq.microbench --cublas            # also time torch bf16 F.linear
    python -m ltxq.microbench --adaln 9216x4096   # the AdaLN pass alone (bf16 / MX outputs)
    python -m ltxq.microbench --attention 9216x9216x32x128   # attention core vs torch SDPA

Each shape is MxKxN (tokens x in x out).  Prints one JSON line per shape
with ms and TFLOP/s (2*M*N*K / time) per mode; the L2 is flushed (256 MiB
write) before every timed launch and each number is the median of
``--iters`` CUDA-event timings.  ``--iters 1 --warmup 1`` gives a short
launch sequence suitable for an ncu capture.

``--graph`` times device work only: the calls are captured in a CUDA graph
over enough copies of the packed weight to exceed the L2 (each call reads
its weight from HBM, as in a block), and the graph's time is divided by the
number of calls.  Without it, a GEMM shorter than the host-side cost of one
call (Python, ctypes, tensor-map encoding, launch) measures that cost.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import _lib
from .quantized_linear import QuantizedLinear

DEFAULT_SHAPES = ["1024x4096x4096", "3456x4096x16384", "3456x16384x4096", "9216x4096x12288", "9216x4096x4096",
                  "9216x16384x4096", "126x2048x8192", "201x4096x2048"]
# name -> (quantization mode, bits, compute mode)
MODES = {"affine8": ("affine", 8, "dequant"), "affine4": ("affine", 4, "dequant"), "mxfp8": ("mxfp8", 8, "dequant"),
         "mxfp8_mx2": ("mxfp8", 8, "mx2"), "mxfp8_mx1": ("mxfp8", 8, "mx1")}


def _time(fn, flush, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return ts[len(ts) // 2]


def _time_graph(fns, iters):
    """Device time per call of a list of calls captured back to back."""
    for f in fns:  # first calls do one-time host work (data-flag scans) outside the capture
        f()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for f in fns:
            f()
    graph.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b) / len(fns))
    ts.sort()
    del graph
    return ts[len(ts) // 2]


def _adaln(spec: str, iters: int) -> None:
    """The AdaLN pass (RMS norm, fp32 modulate vectors) over M x C bf16 rows,
    graph-timed over copies of x larger than the L2, with bf16 output and
    with the output written as 2 / 1 MX terms.  Bytes per call: x read +
    output written + the two vectors."""
    from . import kernels as K

    M, C = (int(v) for v in spec.split("x"))
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    copies = max(1, -(-(256 << 20) // (M * C * 2)))
    xs = [torch.randn(M, C, device=dev, generator=g).to(torch.bfloat16) for _ in range(copies)]
    sc = torch.randn(1, C, device=dev, generator=g) * 0.1
    sh = torch.randn(1, C, device=dev, generator=g) * 0.1
    row = {"adaln": {"M": M, "C": C, "graph_calls": copies}}
    for name, terms in (("bf16_out", 0), ("mx2_out", 2), ("mx1_out", 1)):
        t = _time_graph([lambda x=x: K.adaln_modulate(x, sc, sh, 1e-6, mx_terms=terms) for x in xs], iters)
        out_bytes = M * C * (2 if terms == 0 else terms) + (M * C // 32) * terms
        nbytes = M * C * 2 + out_bytes + 2 * C * 4
        row[name] = {"ms": t, "gbs": nbytes / t / 1e6, "bytes": nbytes}
    print(json.dumps(row), flush=True)


def _attention(spec: str, iters: int) -> None:
    """The attention core at Tq x Tk x heads x D: ``ltxq_attention`` and
    torch's SDPA (cuDNN / flash) on the same bf16 inputs, graph-timed.
    FLOP = 4 * Tq * Tk * heads * D."""
    import math

    import torch.nn.functional as F

    from . import kernels as K

    tq, tk, heads, d = (int(v) for v in spec.split("x"))
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q, k, v = (torch.randn(1, t, heads * d, device=dev, generator=g).to(torch.bfloat16) for t in (tq, tk, tk))
    hv = lambda t: t.view(1, t.shape[1], heads, d).transpose(1, 2)
    flops = 4.0 * tq * tk * heads * d
    row = {"attention": {"Tq": tq, "Tk": tk, "heads": heads, "D": d}}
    t = _time_graph([lambda: K.attention(q, k, v, heads)], iters)
    row["ltxq"] = {"ms": t, "tflops": flops / t / 1e9}
    t = _time_graph([lambda: F.scaled_dot_product_attention(hv(q), hv(k), hv(v), scale=1.0 / math.sqrt(d))], iters)
    row["torch_sdpa"] = {"ms": t, "tflops": flops / t / 1e9}
    print(json.dumps(row), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default=",".join(DEFAULT_SHAPES))
    ap.add_argument("--modes", default="affine8,affine4,mxfp8")
    ap.add_argument("--epilogue", choices=["none", "gelu", "gated"], default="none")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--cublas", action="store_true")
    ap.add_argument("--no-split-k", action="store_true", help="give the GEMM no split-K workspace")
    ap.add_argument("--graph", action="store_true", help="device time per call from a captured CUDA graph")
    ap.add_argument("--pretransposed", action="store_true", help="pack W^T (the cache's pretranspose mode; mxfp8)")
    ap.add_argument("--adaln", default=None, help="MxC: time the AdaLN pass instead of the GEMMs")
    ap.add_argument("--attention", default=None, help="TqxTkxHxD: time the attention core instead of the GEMMs")
    args = ap.parse_args(argv)
    if args.adaln:
        _adaln(args.adaln, args.iters)
        return
    if args.attention:
        for spec in args.attention.split(","):
            _attention(spec, args.iters)
        return
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for spec in args.shapes.split(","):
        M, K, N = (int(v) for v in spec.split("x"))
        x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        b = (torch.randn(N, device=dev, generator=g) * 0.01).to(torch.bfloat16)
        res = torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16)
        gate = torch.randn(N, device=dev, generator=g) * 0.1
        row = {"M": M, "K": K, "N": N, "epilogue": args.epilogue, "split_k": not args.no_split_k,
               "pretransposed": args.pretransposed}
        flops = 2.0 * M * N * K
        if args.cublas:
            t = _time(lambda: torch.nn.functional.linear(x, w, b), flush, args.iters, args.warmup)
            row["cublas_bf16"] = {"ms": t, "tflops": flops / t / 1e9}
        for name in args.modes.split(","):
            mode, bits, compute = MODES[name]
            ql = QuantizedLinear.from_linear(w, b, mode=mode, bits=bits, pretransposed=args.pretransposed)
            ql.set_compute(compute)
            kw = {"gelu": True} if args.epilogue == "gelu" else (
                {"residual": res, "gate": gate} if args.epilogue == "gated" else {})
            kw["split_k"] = not args.no_split_k
            if args.graph:
                wbytes = ql.weight.numel() * ql.weight.element_size()
                copies = max(1, min(64, -(-(256 << 20) // max(wbytes, 1))))
                qls = [ql] + [QuantizedLinear(ql.weight.clone(), ql.scales.clone(),
                                              None if ql.biases is None else ql.biases.clone(), ql.bias,
                                              group_size=ql.group_size, bits=ql.bits, mode=ql.mode,
                                              pretransposed=ql.pretransposed, in_features=ql.in_features,
                                              out_features=ql.out_features).set_compute(compute)
                              for _ in range(copies - 1)]
                t = _time_graph([lambda q=q: q(x, **kw) for q in qls], args.iters)
                row["graph_calls"] = copies
            else:
                t = _time(lambda: ql(x, **kw), flush, args.iters, args.warmup)
            row[name] = {"ms": t, "tflops": flops / t / 1e9}
        print(json.dumps(row), flush=True)
    err = _lib.device_error()
    if err:
        raise SystemExit(f"device error word {err}")


if __name__ == "__main__":
    main()
