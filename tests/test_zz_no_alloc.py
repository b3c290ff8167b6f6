"""The allocation-free AdaLN + quantized linear entry point.

ltxq_adaln_qlinear_noalloc exists for hosts that cannot let a library
allocate device memory (a runtime owning the GPU's memory through its own
pool, a plugin inside another framework's allocator, a loop where a
cudaMalloc would synchronize the device).  Its scratch is a fixed array in the
library's device image.  This test calls it through the C ABI twice in a row,
with different inputs, and checks each result against the workspace-taking
entry point ltxq_adaln_qlinear on the same inputs and against the numpy
oracle's AdaLN + affine int8 g64 linear + gated residual composition, within
the GEMM tolerance used by the other parity tests.  The file is named to be
collected last.
"""

import ctypes

import pytest

from helpers import from_dev_bf16, normal_bf16, normal_f32, rng, to_dev, to_dev_bf16
from oracle import quant as oq
from oracle import ref_ops as ro

pytestmark = pytest.mark.gpu

MAX_ABS_REL = 2e-2
COS_MIN = 0.9995


def _case(seed, M, K, N):
    import torch

    from ltxq import _lib

    g = rng(seed)
    x_h = normal_bf16(g, (M, K))
    W = normal_bf16(g, (N, K), 0.02)
    q = oq.quantize(W, "affine", 64, 8)
    host = {"x": x_h, "q": q, "bias": normal_bf16(g, (N,), 0.01), "scale": normal_f32(g, (K,), 0.1),
            "shift": normal_f32(g, (K,), 0.1), "gate": normal_f32(g, (N,), 0.1), "res": normal_bf16(g, (M, N))}
    keep = {
        "x": to_dev_bf16(x_h),
        "w": to_dev(q["weight"]),
        "s": to_dev(q["scales"]),
        "b": to_dev(q["biases"]),
        "bias": to_dev_bf16(host["bias"]),
        "scale": torch.from_numpy(host["scale"]).cuda(),
        "shift": torch.from_numpy(host["shift"]).cuda(),
        "gate": torch.from_numpy(host["gate"]).cuda(),
        "res": to_dev_bf16(host["res"]),
        "host": host,
    }
    qw = _lib.QWeight(keep["w"].data_ptr(), keep["s"].data_ptr(), keep["b"].data_ptr(), keep["bias"].data_ptr(),
                      N, K, _lib.AFFINE, 8, 64, _lib.LAYOUT_STD)
    pro = _lib.Prologue(_lib.NORM_RMS, 1e-6, _lib.Vec(keep["scale"].data_ptr(), _lib.F32, 0, 0, 0),
                        _lib.Vec(keep["shift"].data_ptr(), _lib.F32, 0, 0, 0))
    epi = _lib.Epilogue(_lib.EPI_GATED_RESIDUAL, 0, _lib.Vec(keep["gate"].data_ptr(), _lib.F32, 0, 0, 0),
                        keep["res"].data_ptr())
    return keep, qw, pro, epi


def _with_workspace(lib, keep, qw, pro, epi, M, N):
    import torch

    from ltxq import _lib

    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    ws_bytes = lib.ltxq_adaln_qlinear_workspace_size(M, ctypes.byref(qw))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    _lib.check(lib.ltxq_adaln_qlinear(keep["x"].data_ptr(), M, ctypes.byref(pro), ctypes.byref(qw), ctypes.byref(epi),
                                      out.data_ptr(), ws.data_ptr(), ws_bytes, None), "adaln_qlinear")
    return out


def _no_alloc(lib, keep, qw, pro, epi, M, N):
    import torch

    from ltxq import _lib

    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    _lib.check(lib.ltxq_adaln_qlinear_noalloc(keep["x"].data_ptr(), M, ctypes.byref(pro), ctypes.byref(qw),
                                              ctypes.byref(epi), out.data_ptr(), None), "adaln_qlinear_noalloc")
    return out


def test_no_alloc_entry_point_matches_workspace_entry_point_twice(cuda):
    import torch

    from ltxq import _lib

    lib = _lib.load()
    for seed, (M, K, N) in ((21, (700, 1024, 768)), (22, (256, 2048, 512))):
        keep, qw, pro, epi = _case(seed, M, K, N)
        got = from_dev_bf16(_no_alloc(lib, keep, qw, pro, epi, M, N))
        want = from_dev_bf16(_with_workspace(lib, keep, qw, pro, epi, M, N))
        torch.cuda.synchronize()
        mar, cos = ro.max_abs_rel(got, want), ro.cosine(got, want)
        assert mar <= MAX_ABS_REL and cos >= COS_MIN, f"call seed={seed}: max_abs_rel={mar:.3e} cos={cos:.6f}"
        h = keep["host"]
        y = ro.linear(ro.adaln(h["x"], h["scale"], h["shift"], 1e-6, "rms"), oq.dequantize(h["q"], K), h["bias"])
        ref = ro.gated_add(h["res"], y, h["gate"])
        for name, out in (("no-alloc", got), ("workspace", want)):
            mar, cos = ro.max_abs_rel(out, ref), ro.cosine(out, ref)
            assert mar <= MAX_ABS_REL and cos >= COS_MIN, f"{name} seed={seed} vs oracle: {mar:.3e} {cos:.6f}"
    assert _lib.device_error() == 0


def test_no_alloc_entry_point_rejects_oversized_requests(cuda):
    from ltxq import _lib

    lib = _lib.load()
    qw = _lib.QWeight(16, 16, 16, None, 128, 4096, _lib.AFFINE, 8, 64, _lib.LAYOUT_STD)
    pro = _lib.Prologue(_lib.NORM_RMS, 1e-6, _lib.Vec(16, _lib.F32, 0, 0, 0), _lib.Vec(16, _lib.F32, 0, 0, 0))
    st = lib.ltxq_adaln_qlinear_noalloc(16, 1025, ctypes.byref(pro), ctypes.byref(qw), None, 16, None)
    assert st == _lib.ERR_UNSUPPORTED
    assert b"static scratch" in lib.ltxq_last_error()
