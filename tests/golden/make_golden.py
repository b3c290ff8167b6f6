"""Writes the golden fixtures of tests/golden (run from the repository root:
``python tests/golden/make_golden.py``).

The reference's arithmetic lives in MLX, which cannot be installed here, so
no vector below was produced by the reference itself:

* ``reference_kats.json``: known answers transcribed from the reference's own
  tests (file:line of dmlsrc/LTX-2-MLX given per entry);
* ``oracle_vectors.npz``: outputs of this repository's oracle (a numpy
  restatement of the reference's MLX composition) on seeded inputs, so that
  a change to the oracle shows up as a diff against committed values.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import quant as oq  # noqa: E402
from oracle import ref_ops as ro  # noqa: E402
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits  # noqa: E402

KATS = {
    "e4m3_decode": {
        "source": "tests/test_transformer_cache.py:64-95",
        "note": "FP8 checkpoint weight byte 0x38 with weight_scale 2.0 loads as bf16 2.0",
        "code": 0x38, "value": 1.0, "weight_scale": 2.0, "scaled_bf16": 2.0,
    },
    "payload_group_override": {
        "source": "tests/test_transformer_cache.py:98-115",
        "note": "the cache payload records the quantization group size; 32 and 64 give different payloads",
        "mode": "mxfp8-blocks", "group_sizes": [32, 64],
        "key": "transformer_cache_quantize_group_size",
    },
    "safetensors_metadata": {
        "source": "tests/test_safetensors_header.py:12-34",
        "note": "metadata strings and dtypes round-trip through a safetensors header; no metadata reads as {}",
        "metadata": {"model_version": "2.3.0", "config": "{\"x\": 1}"},
        "dtypes": {"w": "F32", "b": "BF16"},
    },
    "fused_ops_thresholds": {
        "source": "tests/test_fused_ops.py:63-217",
        "note": "fused AdaLN / gated-add kernels agree with the MLX compositions to cosine >= 0.9999",
        "cosine_min": 0.9999,
    },
}


def oracle_vectors() -> dict[str, np.ndarray]:
    g = np.random.Generator(np.random.PCG64(0))
    out: dict[str, np.ndarray] = {}
    # GELU (feed_forward.py:8-14) on every bf16 input
    pats = np.arange(0x10000, dtype=np.uint32).astype(np.uint16)
    with np.errstate(all="ignore"):
        out["gelu_all_bf16"] = f32_to_bf16_bits(ro.gelu_approx(bf16_bits_to_f32(pats)))
    # mxfp8 dequant: every code under scales 0..254 (one row per scale)
    codes = np.tile(np.arange(256, dtype=np.uint8), (255, 1))
    scales = np.repeat(np.arange(255, dtype=np.uint8)[:, None], 8, axis=1)
    q = {"weight": codes.reshape(255, 64, 4).copy().view(np.uint32).reshape(255, 64), "scales": scales,
         "group_size": 32, "bits": 8, "mode": "mxfp8"}
    with np.errstate(over="ignore", invalid="ignore"):  # scales near 254 overflow to inf, NaN codes stay NaN
        out["mxfp8_dequant_all_codes"] = f32_to_bf16_bits(oq.dequantize(q, 256))
    # affine int8 / int4 quantize + dequantize of a seeded bf16 weight
    w = ro.rbf16(g.standard_normal((16, 256)).astype(np.float32) * np.float32(0.02))
    for bits in (8, 4):
        qa = oq.quantize(w, "affine", 64, bits)
        out[f"affine{bits}_weight"] = qa["weight"]
        out[f"affine{bits}_scales"] = qa["scales"]
        out[f"affine{bits}_biases"] = qa["biases"]
        out[f"affine{bits}_dequant"] = f32_to_bf16_bits(oq.dequantize(qa, 256))
    # benchmark config 1 structure at a small size: x + gate * (mod(LN(x)) @ W^T + b)
    x = ro.rbf16(g.standard_normal((8, 256)).astype(np.float32))
    sc = ro.rbf16(g.standard_normal((1, 256)).astype(np.float32) * np.float32(0.1))
    sh = ro.rbf16(g.standard_normal((1, 256)).astype(np.float32) * np.float32(0.1))
    gt = ro.rbf16(g.standard_normal((1, 256)).astype(np.float32) * np.float32(0.1))
    wq = oq.quantize(ro.rbf16(g.standard_normal((256, 256)).astype(np.float32) * np.float32(0.02)), "affine", 64, 8)
    b = ro.rbf16(g.standard_normal((256,)).astype(np.float32) * np.float32(0.01))
    out["cfg1_x"], out["cfg1_scale"], out["cfg1_shift"], out["cfg1_gate"] = (f32_to_bf16_bits(a) for a in (x, sc, sh, gt))
    out["cfg1_weight"], out["cfg1_scales"], out["cfg1_biases"] = wq["weight"], wq["scales"], wq["biases"]
    out["cfg1_bias"] = f32_to_bf16_bits(b)
    for norm in ("layer", "rms"):
        y = ro.adaln_linear_gated(x, sc, sh, gt, oq.dequantize(wq, 256), b, 1e-6, norm, vec_bf16=True)
        out[f"cfg1_out_{norm}"] = f32_to_bf16_bits(y)
    return out


def main() -> None:
    with open(os.path.join(HERE, "reference_kats.json"), "w") as f:
        json.dump(KATS, f, indent=1, sort_keys=True)
    np.savez_compressed(os.path.join(HERE, "oracle_vectors.npz"), **oracle_vectors())


if __name__ == "__main__":
    main()
