"""Golden fixtures (tests/golden, written by tests/golden/make_golden.py).

CPU: the reference's known answers (transcribed from its tests) hold for the
oracle and the cache module, and the oracle still reproduces its committed
vectors bit for bit.  GPU: the CUDA path against the committed vectors."""

import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, HERE)


def _kats():
    with open(os.path.join(HERE, "reference_kats.json")) as f:
        return json.load(f)


def _vectors():
    return dict(np.load(os.path.join(HERE, "oracle_vectors.npz")))


def _nan_bits(b):
    return ((b & 0x7F80) == 0x7F80) & ((b & 0x7F) != 0)


def test_reference_kats_hold():
    from oracle.bf16 import e4m3_decode, rbf16

    from ltxq import cache

    k = _kats()
    e = k["e4m3_decode"]
    v = e4m3_decode(np.array([e["code"]], dtype=np.uint8))
    assert v[0] == e["value"]
    assert float(rbf16(np.float32(v[0] * e["weight_scale"]))) == e["scaled_bf16"]
    p = k["payload_group_override"]
    a, b = (cache.cache_payload(p["mode"], group_size=gs) for gs in p["group_sizes"])
    assert a[p["key"]] == p["group_sizes"][0] and b[p["key"]] == p["group_sizes"][1] and a != b


def test_safetensors_kat(tmp_path):
    import torch

    from ltxq import cache

    s = _kats()["safetensors_metadata"]
    f = tmp_path / "t.safetensors"
    cache.save_safetensors(f, {"w": torch.zeros(2, 3), "b": torch.ones(3, dtype=torch.bfloat16)}, s["metadata"])
    assert cache.read_safetensors_metadata(f) == s["metadata"]
    assert cache.read_safetensors_dtypes(f) == s["dtypes"]


def test_oracle_reproduces_committed_vectors():
    import make_golden

    now = make_golden.oracle_vectors()
    ref = _vectors()
    assert set(now) == set(ref)
    for name, arr in ref.items():
        assert np.array_equal(now[name], arr), name


@pytest.mark.gpu
def test_gpu_dequant_all_codes_against_golden(cuda):
    import torch

    import ltxq

    v = _vectors()
    codes = np.tile(np.arange(256, dtype=np.uint8), (255, 1))
    scales = np.repeat(np.arange(255, dtype=np.uint8)[:, None], 8, axis=1)
    w = torch.from_numpy(codes.reshape(255, 64, 4).copy().view(np.int32).reshape(255, 64)).cuda()
    ql = ltxq.QuantizedLinear(w, torch.from_numpy(scales).cuda(), None, None, group_size=32, bits=8, mode="mxfp8",
                              in_features=256, out_features=255)
    got = ql.dequantize().view(torch.int16).cpu().numpy().view(np.uint16)
    want = v["mxfp8_dequant_all_codes"]
    assert np.array_equal(_nan_bits(got), _nan_bits(want))
    assert np.array_equal(got[~_nan_bits(want)], want[~_nan_bits(want)])


@pytest.mark.gpu
@pytest.mark.parametrize("norm", ["layer", "rms"])
def test_gpu_config1_against_golden(cuda, norm):
    import torch

    import ltxq
    from oracle import ref_ops as ro
    from oracle.bf16 import bf16_bits_to_f32

    v = _vectors()

    def dev(bits):
        return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).cuda().view(torch.bfloat16)

    ql = ltxq.QuantizedLinear(torch.from_numpy(v["cfg1_weight"].view(np.int32)).cuda(), dev(v["cfg1_scales"]),
                              dev(v["cfg1_biases"]), dev(v["cfg1_bias"]), group_size=64, bits=8, mode="affine",
                              in_features=256, out_features=256)
    x = dev(v["cfg1_x"])
    out = ql(x, residual=x, gate=dev(v["cfg1_gate"]),
             adaln=(dev(v["cfg1_scale"]), dev(v["cfg1_shift"]), 1e-6, norm))
    got = bf16_bits_to_f32(out.view(torch.int16).cpu().numpy().view(np.uint16))
    ref = bf16_bits_to_f32(v[f"cfg1_out_{norm}"])
    assert ro.max_abs_rel(got, ref) <= 2e-2 and ro.cosine(got, ref) >= 0.9995
