"""CPU tests of bench.py's host-side accounting: the algorithmic FLOPs and
packed-weight bytes the reported figures divide by, against the figures the
reference's configs give (the 22B block: 5.071 TFLOP of block linears at
9216 video / 201 audio / 1024 text tokens, 1.963 TFLOP at 3456 / 126 / 1024;
398.5 / 410.6 / 217.4 MB of packed mxfp8 g32 / int8 g64 / int4 g64 weights per
block), and the config text of the JSON line."""

import pytest


def test_block_linear_flops():
    import bench

    assert bench.step_linear_flops(9216, 201, 1024) / 1e12 == pytest.approx(5.071, abs=5e-4)
    assert bench.step_linear_flops(9216, 201, 1024) * 48 / 1e12 == pytest.approx(243.4, abs=0.05)
    assert bench.step_linear_flops(3456, 126, 1024) / 1e12 == pytest.approx(1.963, abs=5e-4)
    # linear in the video rows at fixed audio / text rows
    f0 = bench.step_linear_flops(0, 201, 1024)
    assert bench.step_linear_flops(2 * 1152, 201, 1024) - f0 == pytest.approx(
        2 * (bench.step_linear_flops(1152, 201, 1024) - f0))


@pytest.mark.parametrize("quant,mb", [("mxfp8", 398.5), ("int8", 410.6), ("int4", 217.4)])
def test_packed_bytes_per_block(quant, mb):
    import bench
    from ltxq.block import linear_specs

    total = sum(bench._packed_bytes(quant, n, k) for n, k in linear_specs().values())
    assert total / 1e6 == pytest.approx(mb, abs=0.05)


def test_step_config_names_the_exchange():
    import bench

    assert bench._step_config(1)["parallelism"] == "single GPU (no collective)"
    p8 = bench._step_config(8)["parallelism"]
    assert "x8" in p8 and "K/V all-gather" in p8
    hp = bench._step_config(8, self_attention="head_parallel", v2a="split_keys")["parallelism"]
    assert "all-to-all" in hp and "log-sum-exp" in hp
    cfg = bench._step_config(1)
    assert cfg["workload"] == "config4_22b_denoise_step_mxfp8g32" and cfg["video_tokens"] == 9216
    assert cfg["blocks"] == 48 and cfg["audio_tokens"] == 201 and cfg["text_tokens"] == 1024
