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


def test_cpu_block_rotation_times_every_sublayer_and_sums_them():
    """The reference arm's unit: each timed step runs one sub-layer of the
    block at full size in turn; every sub-layer is timed at least once and a
    block is the sum of the sub-layer means (a stub stands in for the numpy
    work here)."""
    import bench

    class Stub:
        video_tokens, audio_tokens, quant = 9216, 201, "mxfp8"

        def __init__(self):
            self.calls = []

        def run(self, sub):
            self.calls.append(sub)
            return 1.0 + list(bench.CpuBlock.SUBLAYERS).index(sub)

    stub = Stub()
    per_sub = bench._cpu_block_rotation(stub, 3, warmup=2)
    assert set(per_sub) == set(bench.CpuBlock.SUBLAYERS) and len(stub.calls) == 2 + 7
    assert sum(per_sub.values()) == pytest.approx(sum(range(1, 8)))
    ms, desc = bench._cpu_block_line(per_sub, stub, 48)
    assert ms == pytest.approx(28.0 * 48 * 1e3) and "extrapolated x48" in desc and "attention included" in desc
    ms1, desc1 = bench._cpu_block_line(per_sub, stub, 1)
    assert ms1 == pytest.approx(28.0 * 1e3) and "not extrapolated" in desc1


def test_presets_name_the_baseline_configs():
    import bench

    assert bench.STEP_PRESETS["config3"][:5] == (1, "int8", 3456, 126, 1)
    assert bench.STEP_PRESETS["config5"][:5] == (48, "int4", 30576, 751, 2)
    cfg = bench._step_config(1, 48, True, "int4", 30576, audio_tokens=751, batch=2,
                             workload=bench.STEP_PRESETS["config5"][5])
    assert cfg["global_batch"] == 2 and cfg["audio_tokens"] == 751 and cfg["workload"].startswith("config5")
    assert bench._config1_config(1)["workload"].startswith("config1")


def test_exchange_forms_by_gpu_count():
    """--self-attention / --v2a auto: the K/V all-gathers below 8 GPUs, the
    all-to-all and split-key forms from 8 up; explicit choices pass through."""
    import bench

    assert bench.exchange_forms(1) == ("gather", "gather")
    assert bench.exchange_forms(2) == ("gather", "gather")
    assert bench.exchange_forms(4) == ("gather", "gather")
    assert bench.exchange_forms(8) == ("head_parallel", "split_keys")
    assert bench.exchange_forms(8, "gather", "gather") == ("gather", "gather")
    assert bench.exchange_forms(2, "head_parallel", "split_keys") == ("head_parallel", "split_keys")


def test_exchange_ms_pairs_probe_events():
    """bench.exchange_ms: the time between each phase-0 / phase-1 probe pair
    is summed per kind; unpaired or out-of-order records raise."""
    import bench

    class Ev:
        def __init__(self, t):
            self.t = t

        def elapsed_time(self, other):
            return other.t - self.t

    evs = [("wait", 0, Ev(1.0)), ("wait", 1, Ev(1.5)), ("sync", 0, Ev(2.0)), ("sync", 1, Ev(2.25)),
           ("wait", 0, Ev(3.0)), ("wait", 1, Ev(3.0))]
    assert bench.exchange_ms(evs) == {"wait": 0.5, "sync": 0.25}
    assert bench.exchange_ms([]) == {"wait": 0.0, "sync": 0.0}
    with pytest.raises(ValueError):
        bench.exchange_ms(evs[:3])
    with pytest.raises(ValueError):
        bench.exchange_ms([("wait", 0, Ev(0.0)), ("sync", 1, Ev(1.0))])
