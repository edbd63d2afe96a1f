"""bench.py's host-side pieces on the CPU: the FLOP count of the metric, the workload
description, the per-launch traffic figures it reads from profiles/, the clock record
it parses from nvidia-smi, and the CPU baseline sampler on a small shape."""
import math

import bench


def test_metric_flop_count_is_the_two_gemm_convention():
    # 4 * B * H * T^2 * D at config 2: 3.436e10 per fwd+bwd step
    assert bench.flops_per_step() == 4.0 * 2 * 16 * 2048 * 2048 * 64
    assert math.isclose(bench.flops_per_step(), 3.436e10, rel_tol=1e-3)


def test_workload_description():
    cfg = bench._config(2, "auto")
    assert cfg["global_batch"] == 4 and cfg["seq_len"] == 2048 and cfg["head_dim"] == 64
    assert cfg["parallelism"] == "bh-shard x2"
    assert "config 2" in cfg["workload"]


def test_traffic_figures_come_from_the_committed_profile():
    for tag in ("auto_backward", "tcgen05_backward", "auto_forward", "tcgen05_forward"):
        t = bench._profile_traffic(tag)
        assert t is not None and t > 1e7, tag
    # backward reads q, k, v, dO and the fp32 dQ accumulator at least once (50.3 MB)
    assert bench._profile_traffic("auto_backward") >= 4 * 8388608 + 16777216
    assert bench._profile_traffic("no_such_kernel") is None


def test_clock_record_parsing():
    s = bench.ClockSampler(0)
    s.lines = [
        "0, 1965, 1965, 250.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1950, 1965, 340.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1965, 1965, 300.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "garbage line",
    ]
    out = s.summary()
    assert out["samples"] == 3
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]
    assert math.isclose(out["power_w"], 300.0)
    s.lines = ["0, 1400, 1965, 500.0, 0x0000000000000008, Active, Not Active, Not Active, Not Active"]
    assert s.summary()["reasons"] == ["hw_slowdown"]
    s.lines = []
    assert s.summary() is None


def test_cpu_baseline_sampler_on_a_small_shape():
    tflops, med, threads, sample = bench.cpu_reference_sample(1, 0, shape=(1, 2, 64, 16))
    assert tflops > 0 and med > 0 and threads >= 1
    assert "[1, 2, 64, 16]" in sample
