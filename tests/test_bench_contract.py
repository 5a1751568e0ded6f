"""Host-side pieces of bench.py: clock-record parsing and the argument contract."""

import sys

import bench


def test_clock_summary_median_under_load_and_reasons():
    lines = [
        "0, 1965, 1965, 300.0, Not Active, Not Active, Not Active, Not Active\n",  # idle, before load
        "0, 1282, 1965, 990.5, Not Active, Not Active, Not Active, Active\n",
        "0, 1300, 1965, 995.1, Not Active, Not Active, Not Active, Active\n",
        "0, 1250, 1965, 998.0, Not Active, Not Active, Not Active, Active\n",
        "0, 180, 1965, 80.0, Not Active, Not Active, Not Active, Not Active\n",  # idle after load
    ]
    out = bench.ClockSampler.summarize(lines)
    assert out["sm_max_mhz"] == 1965.0
    assert out["sm_mhz"] == 1291.0  # median of the samples above half of max (1965, 1300, 1282, 1250)
    assert out["reasons"] == ["sw_power_cap"]
    assert out["samples"] == 5


def test_clock_summary_tolerates_na_and_junk():
    lines = ["0, [N/A], [N/A], [N/A], [N/A], [N/A], [N/A], [N/A]\n", "garbage\n", "\n"]
    out = bench.ClockSampler.summarize(lines)
    assert out["sm_mhz"] is None and out["sm_max_mhz"] is None and out["samples"] == 1
    assert bench.ClockSampler.summarize([])["reasons"] == ["no samples"]


def test_clock_summary_flags_thermal_reasons():
    lines = ["0, 1500, 1965, 700, Active, Not Active, Active, Not Active\n"]
    assert bench.ClockSampler.summarize(lines)["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]


def test_default_arguments_are_one_gpu_and_valid_warmup(monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    args = bench.parse_args()
    assert args.gpus == 1 and args.warmup >= 3 and args.steps >= 1
    assert args.impl == "ours"
