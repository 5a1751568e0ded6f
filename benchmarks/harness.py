"""Timing and reporting helpers shared by the benchmarks.

GPU timings use CUDA events on the launching stream after warm-up, with a
synchronize on both sides, and report the median; CPU timings use
``time.perf_counter``. Roofline denominators come from MEASURED_PEAKS.json at
the repository root when present (else the pool's fallback figures).
"""

from __future__ import annotations

import json
import os
import platform
import statistics
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    d = dict(FALLBACK_PEAKS)
    d["source"] = "fallback"
    return d


def bench(fn, *, warmup: int = 3, reps: int = 10, flush_l2: bool = True) -> float:
    """Median milliseconds of ``fn()``."""
    if torch.cuda.is_available():
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if flush_l2 else None
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(reps):
            if flush is not None:
                flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        return statistics.median(times)
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times)


class clocks:
    """``with clocks() as c: ...`` samples the SM clock of GPU 0 during the block
    (bench.py's nvidia-smi sampler); ``c.result`` = {sm_mhz (median under load),
    sm_max_mhz, reasons, samples}."""

    def __init__(self, gpu_index: int = 0):
        import sys

        sys.path.insert(0, ROOT)
        from bench import ClockSampler

        self.sampler = ClockSampler(gpu_index)
        self.result: dict | None = None

    def __enter__(self):
        self.sampler.start()
        return self

    def __exit__(self, *exc):
        self.result = self.sampler.stop()
        return False


def ortho_flops(batch: int, rows: int, cols: int, steps: int = 5) -> float:
    """Dense FLOPs of the iteration: steps * (4 N^2 M + 2 N^3), N = min dim."""
    n, m = min(rows, cols), max(rows, cols)
    return batch * steps * (4.0 * n * n * m + 2.0 * n**3)


def capture_env() -> dict:
    env = {"python": platform.python_version(), "torch": torch.__version__}
    if torch.cuda.is_available():
        env["gpu"] = torch.cuda.get_device_name()
        env["cuda"] = torch.version.cuda
    return env


def markdown_table(headers: list[str], rows: list[list]) -> str:
    def fmt(x):
        return f"{x:.4f}" if isinstance(x, float) else str(x)

    out = ["| " + " | ".join(headers) + " |", "|" + "---|" * len(headers)]
    out += ["| " + " | ".join(fmt(c) for c in r) + " |" for r in rows]
    return "\n".join(out)
