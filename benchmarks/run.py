"""Run the benchmark suite and write RESULTS.md (kernels, optimizer step).

    python benchmarks/run.py [--quick] [--with-reference] [--no-distributed] [--out benchmarks/RESULTS.md]

With two or more visible GPUs (and no ``--no-distributed``) the distributed
benchmark also runs, as its own ``torch.distributed.run`` job over every
visible GPU (reference runner: benchmark/run.py:27-56).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from benchmarks import bench_kernels, bench_optim  # noqa: E402
from benchmarks.harness import capture_env  # noqa: E402


def run_distributed(quick: bool) -> str:
    import torch

    n = torch.cuda.device_count()
    if n < 2:
        return "skipped: fewer than 2 GPUs visible"
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", "29577", os.path.join(here, "bench_distributed.py")]
    if quick:
        cmd.append("--quick")
    res = subprocess.run(cmd, capture_output=True, text=True, cwd=os.path.dirname(here))
    rows = [ln for ln in res.stdout.splitlines() if ln.startswith("|")]
    if res.returncode != 0:
        return f"failed (exit {res.returncode}): " + (res.stderr.strip().splitlines() or ["no output"])[-1]
    return "\n".join(rows) if rows else res.stdout.strip()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--with-reference", action="store_true")
    ap.add_argument("--no-distributed", action="store_true")
    ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)), "RESULTS.md"))
    args = ap.parse_args()
    parts = ["# Benchmark results", "", "```", json.dumps(capture_env(), indent=1), "```", ""]
    parts += ["## Orthogonalisation kernels", "",
              bench_kernels.run(bench_kernels.QUICK if args.quick else bench_kernels.CONFIG2, args.with_reference), ""]
    parts += ["## optimizer.step()", "", bench_optim.run(bench_optim.QUICK if args.quick else bench_optim.FULL, args.with_reference), ""]
    if not args.no_distributed:
        parts += ["## Distributed orthogonalisation", "", run_distributed(args.quick), ""]
    text = "\n".join(parts)
    with open(args.out, "w") as f:
        f.write(text)
    print(text)


if __name__ == "__main__":
    main()
