"""Run the benchmark suite and write RESULTS.md (kernels, optimizer step).

    python benchmarks/run.py [--quick] [--with-reference] [--out benchmarks/RESULTS.md]

The distributed benchmark needs torchrun (see bench_distributed.py).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from benchmarks import bench_kernels, bench_optim  # noqa: E402
from benchmarks.harness import capture_env  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--with-reference", action="store_true")
    ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)), "RESULTS.md"))
    args = ap.parse_args()
    parts = ["# Benchmark results", "", "```", json.dumps(capture_env(), indent=1), "```", ""]
    parts += ["## Orthogonalisation kernels", "",
              bench_kernels.run(bench_kernels.QUICK if args.quick else bench_kernels.CONFIG2, args.with_reference), ""]
    parts += ["## optimizer.step()", "", bench_optim.run(bench_optim.QUICK if args.quick else bench_optim.FULL, args.with_reference), ""]
    text = "\n".join(parts)
    with open(args.out, "w") as f:
        f.write(text)
    print(text)


if __name__ == "__main__":
    main()
