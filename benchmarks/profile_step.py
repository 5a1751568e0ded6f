"""Kernel-time shares of one Llama training step (diagnostic; torch.profiler).

    python benchmarks/profile_step.py [--model llama3-8b] [--layers N]

Prints total CUDA kernel time and the top kernels by time. Use the numbers as
shares only: timings under a profiler are not reported as results (bench.py
times the step with CUDA events and no profiler).
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--top", type=int, default=40)
    args = ap.parse_args()
    from torch.profiler import ProfilerActivity, profile

    from dtensor_muon_b200.models import preset
    from dtensor_muon_b200.models.llama import lm_loss
    from dtensor_muon_b200.train import build_llama, build_optimizer

    cfg = preset(args.model, **({"n_layers": args.layers} if args.layers else {}))
    model = build_llama(cfg, torch.device("cuda"), seed=0)
    opt = build_optimizer(model, lr=1e-3)
    ids = torch.randint(0, cfg.vocab_size, (1, cfg.max_seq_len + 1)).cuda()

    def step():
        lm_loss(model(ids[:, :-1]), ids[:, 1:]).backward()
        opt.step()
        opt.zero_grad(set_to_none=True)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    agg: dict[str, list] = {}
    for e in prof.events():
        if e.device_type.name == "CUDA":
            a = agg.setdefault(e.name[:90], [0.0, 0])
            a[0] += e.device_time_total
            a[1] += 1
    tot = sum(t for t, _ in agg.values())
    print(f"total kernel time {tot / 1e3:.1f} ms")
    for k, (t, n) in sorted(agg.items(), key=lambda kv: -kv[1][0])[: args.top]:
        print(f"{t / 1e3:9.2f} ms {100 * t / tot:5.1f}% n={n:5d} {k}")


if __name__ == "__main__":
    main()
