"""Distributed orthogonalisation + update: fused owner-compute (P2P over NVLink)
vs the NCCL DTensor-redistribute path vs one device doing everything.

Workload: 8 x (16, 2048, 1024) dim-0-sharded stacks as in the reference's
benchmark/bench_distributed.py, plus 2-D FSDP-sharded matrices (the shapes that
take the owner-compute path). Launch with
``python -m torch.distributed.run --nproc-per-node N benchmarks/bench_distributed.py``.
Times are CUDA-event device times, max over ranks, median of reps.
"""

from __future__ import annotations

import argparse
import os
import statistics
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def timed(fn, reps=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    t = torch.tensor([statistics.median(ts)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Shard, distribute_tensor

    import dtensor_muon_b200.optim.algorithms.base as algo_base
    from dtensor_muon_b200 import Muon
    from dtensor_muon_b200.orthogonalize import orthogonalize as om

    world = dist.get_world_size()
    mesh = init_device_mesh("cuda", (world,))
    shapes = [(4096, 4096)] * 8 + [(14336, 4096)] * 8 if not args.quick else [(1024, 1024)] * 8
    torch.manual_seed(0)
    fulls = [torch.randn(s, device="cuda") .bfloat16() for s in shapes]
    grads = [torch.randn(s, device="cuda").bfloat16() for s in shapes]
    results = {}

    def make(dist_params):
        ps = [torch.nn.Parameter(distribute_tensor(f.clone(), mesh, [Shard(0)])) if dist_params
              else torch.nn.Parameter(f.clone()) for f in fulls]
        gs = [distribute_tensor(g, mesh, [Shard(0)]) if dist_params else g for g in grads]
        return ps, gs

    for name, dist_params, force_generic in [("fused owner-compute (P2P)", True, False),
                                             ("NCCL DTensor redistribute", True, True),
                                             ("single device (no comm)", False, False)]:
        ps, gs = make(dist_params)
        opt = Muon(ps, foreach=True)
        if force_generic:
            algo_base.foreach_zeropower = lambda g, **k: om.foreach_zeropower(g, **k)

        def step():
            for p, g in zip(ps, gs):
                p.grad = g
            opt.step()

        results[name] = timed(step)
        algo_base.foreach_zeropower = om.foreach_zeropower
    if dist.get_rank() == 0:
        for k, v in results.items():
            print(f"| {k} | W={world} | {v:.3f} ms |")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
