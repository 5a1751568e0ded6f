"""Config 2, distributed: orthogonalisation of dim-0-sharded bf16 inputs across W GPUs.

    python -m torch.distributed.run --nproc-per-node W benchmarks/bench_distributed.py [--impl ours|reference]

Shapes (orthogonalisation microbench): 4096x4096, 4096x14336, 14336x4096 (one matrix each,
its rows sharded over the W ranks: a 2-D ``Shard(0)`` DTensor) and 64 x 1024x1024
(a 3-D ``Shard(0)`` stack: each rank holds 64/W whole matrices). Entries N(0,1),
seed 0, Frobenius-normalised; Newton-Schulz and Polar Express, 5 steps.

``--impl ours`` calls this package's public ``zeropower`` (row-sharded: the
sharded iteration with the all-reduced partial Gram, no gather) and
``foreach_zeropower_3d_fsdp`` (stack: local engine). ``--impl reference`` calls
the same public functions of the unmodified reference (``muonium`` from
baseline/_ref, Triton kernels): its ``zeropower`` gathers the full matrix on
every rank. Timing: CUDA events around each call after warm-up, median of the
reps, max over ranks; an L2 flush (256 MiB write) precedes every timed call.
Every row records the median SM clock sampled during its timed loop.
Roofline: dense FLOPs / (time x W x measured bf16 burst peak), and, for the
row-sharded shapes, the NVLink lower bound of the Gram all-reduces.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from benchmarks.harness import clocks, ortho_flops, peaks  # noqa: E402

SINGLE = [(4096, 4096), (4096, 14336), (14336, 4096)]
STACK = (64, 1024, 1024)
NVLINK_GBS = 770.0  # measured peer copy per direction (pool figure)


def timed(fn, reps: int, warmup: int = 3) -> float:
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(reps):
        flush.zero_()
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
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--reps", type=int, default=10)
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Shard, distribute_tensor

    if args.impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        from install_reference import ensure_reference

        sys.path.insert(0, ensure_reference())
        import torch._dynamo as _dynamo

        _dynamo.config.suppress_errors = True
        from muonium.orthogonalize import foreach_zeropower_3d_fsdp, zeropower

        kw = {"use_triton": True}
    else:
        from dtensor_muon_b200.orthogonalize import foreach_zeropower_3d_fsdp, zeropower

        kw = {}
    mesh = init_device_mesh("cuda", (world,))
    pk = peaks()
    rows = []
    for strategy in ("newton_schulz", "polar_express"):
        for R, C in SINGLE:
            torch.manual_seed(0)
            full = torch.randn(R, C, device="cuda")
            full = (full / full.norm()).bfloat16()
            d = distribute_tensor(full, mesh, [Shard(0)])
            with clocks(local) as ck:
                ms = timed(lambda: zeropower(d, steps=5, strategy=strategy, **kw), args.reps)
            fl = ortho_flops(1, R, C)
            n = min(R, C)
            # sharded iteration: 5 all-reduces of an n x n bf16 Gram + the norm
            comm_ms = 5 * 2 * (world - 1) / world * n * n * 2 / (NVLINK_GBS * 1e9) * 1e3 if world > 1 else 0.0
            rows.append(dict(strategy=strategy, shape=f"{R}x{C} (rows sharded)", ms=ms,
                             frac_of_W_peak=fl / (ms * 1e-3) / (world * pk["bf16_tflops"] * 1e12),
                             nvlink_bound_ms=comm_ms, sm_mhz=(ck.result or {}).get("sm_mhz"),
                             reasons=(ck.result or {}).get("reasons")))
        B, R, C = STACK
        torch.manual_seed(0)
        full = torch.randn(B, R, C, device="cuda")
        full = (full / full.norm(dim=(-2, -1), keepdim=True)).bfloat16()
        ds = [distribute_tensor(full, mesh, [Shard(0)])]
        with clocks(local) as ck:
            ms = timed(lambda: foreach_zeropower_3d_fsdp(ds, steps=5, strategy=strategy, **kw), args.reps)
        fl = ortho_flops(B, R, C)
        rows.append(dict(strategy=strategy, shape=f"{B}x{R}x{C} (stack sharded)", ms=ms,
                         frac_of_W_peak=fl / (ms * 1e-3) / (world * pk["bf16_tflops"] * 1e12),
                         nvlink_bound_ms=0.0, sm_mhz=(ck.result or {}).get("sm_mhz"),
                         reasons=(ck.result or {}).get("reasons")))
    if rank == 0:
        for r in rows:
            print(json.dumps({"impl": args.impl, "world": world, **r}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
