"""FSDP collectives in isolation and under a concurrent GEMM: our schemes vs NCCL.

    python -m torch.distributed.run --nproc-per-node W benchmarks/bench_fsdp_comm.py

For a Llama-3-8B decoder layer (218 M bf16 parameters: all-gather output and
reduce-scatter input of 436 MB) every scheme is timed (CUDA events, median,
max over ranks) twice: alone, and while a bf16 GEMM loop runs on a second stream
(the situation inside FSDP, where the collective overlaps the neighbouring
layer's compute). The second number reports the collective's time and the
GEMM loop's slowdown, i.e. the SMs and memory bandwidth the collective takes.
"""

from __future__ import annotations

import json
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
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    from dtensor_muon_b200.parallel import fsdp_comm

    group = dist.group.WORLD
    numel = 218 * (1 << 20) // world * world
    shard = torch.randn(numel // world, device="cuda").bfloat16()
    full = torch.empty(numel, device="cuda", dtype=torch.bfloat16)
    rs_in = torch.randn(numel, device="cuda").bfloat16()
    rs_out = torch.empty(numel // world, device="cuda", dtype=torch.bfloat16)
    a = torch.randn(8192, 8192, device="cuda").bfloat16()
    b = torch.randn(8192, 8192, device="cuda").bfloat16()
    side = torch.cuda.Stream()

    def gemm_loop(n=6):
        for _ in range(n):
            torch.mm(a, b)

    def with_gemm(fn):
        """collective on the current stream while the GEMM loop runs on `side`;
        returns (collective ms, GEMM loop ms)."""
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            ev0.record()
            gemm_loop()
            ev1.record()
        c0.record()
        fn()
        c1.record()
        torch.cuda.synchronize()
        return c0.elapsed_time(c1), ev0.elapsed_time(ev1)

    def overlapped(fn, reps=8):
        for _ in range(3):
            with_gemm(fn)
        dist.barrier()
        res = [with_gemm(fn) for _ in range(reps)]
        t = torch.tensor([statistics.median(r[0] for r in res), statistics.median(r[1] for r in res)],
                         device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    gemm_alone = timed(gemm_loop)
    ag, rs = fsdp_comm.P2PAllGather(), fsdp_comm.P2PReduceScatter()
    cases = []
    for mode in ("nccl", "ce", "pull", "push"):
        def run_ag(mode=mode):
            if mode == "nccl":
                dist.all_gather_into_tensor(full, shard, group=group)
            else:
                fsdp_comm.AG_MODE = mode
                ag(full, shard, group)

        cases.append((f"all-gather {mode}", run_ag))
    for mode in ("nccl", "nvls", "ce", "push"):
        def run_rs(mode=mode):
            if mode == "nccl":
                dist.reduce_scatter_tensor(rs_out, rs_in, op=dist.ReduceOp.AVG, group=group)
            else:
                fsdp_comm.RS_MODE = mode
                rs(rs_out, rs_in, group, dist.ReduceOp.AVG)

        cases.append((f"reduce-scatter {mode}", run_rs))
    for ctas in (16, 32, 64):
        def run_pull(ctas=ctas):
            fsdp_comm.AG_MODE = "pull"
            fsdp_comm.COMM_CTAS = ctas
            ag(full, shard, group)

        cases.append((f"all-gather pull {ctas} CTAs", run_pull))
    fsdp_comm.COMM_CTAS = 64
    out = []
    for name, fn in cases:
        alone = timed(fn)
        coll, gemm = overlapped(fn)
        out.append({"case": name, "world": world, "alone_ms": alone,
                    "GB_per_s_per_rank": numel * 2 * (world - 1) / world / (alone * 1e-3) / 1e9,
                    "overlapped_ms": coll, "gemm_loop_ms": gemm, "gemm_alone_ms": gemm_alone})
    if rank == 0:
        for r in out:
            print(json.dumps(r))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
