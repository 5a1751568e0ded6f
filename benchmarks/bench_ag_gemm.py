"""Parameter all-gather fused into the first forward GEMM vs all-gather + cuBLAS.

    python benchmarks/bench_ag_gemm.py                                  # 1 GPU: GEMM engine vs cuBLAS
    python -m torch.distributed.run --nproc-per-node W benchmarks/bench_ag_gemm.py

Shapes are the Llama-3-8B first forward GEMMs of a decoder layer at seq 4096,
micro-batch 1: the fused q/k/v projection (W [6144, 4096]) and the fused
gate/up projection (W [28672, 4096]), W row-sharded over the W ranks as FSDP
shards it. Arms (CUDA events, median of 10 after 3 warm-ups, L2 flushed between
repetitions, max over ranks):

* ``fused``: ``ops/csrc/ag_gemm.cu`` (gather of the peers' shards over NVLink
  inside the tcgen05 GEMM kernel);
* ``nccl+cublas``: ``all_gather_into_tensor`` then ``torch.matmul``;
* ``cublas``: the GEMM alone on a pre-gathered W (lower bound for any AG + GEMM).

Roofline for the fused kernel: max(FLOPs / measured bf16 peak, remote bytes /
770 GB/s peer copy bandwidth per direction).
"""

from __future__ import annotations

import json
import os
import statistics
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from benchmarks.harness import clocks, peaks  # noqa: E402

PEER_GBS = 770.0
SHAPES = {"qkv": (6144, 4096), "gate_up": (28672, 4096)}


def timed(fn, reps=10, warmup=3, distributed=False):
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if distributed:
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
    t = statistics.median(ts)
    if distributed:
        v = torch.tensor([t], device="cuda")
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        t = v.item()
    return t


def main():
    distributed = "RANK" in os.environ
    if distributed:
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        world, rank, group = dist.get_world_size(), dist.get_rank(), dist.group.WORLD
    else:
        world, rank, group = 1, 0, None
    from dtensor_muon_b200.parallel.ag_gemm import AllGatherGemm

    dev = torch.device("cuda", torch.cuda.current_device())
    pk = peaks()
    eng = AllGatherGemm(group, dev)
    tokens = int(os.environ.get("AG_TOKENS", "4096"))
    g = torch.Generator(device=dev).manual_seed(rank)
    rows = []
    with clocks(dev.index) as clk:
        for name, (n, k) in SHAPES.items():
            x = torch.randn(tokens, k, device=dev, generator=g).bfloat16()
            shard = (0.02 * torch.randn(n // world, k, device=dev, generator=g)).bfloat16()
            wg = torch.empty(n, k, device=dev, dtype=torch.bfloat16)
            out = torch.empty(tokens, n, device=dev, dtype=torch.bfloat16)
            t_fused = timed(lambda: eng(x, shard, wg, out), distributed=distributed)
            eng.check()
            ref = x @ wg.t()
            err = ((out.float() - ref.float()).abs().max() / ref.float().abs().max()).item()

            def unfused():
                if distributed:
                    dist.all_gather_into_tensor(wg, shard, group=group)
                else:
                    wg.copy_(shard)
                torch.matmul(x, wg.t(), out=out)

            t_unfused = timed(unfused, distributed=distributed)
            t_gemm = timed(lambda: torch.matmul(x, wg.t(), out=out), distributed=distributed)
            flops = 2.0 * tokens * n * k
            remote = (world - 1) / world * n * k * 2
            t_roof = max(flops / (pk["bf16_tflops"] * 1e9), remote / (PEER_GBS * 1e6))
            rows.append({
                "shape": name, "M": tokens, "N": n, "K": k, "world": world,
                "fused_ms": round(t_fused, 4), "nccl_cublas_ms": round(t_unfused, 4),
                "cublas_gemm_only_ms": round(t_gemm, 4),
                "fused_tflops": round(flops / t_fused / 1e9, 1),
                "roofline_ms": round(t_roof, 4), "fused_frac_of_roofline": round(t_roof / t_fused, 3),
                "max_rel_err_vs_cublas": err,
            })
    if rank == 0:
        for r in rows:
            r["clocks"] = clk.result
            r["peaks_source"] = pk["source"]
            print(json.dumps(r))
    if distributed:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
