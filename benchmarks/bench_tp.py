"""Config 4: Llama-2-13B-shaped decoder (40 layers, d 5120, 40 heads, SwiGLU
13824, vocab 32000), bf16, on a 2-D mesh FSDP x TP (default dp = world/2,
tp = 2), NorMuon with Newton-Schulz (5 steps), seq 4096, one sequence per dp rank.

    python -m torch.distributed.run --nproc-per-node 8 benchmarks/bench_tp.py [--layers 40] [--tp 2]

Prints training tokens/s (all dp ranks) and optimizer.step() ms, device-timed,
max over ranks. Synthetic uniform tokens, N(0, 0.02) init.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=40)
    ap.add_argument("--tp", type=int, default=2)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    from torch.distributed.device_mesh import init_device_mesh

    from dtensor_muon_b200.models.llama import Llama, lm_loss, preset
    from dtensor_muon_b200.parallel.tensor_parallel import apply_fsdp_tp
    from dtensor_muon_b200.train import build_optimizer

    dp = world // args.tp
    mesh = init_device_mesh("cuda", (dp, args.tp), mesh_dim_names=("dp", "tp"))
    cfg = preset("llama2-13b", n_layers=args.layers, max_seq_len=args.seq)
    with torch.device("meta"):
        model = Llama(cfg).to(torch.bfloat16)
    apply_fsdp_tp(model, mesh)
    model.to_empty(device="cuda")
    torch.manual_seed(mesh.get_local_rank("dp"))
    model.init_weights()
    opt = build_optimizer(model, lr=1e-3, muon_group={"algorithm": "normuon"},
                          orthogonalization_strategy="newton_schulz")
    gen = torch.Generator().manual_seed(mesh.get_local_rank("dp"))

    def step():
        ids = torch.randint(0, cfg.vocab_size, (1, args.seq + 1), generator=gen).cuda()
        loss = lm_loss(model(ids[:, :-1]), ids[:, 1:])
        loss.backward()
        o0, o1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        o0.record()
        opt.step()
        o1.record()
        opt.zero_grad(set_to_none=True)
        return o0, o1

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    evs = [step() for _ in range(args.steps)]
    t1.record()
    torch.cuda.synchronize()
    st = torch.tensor([t0.elapsed_time(t1) / args.steps, sum(a.elapsed_time(b) for a, b in evs) / args.steps],
                      device="cuda")
    dist.all_reduce(st, op=dist.ReduceOp.MAX)
    if rank == 0:
        ms, opt_ms = st.tolist()
        print(json.dumps({"metric": "train tokens/s (FSDPxTP, NorMuon NS-5)", "value": dp * args.seq / (ms / 1e3),
                          "ms_per_step": ms, "optimizer_step_ms": opt_ms, "n_gpus": world, "dp": dp, "tp": args.tp,
                          "layers": args.layers, "dtype": "bf16", "data": "synthetic"}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
