"""Config 5: Mixtral-shaped MoE (8 experts, SwiGLU 14336, d 4096, 32 heads / 8 KV,
vocab 32000, seq 4096) with expert parallelism EP = world size, top-2
dispatch/combine (P2P over NVLink or NCCL all-to-all) and MuonLP quantised
momentum (fp8 by default; --opt muon8bit / muon4bit / muon / muonlp).

    python -m torch.distributed.run --nproc-per-node 8 benchmarks/bench_moe.py [--layers 32]

Expert weights are stacked [E, F, D] DTensors sharded on dim 0 (one expert per
rank at EP=8): the optimizer orthogonalises each local expert matrix with no
communication. Dense weights are replicated and their grads averaged. Prints
tokens/s (all ranks), optimizer.step() ms, device-timed, max over ranks.
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
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--opt", default="muonfp8", choices=["muon", "muonlp", "muon8bit", "muon4bit", "muonfp8"])
    ap.add_argument("--ep-backend", default="p2p", choices=["p2p", "nccl"])
    ap.add_argument("--preset", default="mixtral-8x7b")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    from torch.distributed.device_mesh import init_device_mesh

    import dtensor_muon_b200 as dmb
    from dtensor_muon_b200.models.llama import lm_loss
    from dtensor_muon_b200.models.mixtral import Mixtral, mixtral_preset
    from dtensor_muon_b200.parallel.expert_parallel import ExpertParallel, reduce_dense_grads, shard_experts
    from dtensor_muon_b200.train import build_optimizer

    cfg = mixtral_preset(args.preset, n_layers=args.layers, max_seq_len=args.seq)
    mesh = init_device_mesh("cuda", (world,))
    ep = ExpertParallel(mesh.get_group(), cfg.n_experts, backend=args.ep_backend)
    with torch.device("meta"):
        model = Mixtral(cfg).to(torch.bfloat16)
    model.to_empty(device="cuda")
    torch.manual_seed(0)  # identical dense weights on every rank
    model.init_weights()
    experts = shard_experts(model, mesh, ep)
    cls = {"muon": dmb.Muon, "muonlp": dmb.MuonLP, "muon8bit": dmb.Muon8bit, "muon4bit": dmb.Muon4bit,
           "muonfp8": dmb.MuonFp8}[args.opt]
    opt = build_optimizer(model, cls, lr=1e-3) if cls is dmb.Muon else build_optimizer(model, cls, lr=1e-3, foreach=True)
    gen = torch.Generator().manual_seed(rank)

    def step():
        ids = torch.randint(0, cfg.vocab_size, (1, args.seq + 1), generator=gen).cuda()
        loss = lm_loss(model(ids[:, :-1]), ids[:, 1:])
        loss.backward()
        reduce_dense_grads(list(model.parameters()), mesh.get_group(), experts)
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
        print(json.dumps({"metric": "MoE train tokens/s", "value": world * args.seq / (ms / 1e3), "ms_per_step": ms,
                          "optimizer_step_ms": opt_ms, "n_gpus": world, "layers": args.layers, "opt": args.opt,
                          "ep_backend": args.ep_backend, "dtype": "bf16", "data": "synthetic"}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
