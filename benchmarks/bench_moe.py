"""Config 5: Mixtral-shaped MoE (8 experts, SwiGLU 14336, d 4096, 32 heads / 8 KV,
vocab 32000, seq 4096) with expert parallelism EP = world size, top-2
dispatch/combine (P2P over NVLink or NCCL all-to-all) and MuonLP quantised
momentum (fp8 by default; --opt muon8bit / muon4bit / muon / muonlp).

    python -m torch.distributed.run --nproc-per-node 8 benchmarks/bench_moe.py [--layers 32]

Expert weights are stacked [E, F, D] DTensors sharded on dim 0 (one expert per
rank at EP=8): the optimizer orthogonalises each local expert matrix with no
communication. Dense weights are replicated and their grads averaged. Prints
tokens/s (all ranks), optimizer.step() ms, device-timed, max over ranks.

``--impl reference`` runs the unmodified reference's base ``MuonLP`` (fp32 state,
``foreach=False``: the only MuonLP the reference can step) on the stock Hugging
Face ``MixtralForCausalLM`` of the same shape, FSDP2 over all ranks. The
reference has no token exchange: its MoE story is FSDP-sharded 3-D expert stacks
(``gate_up_proj`` [E, 2F, D], ``down_proj`` [E, D, F] in HF), which its optimizer
orthogonalises locally (the 3-D dim-0 fast path), while FSDP all-gathers the
experts for compute. Same data, seq and timing.
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
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
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
    if args.impl == "reference":
        return run_reference(cfg, mesh, args, world, rank)
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


def run_reference(cfg, mesh, args, world, rank):
    import torch.nn.functional as F
    from torch.distributed.fsdp import fully_shard

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    try:
        sys.path.insert(0, os.path.join(root, "baseline"))
        from install_reference import ensure_reference

        sys.path.insert(0, ensure_reference())
        import torch._dynamo as _dynamo

        _dynamo.config.suppress_errors = True  # reference pins torch 2.12; see bench.py
        try:
            from muonium import MuonLP

            opt_name = "muonium.MuonLP (fp32 state, foreach=False)"
        except ImportError:
            # The reference's MuonLP module imports torchao at load time (not installable
            # here). Its base class adds nothing to Muon but foreach=False and fp32 buffers,
            # which muonium.Muon(foreach=False) is.
            from muonium import Muon as _RefMuon

            def MuonLP(groups, **kw):  # noqa: N802
                return _RefMuon(groups, foreach=False, **kw)

            opt_name = "muonium.Muon(foreach=False): the base MuonLP's math (MuonLP needs torchao)"
        from transformers import MixtralConfig, MixtralForCausalLM

        hf = MixtralConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.dim, intermediate_size=cfg.ffn_dim,
                           num_hidden_layers=cfg.n_layers, num_attention_heads=cfg.n_heads,
                           num_key_value_heads=cfg.n_kv_heads, num_local_experts=cfg.n_experts,
                           num_experts_per_tok=cfg.top_k, rope_theta=cfg.rope_theta,
                           max_position_embeddings=args.seq, tie_word_embeddings=False)
        hf._attn_implementation = "sdpa"
        with torch.device("meta"):
            model = MixtralForCausalLM(hf).to(torch.bfloat16)
        for layer in model.model.layers:
            fully_shard(layer, mesh=mesh)
        fully_shard(model, mesh=mesh)
        model.to_empty(device="cuda")
        torch.manual_seed(0)
        with torch.no_grad():
            for name, p in model.named_parameters():
                local = p.to_local() if hasattr(p, "to_local") else p
                local.fill_(1.0) if "norm" in name else local.normal_(0.0, 0.02)
            for name, b in model.named_buffers():
                if "inv_freq" in name:
                    dim = b.numel() * 2
                    b.copy_(1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, device="cuda").float() / dim)))
        muon, adam = [], []
        for name, p in model.named_parameters():
            (muon if "layers." in name and p.ndim >= 2 and "mlp.gate." not in name else adam).append(p)
        opt = MuonLP([{"params": muon}, {"params": adam, "algorithm": "adamw"}], lr=1e-3, wd=0.1)
    except Exception as exc:  # report, do not hang the job
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"[:300]}))
        dist.destroy_process_group()
        return
    gen = torch.Generator().manual_seed(rank)

    def step():
        ids = torch.randint(0, cfg.vocab_size, (1, args.seq + 1), generator=gen).cuda()
        logits = model(input_ids=ids[:, :-1]).logits
        loss = F.cross_entropy(logits.float().reshape(-1, logits.size(-1)), ids[:, 1:].reshape(-1))
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
        print(json.dumps({"metric": "MoE train tokens/s", "impl": "reference", "value": world * args.seq / (ms / 1e3),
                          "ms_per_step": ms, "optimizer_step_ms": opt_ms, "n_gpus": world, "layers": args.layers,
                          "opt": opt_name, "parallelism": f"fsdp{world}",
                          "dtype": "bf16", "data": "synthetic"}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
