"""Config 4: Llama-2-13B-shaped decoder (40 layers, d 5120, 40 heads, SwiGLU
13824, vocab 32000), bf16, on a 2-D mesh FSDP x TP (default dp = world/2,
tp = 2), NorMuon with Newton-Schulz (5 steps), seq 4096, one sequence per dp rank.

    python -m torch.distributed.run --nproc-per-node 8 benchmarks/bench_tp.py [--layers 40] [--tp 2]
        [--impl ours|reference]

Prints training tokens/s (all dp ranks) and optimizer.step() ms, device-timed,
max over ranks. Synthetic uniform tokens, N(0, 0.02) init.

``--impl reference`` runs the unmodified reference optimizer (``muonium``'s
NorMuon from baseline/_ref, its own DTensor gather path for TP shards) on the
stock Hugging Face ``LlamaForCausalLM`` of the same shape, TP-parallelised with
torch's ``parallelize_module`` (q/k/v/gate/up column-wise, o/down row-wise) and
FSDP2 over dp, with the same data and timing.
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
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
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
    if args.impl == "reference":
        try:
            model, opt, fwd_loss = build_reference(cfg, mesh, args)
        except Exception as exc:  # report, do not hang the job
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"[:300]}))
            dist.destroy_process_group()
            return
    else:
        with torch.device("meta"):
            model = Llama(cfg).to(torch.bfloat16)
        apply_fsdp_tp(model, mesh)
        model.to_empty(device="cuda")
        torch.manual_seed(mesh.get_local_rank("dp"))
        model.init_weights()
        opt = build_optimizer(model, lr=1e-3, muon_group={"algorithm": "normuon"},
                              orthogonalization_strategy="newton_schulz")

        def fwd_loss(ids):
            return lm_loss(model(ids[:, :-1]), ids[:, 1:])

    gen = torch.Generator().manual_seed(mesh.get_local_rank("dp"))

    def step():
        ids = torch.randint(0, cfg.vocab_size, (1, args.seq + 1), generator=gen).cuda()
        loss = fwd_loss(ids)
        loss.backward()
        o0, o1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        o0.record()
        opt.step()
        o1.record()
        opt.zero_grad(set_to_none=True)
        return o0, o1

    try:
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
    except Exception as exc:  # the reference's own step failed on this config: report it
        if args.impl != "reference":
            raise
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"[:400]}), flush=True)
        os._exit(0)  # peers may be inside a collective
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
                          "layers": args.layers, "dtype": "bf16", "data": "synthetic", "impl": args.impl}))
    dist.destroy_process_group()


def build_reference(cfg, mesh, args):
    """Stock HF Llama (TP plan + FSDP2) with the reference's NorMuon; see the module docstring."""
    import torch.nn.functional as F
    from torch.distributed.fsdp import fully_shard
    from torch.distributed.tensor.parallel import ColwiseParallel, RowwiseParallel, parallelize_module
    from transformers import LlamaConfig, LlamaForCausalLM

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "baseline"))
    from install_reference import ensure_reference

    sys.path.insert(0, ensure_reference())
    import torch._dynamo as _dynamo

    _dynamo.config.suppress_errors = True  # reference pins torch 2.12; see bench.py
    from muonium import Muon as RefMuon

    hf_cfg = LlamaConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.dim, intermediate_size=cfg.ffn_dim,
                         num_hidden_layers=cfg.n_layers, num_attention_heads=cfg.n_heads,
                         num_key_value_heads=cfg.n_kv_heads, rope_theta=cfg.rope_theta,
                         max_position_embeddings=args.seq, rms_norm_eps=1e-5, tie_word_embeddings=False)
    hf_cfg._attn_implementation = "sdpa"
    with torch.device("meta"):
        model = LlamaForCausalLM(hf_cfg).to(torch.bfloat16)
    plan = {"self_attn.q_proj": ColwiseParallel(), "self_attn.k_proj": ColwiseParallel(),
            "self_attn.v_proj": ColwiseParallel(), "self_attn.o_proj": RowwiseParallel(),
            "mlp.gate_proj": ColwiseParallel(), "mlp.up_proj": ColwiseParallel(), "mlp.down_proj": RowwiseParallel()}
    for layer in model.model.layers:
        parallelize_module(layer, mesh["tp"], plan)
        fully_shard(layer, mesh=mesh["dp"])
    fully_shard(model, mesh=mesh["dp"])
    model.to_empty(device="cuda")
    torch.manual_seed(mesh.get_local_rank("dp"))
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
        (muon if "layers." in name and p.ndim >= 2 else adam).append(p)
    opt = RefMuon([{"params": muon, "algorithm": "normuon"}, {"params": adam, "algorithm": "adamw"}], lr=1e-3,
                  wd=0.1, orthogonalization_strategy="newton_schulz", batch_size=32)

    def fwd_loss(ids):
        logits = model(input_ids=ids[:, :-1]).logits
        return F.cross_entropy(logits.float().reshape(-1, logits.size(-1)), ids[:, 1:].reshape(-1))

    return model, opt, fwd_loss


if __name__ == "__main__":
    main()
