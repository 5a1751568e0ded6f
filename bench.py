"""Headline benchmark: Llama-3-8B-shaped training with Muon (+AdamW), FSDP2 for N > 1.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch one process per GPU with torch.distributed.run (rendezvous on
127.0.0.1). Rank 0 prints one JSON line. The metric is training tokens/s over
all GPUs (synthetic uniform token ids, random N(0, 0.02) init, bf16 params,
fp32 Muon momentum), device-timed with CUDA events over exactly K steps after
W warm-up steps, max over ranks. The mean optimizer.step() time is reported
alongside. Every step streams the 16 GB of bf16 weights (plus grads and
optimizer state), far more than the 126 MB L2, so no explicit L2 flush is
needed between steps.

``--impl reference`` runs the unmodified reference optimizer (``muonium``
installed under baseline/_ref) on the stock Hugging Face Llama model through
their public APIs, with the same shapes, data and timing.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
BASELINE_VALUE = None  # the reference publishes no B200 tokens/s for this config
METRIC = "Muon optimizer.step() ms and train tokens/s, Llama-8B FSDP at 1/2/4/8 B200"


# ----------------------------------------------------------------- clocks --
class ClockSampler:
    """Samples SM clocks / throttle reasons with nvidia-smi while running."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
        "clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"],
                stdout=open(self.path, "w"),
                stderr=subprocess.DEVNULL,
            )
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        with open(self.path) as f:
            lines = f.readlines()
        os.unlink(self.path)
        return self.summarize(lines)

    @staticmethod
    def summarize(lines: list[str]) -> dict:
        """Median SM clock under load, max clock and the throttle reasons seen, from
        ``nvidia-smi --format=csv,noheader,nounits`` lines of FIELDS. Tolerates
        ``[N/A]`` fields and partial lines."""

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        rows = [[x.strip() for x in line.split(",")] for line in lines]
        rows = [r for r in rows if len(r) >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        mhz = [v for v in (num(r[1]) for r in rows) if v is not None]
        maxes = [v for v in (num(r[2]) for r in rows) if v is not None]
        max_mhz = max(maxes) if maxes else None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].lower().startswith("active")})
        loaded = ([m for m in mhz if m > 0.5 * max_mhz] if max_mhz else []) or mhz
        return {
            "sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": max_mhz,
            "reasons": reasons,
            "samples": len(rows),
        }


# ------------------------------------------------------------------ setup --
def init_dist(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(minutes=5))
    return rank, world, local


def hidden_and_rest(model):
    muon, adam = [], []
    for name, p in model.named_parameters():
        if "layers." in name and p.ndim >= 2 and "router" not in name and "gate." not in name:
            muon.append(p)
        else:
            adam.append(p)
    return muon, adam


def build_ours(args, world, device):
    sys.path.insert(0, HERE)
    from dtensor_muon_b200.models import preset
    from dtensor_muon_b200.optim import Muon
    from dtensor_muon_b200.train import build_llama, build_optimizer

    cfg = preset(args.model, max_seq_len=args.seq, **({"n_layers": args.layers} if args.layers else {}))
    mesh = None
    if world > 1:
        from torch.distributed.device_mesh import init_device_mesh

        mesh = init_device_mesh("cuda", (world,))
    model = build_llama(cfg, device, mesh=mesh, seed=0, fsdp_comm=args.fsdp_comm,
                        fused_gather={0: False, 1: True, 2: "all"}[args.fused_gather] if world > 1 else False)
    opt = build_optimizer(model, Muon, lr=args.lr, wd=0.1, orthogonalization_strategy=args.strategy,
                          fuse_momentum=world > 1 and args.fsdp_comm == "p2p" and args.fuse_momentum)
    from dtensor_muon_b200.models.llama import lm_loss

    def step(tokens, targets):
        loss = lm_loss(model(tokens), targets)
        loss.backward()
        return loss.detach()

    return cfg.vocab_size, model, opt, step


def build_reference(args, world, device):
    sys.path.insert(0, os.path.join(HERE, "baseline"))
    from install_reference import ensure_reference

    ref_root = ensure_reference()  # baseline/_ref, installed on demand from the reference source
    sys.path.insert(0, ref_root)
    # The reference pins torch 2.12.1; on this image's torch 2.11 Dynamo asserts
    # while tracing DTensor.stride() inside its compiled Muon update (FSDP runs).
    # Frames that fail to compile run eagerly; everything else stays compiled.
    import torch._dynamo

    torch._dynamo.config.suppress_errors = True
    import muonium  # noqa: F401
    import torch.nn.functional as F
    from muonium import Muon as RefMuon
    from transformers import LlamaConfig, LlamaForCausalLM

    shapes = {
        "llama3-8b": dict(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                          num_attention_heads=32, num_key_value_heads=8, rope_theta=500000.0),
        "tiny": dict(vocab_size=1024, hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=4, rope_theta=10000.0),
    }[args.model]
    hf_cfg = LlamaConfig(max_position_embeddings=args.seq, rms_norm_eps=1e-5, tie_word_embeddings=False,
                         attention_bias=False, mlp_bias=False, **shapes)
    hf_cfg._attn_implementation = "sdpa"
    with torch.device("meta"):
        model = LlamaForCausalLM(hf_cfg).to(torch.bfloat16)
    if world > 1:
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.fsdp import fully_shard

        mesh = init_device_mesh("cuda", (world,))
        for layer in model.model.layers:
            fully_shard(layer, mesh=mesh)
        fully_shard(model, mesh=mesh)
    model.to_empty(device=device)
    torch.manual_seed(0 + (dist.get_rank() if dist.is_initialized() else 0))
    with torch.no_grad():
        for name, p in model.named_parameters():
            local = p.to_local() if hasattr(p, "to_local") else p
            if "norm" in name:
                local.fill_(1.0)
            else:
                local.normal_(0.0, 0.02)
        for name, b in model.named_buffers():
            if "inv_freq" in name:
                dim = b.numel() * 2
                b.copy_(1.0 / (shapes["rope_theta"] ** (torch.arange(0, dim, 2, device=device).float() / dim)))
    muon_p, adam_p = hidden_and_rest(model)
    # batch_size=32: the reference's Triton gram_nd computes the batch offset
    # pid_b * stride_xb in 32-bit; one stacked batch of all 64 gate/up matrices
    # (64 x 4096 x 14336 > 2**31 elements) overflows it and faults. 32 matrices
    # per batch stay below 2**31 elements for every Llama-3-8B shape group.
    opt = RefMuon([{"params": muon_p}, {"params": adam_p, "algorithm": "adamw"}], lr=args.lr, wd=0.1,
                  orthogonalization_strategy=args.strategy, batch_size=args.ref_batch_size)

    def step(tokens, targets):
        logits = model(input_ids=tokens).logits
        loss = F.cross_entropy(logits.float().reshape(-1, logits.size(-1)), targets.reshape(-1))
        loss.backward()
        return loss.detach()

    return shapes["vocab_size"], model, opt, step


# ------------------------------------------------------------------- main --
def main():
    args = parse_args()
    if args.impl != "reference":
        return run(args)
    try:
        return run(args)
    except Exception as exc:  # the reference failed after it was built: report, do not hang the job
        rank = int(os.environ.get("RANK", "0"))
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"[:300]}), flush=True)
        if dist.is_initialized():
            os._exit(0)  # peers may be blocked in a collective; leave without a teardown barrier


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--mb", type=int, default=1, help="micro-batch (sequences) per GPU")
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--strategy", default="polar_express")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="diagnostics only: override the layer count")
    ap.add_argument("--fuse-momentum", type=int, default=int(os.environ.get("DMB_FUSE_MOMENTUM", "0")),
                    help="ours, N > 1: Muon momentum update inside the FSDP gradient reduce-scatter")
    ap.add_argument("--fsdp-comm", default=os.environ.get("DMB_FSDP_COMM", "p2p"), choices=["p2p", "nccl"],
                    help="ours: FSDP collectives on NVLink P2P kernels or NCCL")
    ap.add_argument("--fused-gather", type=int, default=int(os.environ.get("DMB_FUSED_GATHER", "1")),
                    help="ours, N > 1: q/k/v and gate/up weights gathered inside their forward GEMM "
                         "(0: every weight through FSDP2's all-gather; 2: wo and w2 too)")
    ap.add_argument("--ref-batch-size", type=int, default=32,
                    help="reference arm: Muon foreach batch_size (keeps its Gram kernel below 2**31 elements)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    return args


def run(args):
    rank, world, local = init_dist(args.gpus)
    device = torch.device("cuda", local)
    par = f"fsdp{world}" if world > 1 else "single"
    base = {
        "metric": METRIC,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "dtype": "bf16",
        "data": "synthetic",
        "higher_is_better": True,
        "scaling": "weak",
        "unit": "tokens/s",
    }
    if args.impl == "reference":
        base["impl"] = "reference"
    try:
        vocab, model, opt, fwd_bwd = (build_reference if args.impl == "reference" else build_ours)(args, world, device)
    except Exception as exc:  # reference not installable / not runnable here
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"[:300]}))
            return
        raise

    launches = None
    if args.impl == "ours":
        from dtensor_muon_b200.ops import _ext

        launches = _ext

    gen = torch.Generator().manual_seed(1234 + rank)
    tok_per_step = args.mb * args.seq * world

    def make_inputs():
        ids = torch.randint(0, vocab, (args.mb, args.seq + 1), generator=gen)
        return ids[:, :-1].contiguous().to(device), ids[:, 1:].contiguous().to(device)

    # Device-resident inputs for the kernel-timed loop (one fresh batch per step).
    batches = [make_inputs() for _ in range(args.steps + args.warmup)]

    def train_step(tokens, targets):
        loss = fwd_bwd(tokens, targets)
        o0 = torch.cuda.Event(enable_timing=True)
        o1 = torch.cuda.Event(enable_timing=True)
        o0.record()
        opt.step()
        o1.record()
        opt.zero_grad(set_to_none=True)
        return loss, (o0, o1)

    for i in range(args.warmup):
        train_step(*batches[i])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    n0 = launches.launch_count if launches else 0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    opt_events = []
    for i in range(args.steps):
        _, ev = train_step(*batches[args.warmup + i])
        opt_events.append(ev)
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    n1 = launches.launch_count if launches else 0
    clocks = sampler.stop() if sampler else None
    ms_total = t0.elapsed_time(t1)
    opt_ms = sum(a.elapsed_time(b) for a, b in opt_events) / args.steps
    stats = torch.tensor([ms_total, opt_ms], device=device)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms_total, opt_ms = stats.tolist()
    ms_step = ms_total / args.steps
    value = tok_per_step / (ms_step / 1e3)

    # End-to-end through the public step API: pinned host tokens -> device each
    # step, loss read back to the host each step, wall clock.
    e2e = None
    if not args.no_e2e:
        host = []
        for _ in range(args.steps):
            ids = torch.randint(0, vocab, (args.mb, args.seq + 1), generator=gen).pin_memory()
            host.append(ids)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        for ids in host:
            dev = ids.to(device, non_blocking=True)
            loss, _ = train_step(dev[:, :-1], dev[:, 1:])
            float(loss.item())
        torch.cuda.synchronize()
        w1 = time.perf_counter()
        wt = torch.tensor([w1 - w0], device=device)
        if world > 1:
            dist.all_reduce(wt, op=dist.ReduceOp.MAX)
        e2e = {
            "value": tok_per_step * args.steps / wt.item(),
            "unit": "tokens/s",
            "h2d_bytes_per_step": args.mb * (args.seq + 1) * 8,
            "d2h_bytes_per_step": 4,
        }

    if rank == 0:
        out = dict(base)
        out.update(
            value=value,
            ms_per_step=ms_step,
            optimizer_step_ms=opt_ms,
            vs_baseline=(value / BASELINE_VALUE) if BASELINE_VALUE else None,
            config={
                "model": args.model,
                "global_batch": args.mb * world,
                "seq_len": args.seq,
                "parallelism": par,
                "optimizer": f"Muon({args.strategy}, ns_steps=5) + AdamW(embed/norms/head)",
                "l2": "no flush: every step streams >16 GB of weights/grads/state (inputs far larger than L2)",
                **({"collectives": ("q/k/v + gate/up: all-gather fused into the forward GEMM"
                                    + (" (+ wo, w2)" if args.fused_gather == 2 else "")
                                    if args.fused_gather else "FSDP2 all-gather") + f"; FSDP2 comm {args.fsdp_comm}"}
                   if world > 1 and args.impl == "ours" else {}),
            },
            clocks=clocks,
            e2e=e2e,
            gpu_launches=(n1 - n0) if launches else 0,
        )
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
