"""Parameter all-gather fused into the forward GEMM (``ops/csrc/ag_gemm.cu``)
against a plain PyTorch fp32 ``x @ W^T`` of the gathered weight."""

import pytest
import torch

from testkit import assert_close, run_distributed

pytestmark = pytest.mark.gpu


def _check(y, wg, x, w_full):
    assert torch.equal(wg, w_full), "gathered weight differs from the concatenated shards"
    ref = x.float() @ w_full.float().t()
    assert_close(y.float(), ref, rtol=2e-2, atol=2e-2, max_mismatch_pct=0.1)


@pytest.mark.parametrize("m,n,k", [(256, 256, 64), (512, 768, 512), (1024, 2048, 1024)])
def test_ag_gemm_single_rank_matches_fp32(m, n, k):
    from dtensor_muon_b200.ops import _ext
    from dtensor_muon_b200.parallel.ag_gemm import AllGatherGemm

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(m + n + k)
    eng = AllGatherGemm(None, dev)
    for it in range(3):  # both counter parities, then the first again
        x = torch.randn(m, k, generator=g).to(dev, torch.bfloat16)
        w = (0.05 * torch.randn(n, k, generator=g)).to(dev, torch.bfloat16)
        (y,), wg = eng(x, w)
        torch.cuda.synchronize()
        _ext.check_device_errors(dev)
        _check(y, wg, x, w)


def test_ag_gemm_few_pairs():
    """With one CTA pair the single pair must both gather and compute every tile."""
    from dtensor_muon_b200.parallel.ag_gemm import AllGatherGemm

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(512, 256, generator=g).to(dev, torch.bfloat16)
    w = torch.randn(1024, 256, generator=g).to(dev, torch.bfloat16)
    (y,), wg = AllGatherGemm(None, dev)(x, w, max_pairs=1)
    torch.cuda.synchronize()
    _check(y, wg, x, w)


def test_ag_gemm_segments_single_rank():
    """q/k/v-like segments of different heights in one call, each to its own output."""
    from dtensor_muon_b200.parallel.ag_gemm import AllGatherGemm

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(3)
    eng = AllGatherGemm(None, dev)
    x = torch.randn(512, 512, generator=g).to(dev, torch.bfloat16)
    ws = [(0.05 * torch.randn(n, 512, generator=g)).to(dev, torch.bfloat16) for n in (1024, 256, 256)]
    outs, wg = eng(x, ws)
    torch.cuda.synchronize()
    _check(outs[0], wg[:1024], x, ws[0])
    _check(outs[1], wg[1024:1280], x, ws[1])
    _check(outs[2], wg[1280:], x, ws[2])


def _dist_worker(rank, world):
    import torch.distributed as dist

    from dtensor_muon_b200.ops import _ext
    from dtensor_muon_b200.parallel.ag_gemm import AllGatherGemm, all_gather_linear

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    group = dist.group.WORLD
    eng = AllGatherGemm(group, dev)
    g = torch.Generator().manual_seed(7)
    # two shapes interleaved (slot capacity grows between them), several calls each
    for m, n, k in [(512, 512 * world, 256), (1024, 768 * world, 512), (512, 512 * world, 256),
                    (1024, 768 * world, 512), (256, 256 * world, 1024)]:
        x_all = torch.randn(world, m, k, generator=g).to(torch.bfloat16)
        w_full = (0.05 * torch.randn(n, k, generator=g)).to(torch.bfloat16)
        x = x_all[rank].to(dev)
        shard = w_full.chunk(world)[rank].to(dev)
        (y,), wg = eng(x, shard)
        torch.cuda.synchronize()
        _ext.check_device_errors(dev)
        _check(y, wg, x, w_full.to(dev))

    # segments whose shards are 128 rows (k/v at 8 ranks look like this)
    m, k = 512, 256
    rows = (512 * world // 2, 128 * world, 128 * world)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    fulls = [(0.05 * torch.randn(n, k, generator=g)).to(torch.bfloat16) for n in rows]
    outs, wg = eng(x.to(dev), [f.chunk(world)[rank].to(dev) for f in fulls])
    torch.cuda.synchronize()
    _ext.check_device_errors(dev)
    r0 = 0
    for o, f in zip(outs, fulls):
        _check(o, wg[r0:r0 + f.shape[0]], x.to(dev), f.to(dev))
        r0 += f.shape[0]

    # autograd: gradient of the shard equals the reduce-scattered full gradient
    m, n, k = 256, 256 * world, 256
    x_all = torch.randn(world, m, k, generator=g).to(torch.bfloat16)
    w_full = (0.05 * torch.randn(n, k, generator=g)).to(torch.bfloat16)
    x = x_all[rank].to(dev).requires_grad_(True)
    shard = w_full.chunk(world)[rank].to(dev).requires_grad_(True)
    y = all_gather_linear(x, shard, group)
    y.float().square().sum().backward()
    wf = w_full.to(dev).float()
    dw_full = sum(2 * (x_all[r].to(dev).float() @ wf.t()).t() @ x_all[r].to(dev).float() for r in range(world))
    assert_close(shard.grad.float(), dw_full.chunk(world)[rank], rtol=3e-2, atol=5e-1, max_mismatch_pct=0.5)
    dx = 2 * (x.detach().float() @ wf.t()) @ wf
    assert_close(x.grad.float(), dx, rtol=3e-2, atol=5e-2, max_mismatch_pct=0.5)


@pytest.mark.multigpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ag_gemm_two_ranks_matches_fp32():
    run_distributed(_dist_worker, 2, backend="nccl", device_type="cuda", timeout_s=120)


def _train_worker(rank, world):
    """A tiny Llama trained with q/k/v and gate/up through the fused gather matches
    the same model on plain FSDP2 (same init, same data)."""
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    from dtensor_muon_b200.models import preset
    from dtensor_muon_b200.ops import _ext
    from dtensor_muon_b200.train import Trainer, build_llama, build_optimizer, synthetic_batch

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    mesh = init_device_mesh("cuda", (world,))
    cfg = preset("tiny", dim=512, n_heads=4, n_kv_heads=2, ffn_dim=1024)
    losses, finals = {}, {}
    for fused in (False, True, "all"):
        model = build_llama(cfg, dev, mesh=mesh, seed=0, fsdp_comm="nccl", fused_gather=fused)
        # identical weights in both runs: a seeded full tensor per parameter
        gen = torch.Generator().manual_seed(11)
        with torch.no_grad():
            for name, p in sorted(model.named_parameters()):
                full = torch.ones(p.shape) if "norm" in name else 0.02 * torch.randn(p.shape, generator=gen)
                local = p.to_local()
                n = local.shape[0]
                local.copy_(full[rank * n:(rank + 1) * n].to(local.dtype))
        opt = build_optimizer(model, lr=0.02)
        tr = Trainer(model, opt)
        gen = torch.Generator().manual_seed(5)
        ls = []
        for _ in range(3):
            tokens, targets = synthetic_batch(1, 256, cfg.vocab_size, gen)
            ls.append(tr.step(tokens.to(dev), targets.to(dev)).item())
        torch.cuda.synchronize()
        _ext.check_device_errors(dev)
        losses[fused] = ls
        finals[fused] = {n: p.full_tensor().float() for n, p in model.named_parameters()}
    for mode in (True, "all"):
        for a, b in zip(losses[False], losses[mode]):
            assert abs(a - b) < 2e-2 * max(1.0, abs(a)), (mode, losses[False], losses[mode])
        for n, p in finals[False].items():
            assert_close(finals[mode][n], p, rtol=5e-2, atol=5e-3, max_mismatch_pct=2.0, msg=f"{mode} {n}")
    dist.barrier()


@pytest.mark.multigpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_gather_training_matches_fsdp():
    run_distributed(_train_worker, 2, backend="nccl", device_type="cuda", timeout_s=300)
