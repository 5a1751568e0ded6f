"""Expert-parallel MoE (dispatch / combine) against the single-process MoE.

CPU: the NCCL-style all-to-all transport under gloo. GPU (2 ranks): the P2P
transport over symmetric memory."""

import pytest
import torch

from testkit import run_distributed


def _worker(rank, world, backend_kind, device_type):
    import torch
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    from dtensor_muon_b200.models.mixtral import Mixtral, mixtral_preset
    from dtensor_muon_b200.models.llama import lm_loss
    from dtensor_muon_b200.parallel.expert_parallel import ExpertParallel, reduce_dense_grads, shard_experts

    device = torch.device(device_type, rank if device_type == "cuda" else 0)
    dtype = torch.bfloat16 if device_type == "cuda" else torch.float32
    cfg = mixtral_preset("mixtral-tiny")
    torch.manual_seed(0)
    ref = Mixtral(cfg)
    ref.init_weights(seed=0)
    ref = ref.to(device=device, dtype=dtype)
    model = Mixtral(cfg)
    model.load_state_dict(ref.state_dict())
    model = model.to(device=device, dtype=dtype)
    mesh = init_device_mesh(device_type, (world,))
    ep = ExpertParallel(mesh.get_group(), cfg.n_experts, backend=backend_kind)
    experts = shard_experts(model, mesh, ep)

    gen = torch.Generator().manual_seed(1)
    tokens = torch.randint(0, cfg.vocab_size, (world, 2, 33), generator=gen)
    # reference: all ranks' batches on one process, mean loss over ranks
    ref_loss = sum(lm_loss(ref(tokens[r, :, :-1].to(device)), tokens[r, :, 1:].to(device)) for r in range(world)) / world
    ref_loss.backward()
    loss = lm_loss(model(tokens[rank, :, :-1].to(device)), tokens[rank, :, 1:].to(device))
    loss.backward()
    reduce_dense_grads(list(model.parameters()), mesh.get_group(), experts)
    tot = loss.detach().clone()
    dist.all_reduce(tot)
    tol = dict(rtol=2e-2, atol=2e-2) if dtype == torch.bfloat16 else dict(rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(tot / world, ref_loss.detach(), **tol)
    ref_params = dict(ref.named_parameters())
    for name, p in model.named_parameters():
        g = p.grad.full_tensor() if hasattr(p.grad, "full_tensor") else p.grad
        torch.testing.assert_close(g.float(), ref_params[name].grad.float(), **tol, msg=name)


def test_ep_all_to_all_matches_single_process_gloo():
    run_distributed(_worker, 2, args=("nccl", "cpu"))


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("backend_kind", ["p2p", "nccl"])
def test_ep_matches_single_process_cuda(backend_kind):
    run_distributed(_worker, 2, args=(backend_kind, "cuda"), backend="nccl", device_type="cuda")


@pytest.mark.gpu
@pytest.mark.parametrize("opt_name", ["Muon", "MuonFp8", "Muon8bit"])
def test_mixtral_single_gpu_step(opt_name):
    import dtensor_muon_b200 as dmb
    from dtensor_muon_b200.models.mixtral import Mixtral, mixtral_preset
    from dtensor_muon_b200.ops import _ext
    from dtensor_muon_b200.train import Trainer, build_optimizer, synthetic_batch

    cfg = mixtral_preset("mixtral-tiny")
    model = Mixtral(cfg)
    model.init_weights(seed=0)
    model = model.cuda().bfloat16()
    opt = build_optimizer(model, getattr(dmb, opt_name), lr=1e-3, block_size=256) if opt_name != "Muon" \
        else build_optimizer(model, dmb.Muon, lr=1e-3)
    experts = [p for n, p in model.named_parameters() if n.endswith(("w1", "w2", "w3")) and p.ndim == 3]
    before = [p.detach().clone() for p in experts]
    tokens, targets = synthetic_batch(2, 64, cfg.vocab_size)
    loss = Trainer(model, opt).step(tokens.cuda(), targets.cuda())
    torch.cuda.synchronize()
    _ext.check_device_errors("cuda")
    assert torch.isfinite(loss)
    assert all(not torch.equal(b, p) for b, p in zip(before, experts))


@pytest.mark.parametrize("world,n_experts,seed", [(2, 4, 0), (4, 8, 1), (8, 8, 2), (4, 16, 3)])
def test_plan_matches_brute_force(world, n_experts, seed):
    """The vectorised routing plan (device tensor ops) equals a per-row
    construction: receive regions grouped by (local expert, source), each
    source's rows of an expert contiguous, NCCL receive permutation."""
    from dtensor_muon_b200.parallel.expert_parallel import _Plan

    g = torch.Generator().manual_seed(seed)
    counts_all = torch.randint(0, 5, (world, n_experts), generator=g)
    counts_all[0, 0] = 0  # empty blocks
    el = n_experts // world
    for rank in range(world):
        experts = torch.repeat_interleave(torch.arange(n_experts), counts_all[rank])
        plan = _Plan(counts_all, experts, rank, world, n_experts)
        # brute force: walk owners' layouts
        off = {}
        for d in range(world):
            cur = 0
            for e in range(d * el, (d + 1) * el):
                for s in range(world):
                    off[(s, e)] = cur
                    cur += int(counts_all[s, e])
        want_rank, want_row = [], []
        for e in range(n_experts):
            for j in range(int(counts_all[rank, e])):
                want_rank.append(e // el)
                want_row.append(off[(rank, e)] + j)
        assert plan.dst_rank_d.tolist() == want_rank
        assert plan.dst_row_d.tolist() == want_row
        assert plan.recv_rows == [int(counts_all[:, d * el:(d + 1) * el].sum()) for d in range(world)]
        assert plan.send_split == [int(counts_all[rank, d * el:(d + 1) * el].sum()) for d in range(world)]
        assert plan.recv_split == [int(counts_all[s, rank * el:(rank + 1) * el].sum()) for s in range(world)]
        # NCCL order (source, local expert) -> (local expert, source)
        labels = [(s, e) for s in range(world) for e in range(el) for _ in range(int(counts_all[s, rank * el + e]))]
        permuted = [labels[i] for i in plan.nccl_perm_d.tolist()]
        assert permuted == sorted(labels, key=lambda t: (t[1], t[0]))
