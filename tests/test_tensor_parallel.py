"""Tensor-parallel Llama + NorMuon on a TP group (gloo, CPU) against one process."""

import torch

from testkit import run_distributed


def _worker(rank, world):
    import torch
    from torch.distributed.device_mesh import init_device_mesh

    from dtensor_muon_b200 import Muon
    from dtensor_muon_b200.models.llama import Llama, lm_loss, muon_and_adam_params, preset
    from dtensor_muon_b200.parallel.tensor_parallel import apply_tensor_parallel

    cfg = preset("tiny")
    torch.manual_seed(0)
    ref = Llama(cfg)
    ref.init_weights(seed=0)
    model = Llama(cfg)
    model.load_state_dict(ref.state_dict())
    mesh = init_device_mesh("cpu", (world,))
    apply_tensor_parallel(model, mesh)

    def make_opt(m):
        mu, ad = muon_and_adam_params(m)
        return Muon([{"params": mu, "algorithm": "normuon"}, {"params": ad, "algorithm": "adamw"}],
                    lr=0.02, orthogonalization_strategy="newton_schulz")

    o_ref, o_tp = make_opt(ref), make_opt(model)
    gen = torch.Generator().manual_seed(3)
    for _ in range(2):
        tok = torch.randint(0, cfg.vocab_size, (2, 17), generator=gen)
        l_ref = lm_loss(ref(tok[:, :-1]), tok[:, 1:])
        l_tp = lm_loss(model(tok[:, :-1]), tok[:, 1:])
        torch.testing.assert_close(l_tp, l_ref, rtol=1e-4, atol=1e-4)
        l_ref.backward()
        l_tp.backward()
        o_ref.step()
        o_tp.step()
        o_ref.zero_grad()
        o_tp.zero_grad()
    refp = dict(ref.named_parameters())
    for name, p in model.named_parameters():
        full = p.full_tensor() if hasattr(p, "full_tensor") else p
        # bf16 orthogonalisation on different reduction orders: bf16-level budget
        bad = (~torch.isclose(full.detach(), refp[name].detach(), rtol=1e-2, atol=3e-3)).float().mean().item()
        assert bad < 0.02, (name, bad)


def test_tp_normuon_matches_single_process_gloo():
    run_distributed(_worker, 2)


def _mixed_worker(rank, world):
    import torch
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Shard, distribute_tensor

    from dtensor_muon_b200.optim.optim import _group_muon_tensors

    mesh = init_device_mesh("cpu", (world,))
    ps = [distribute_tensor(torch.randn(8, 8), mesh, [pl]) for pl in (Shard(0), Shard(1), Shard(0))]
    groups = _group_muon_tensors(ps, ps, {"momentum_buffer": ps}, [torch.tensor(1.0)] * 3)
    sizes = sorted(len(g[1]) for g in groups)
    assert sizes == [1, 2], sizes  # Shard(0) pair together, Shard(1) alone


def test_same_shape_different_placements_batch_separately():
    run_distributed(_mixed_worker, 2)


def _fsdp_tp_worker(rank, world):
    import torch
    from torch.distributed.device_mesh import init_device_mesh

    from dtensor_muon_b200 import Muon
    from dtensor_muon_b200.models.llama import Llama, lm_loss, muon_and_adam_params, preset
    from dtensor_muon_b200.parallel.tensor_parallel import apply_fsdp_tp

    cfg = preset("tiny")
    torch.manual_seed(0)
    ref = Llama(cfg)
    ref.init_weights(seed=0)
    model = Llama(cfg)
    model.load_state_dict(ref.state_dict())
    mesh = init_device_mesh("cpu", (2, 2), mesh_dim_names=("dp", "tp"))
    apply_fsdp_tp(model, mesh)

    def make_opt(m):
        mu, ad = muon_and_adam_params(m)
        return Muon([{"params": mu, "algorithm": "normuon"}, {"params": ad, "algorithm": "adamw"}],
                    lr=0.02, orthogonalization_strategy="newton_schulz", foreach=False)

    o_ref, o_m = make_opt(ref), make_opt(model)
    tok = torch.randint(0, cfg.vocab_size, (2, 17), generator=torch.Generator().manual_seed(3))
    dp = mesh.get_local_rank("dp")
    # every dp rank sees the same batch, so the averaged grads equal the single-process ones
    lm_loss(ref(tok[:, :-1]), tok[:, 1:]).backward()
    lm_loss(model(tok[:, :-1]), tok[:, 1:]).backward()
    # batched path on the strided-shard grads (FSDP over TP): gather + split-over-mesh
    from dtensor_muon_b200.orthogonalize import foreach_zeropower, orthogonalize_local

    strided = [p.grad for p in model.parameters()
               if p.grad is not None and p.ndim == 2 and any(type(q).__name__ == "_StridedShard" for q in p.placements)]
    assert strided, "expected FSDP x TP strided-shard placements"
    by_shape = {}
    for g in strided:
        by_shape.setdefault((tuple(g.shape), tuple(g.placements)), []).append(g)
    for gs in by_shape.values():
        us = foreach_zeropower(gs, steps=5, strategy="newton_schulz")
        ref_u = orthogonalize_local(torch.stack([g.full_tensor() for g in gs]), 5, 1e-7, "newton_schulz")
        for u, r in zip(us, ref_u):
            assert u.placements == gs[0].placements
            torch.testing.assert_close(u.full_tensor().float(), r.float(), rtol=2e-2, atol=2e-2)
    o_ref.step()
    o_m.step()
    refp = dict(ref.named_parameters())
    for name, p in model.named_parameters():
        full = p.full_tensor() if hasattr(p, "full_tensor") else p
        bad = (~torch.isclose(full.detach(), refp[name].detach(), rtol=1e-2, atol=3e-3)).float().mean().item()
        assert bad < 0.02, (name, bad, dp)


def test_fsdp_x_tp_normuon_gloo_four_ranks():
    run_distributed(_fsdp_tp_worker, 4)


def _layout_worker(rank, world):
    import torch
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    from dtensor_muon_b200.models.llama import Llama, preset
    from dtensor_muon_b200.parallel.owner_compute import shard_layout
    from dtensor_muon_b200.parallel.tensor_parallel import apply_fsdp_tp

    cfg = preset("tiny")
    torch.manual_seed(0)
    model = Llama(cfg)
    model.init_weights(seed=0)
    mesh = init_device_mesh("cpu", (2, 2), mesh_dim_names=("dp", "tp"))
    apply_fsdp_tp(model, mesh)
    seen = 0
    for name, p in model.named_parameters():
        if p.ndim != 2 or "layers." not in name:
            continue
        lay = shard_layout(p)
        assert lay is not None, (name, p.placements)
        assert lay.world == world and lay.rank == rank
        local = p.to_local()
        full = p.full_tensor()
        assert tuple(local.shape) == (lay.r1 - lay.r0, lay.c1 - lay.c0), (name, local.shape, lay)
        torch.testing.assert_close(local, full[lay.r0 : lay.r1, lay.c0 : lay.c1])
        # the rectangles of all ranks tile the matrix exactly once
        rect = torch.tensor([lay.r0, lay.r1, lay.c0, lay.c1])
        rects = [torch.zeros_like(rect) for _ in range(world)]
        dist.all_gather(rects, rect)
        cover = torch.zeros(p.shape, dtype=torch.int32)
        for r0, r1, c0, c1 in (x.tolist() for x in rects):
            cover[r0:r1, c0:c1] += 1
        assert torch.all(cover == 1), name
        seen += 1
    assert seen >= 7 * cfg.n_layers


def test_fsdp_x_tp_shards_are_rectangles_tiling_each_matrix_gloo():
    """Owner compute's layout of FSDP x TP shards (strided row blocks of column-parallel
    weights, row x column blocks of row-parallel ones) on a (2, 2) mesh."""
    run_distributed(_layout_worker, 4)
