"""Fused owner-compute path (FSDP-sharded 2-D DTensors over NVLink peer memory)
against the single-process optimizer, on 2 GPUs (mirrors the reference's
tests/optim/test_optim_foreach.py:318-391)."""

import pytest
import torch

from testkit import assert_close, run_distributed

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

SHAPES = [(256, 512), (512, 256), (200, 384), (384, 200), (64, 96), (1024, 4096)]


def _worker(rank, world, algorithm, strategy, n_steps, dtype_name, mesh_shape=None, placements=None):
    import torch
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Replicate, Shard, distribute_tensor

    from dtensor_muon_b200 import Muon
    from dtensor_muon_b200.ops import _ext

    dtype = getattr(torch, dtype_name)
    device = torch.device("cuda", rank)
    mesh = init_device_mesh("cuda", tuple(mesh_shape) if mesh_shape else (world,))
    # FSDP: (Shard(0),); HSDP: (Replicate(), Shard(0)) over a (replicas, shards) mesh
    pl = [Shard(0)] if mesh.ndim == 1 else [Replicate(), Shard(0)]
    if placements is not None:  # e.g. "S1" (row-parallel TP) or "S0,S1" (FSDP x row-parallel TP)
        pl = [Shard(int(x[1])) if x[0] == "S" else Replicate() for x in placements.split(",")]
    gen = torch.Generator().manual_seed(0)
    fulls = [torch.randn(s, generator=gen).to(dtype) for s in SHAPES for _ in range(3)]
    ref_params = [torch.nn.Parameter(f.clone().to(device)) for f in fulls]
    dist_params = [torch.nn.Parameter(distribute_tensor(f.clone().to(device), mesh, pl)) for f in fulls]
    kw = dict(lr=0.05, wd=0.1, orthogonalization_strategy=strategy)
    ref = Muon([{"params": ref_params, "algorithm": algorithm}], foreach=True, **kw)
    opt = Muon([{"params": dist_params, "algorithm": algorithm}], foreach=True, **kw)
    for _ in range(n_steps):
        grads = [torch.randn(f.shape, generator=gen).to(dtype) for f in fulls]
        for p, g in zip(ref_params, grads):
            p.grad = g.to(device)
        for p, g in zip(dist_params, grads):
            p.grad = distribute_tensor(g.to(device), mesh, pl)
        ref.step()
        opt.step()
    torch.cuda.synchronize()
    _ext.check_device_errors(device)
    for i, (r, d) in enumerate(zip(ref_params, dist_params)):
        assert_close(d.full_tensor(), r.detach(), rtol=1e-2, atol=3e-2, max_mismatch_pct=1.0, msg=f"param {i}")
        if algorithm == "normuon":
            assert_close(
                opt.state[d]["variance_neuron"].full_tensor(), ref.state[r]["variance_neuron"], rtol=2e-2, atol=1e-6
            )


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("algorithm", ["muon", "normuon"])
@pytest.mark.parametrize("strategy", ["polar_express", "newton_schulz"])
def test_owner_compute_matches_single_process(algorithm, strategy):
    run_distributed(
        _worker, 2, args=(algorithm, strategy, 3, "float32"), backend="nccl", device_type="cuda", timeout_s=120
    )


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_owner_compute_bf16_params():
    run_distributed(_worker, 2, args=("muon", "polar_express", 2, "bfloat16"), backend="nccl", device_type="cuda")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_owner_compute_hsdp_mesh_matches_single_process():
    """HSDP placements (Replicate(), Shard(0)) on a (1, 2) mesh take the fused
    owner-compute path (one shard group) and match the single-process step."""
    run_distributed(_hsdp_worker, 2, args=((1, 2),), backend="nccl", device_type="cuda", timeout_s=120)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_owner_compute_hsdp_2x2_matches_single_process():
    run_distributed(_hsdp_worker, 4, args=((2, 2),), backend="nccl", device_type="cuda", timeout_s=180)


def _hsdp_worker(rank, world, mesh_shape):
    from dtensor_muon_b200.parallel import owner_compute

    calls = []
    orig = owner_compute.owner_compute_update
    owner_compute.owner_compute_update = lambda *a, **k: (calls.append(1), orig(*a, **k))[1]
    try:
        _worker(rank, world, "muon", "polar_express", 2, "float32", mesh_shape)
    finally:
        owner_compute.owner_compute_update = orig
    assert calls, "HSDP batches must take the owner-compute path"


def _rect_worker(rank, world, mesh_shape, placements, algorithm):
    from dtensor_muon_b200.parallel import owner_compute

    calls = []
    orig = owner_compute.owner_compute_update
    owner_compute.owner_compute_update = lambda *a, **k: (calls.append(1), orig(*a, **k))[1]
    try:
        _worker(rank, world, algorithm, "newton_schulz", 2, "float32", mesh_shape, placements)
    finally:
        owner_compute.owner_compute_update = orig
    assert calls, "column-sharded batches must take the owner-compute path"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("algorithm", ["muon", "normuon"])
def test_owner_compute_column_shards_match_single_process(algorithm):
    """Row-parallel TP placement (Shard(1)): every rank holds a column block; owner
    compute packs and applies rectangles."""
    run_distributed(_rect_worker, 2, args=((2,), "S1", algorithm), backend="nccl", device_type="cuda",
                    timeout_s=120)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_owner_compute_2d_rectangles_match_single_process():
    """FSDP x row-parallel TP on a (2, 2) mesh: row x column blocks."""
    run_distributed(_rect_worker, 4, args=((2, 2), "S0,S1", "muon"), backend="nccl", device_type="cuda",
                    timeout_s=180)


def _sharded_worker(rank, world, strategy, dtype_name):
    from dtensor_muon_b200.parallel import sharded_ns

    calls = []
    orig = sharded_ns.sharded_update
    sharded_ns._FORCE = "1"
    sharded_ns.sharded_update = lambda *a, **k: (calls.append(1), orig(*a, **k))[1]
    try:
        _worker(rank, world, "muon", strategy, 3, dtype_name)
    finally:
        sharded_ns.sharded_update = orig
        sharded_ns._FORCE = None
    assert calls, "tall row-sharded batches must take the sharded Newton-Schulz path"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("strategy", ["newton_schulz", "polar_express"])
def test_sharded_newton_schulz_matches_single_process(strategy):
    """Row shards orthogonalised in place with the all-reduced partial Gram
    (tall shapes), against the single-process step."""
    run_distributed(_sharded_worker, 2, args=(strategy, "float32"), backend="nccl", device_type="cuda",
                    timeout_s=120)


def _zeropower_worker(rank, world):
    import torch
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Shard, distribute_tensor

    from dtensor_muon_b200.ops import _ext, ortho
    from dtensor_muon_b200.orthogonalize import foreach_zeropower, zeropower

    device = torch.device("cuda", rank)
    mesh = init_device_mesh("cuda", (world,))
    gen = torch.Generator().manual_seed(4)
    for shape in [(4096, 1024), (2048, 2048), (1000, 600)]:
        full = torch.randn(shape, generator=gen).to(device)
        d = distribute_tensor(full, mesh, [Shard(0)])
        for strategy in ("newton_schulz", "polar_express"):
            want = ortho.orthogonalize_native([full], 5, strategy)[0]
            got = zeropower(d, steps=5, strategy=strategy)
            assert list(got.placements) == [Shard(0)] and got.dtype == torch.bfloat16
            assert_close(got.full_tensor(), want, rtol=2e-2, atol=2e-2, max_mismatch_pct=1.0, msg=f"{shape}")
            (got2,) = foreach_zeropower([d], steps=5, strategy=strategy)
            assert_close(got2.full_tensor(), want, rtol=2e-2, atol=2e-2, max_mismatch_pct=1.0)
    torch.cuda.synchronize()
    _ext.check_device_errors(device)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_zeropower_matches_gathered():
    """Public zeropower / foreach_zeropower on a row-sharded matrix (no gather,
    all-reduced partial Grams) against the single-GPU engine on the full matrix."""
    run_distributed(_zeropower_worker, 2, backend="nccl", device_type="cuda", timeout_s=120)
