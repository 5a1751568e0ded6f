"""Orthogonalisation math and the zeropower API on CPU (PyTorch loops), plus
DTensor distribution under gloo (mirrors the reference's
tests/orthogonalize/*.py and tests/utils/test_dtensor.py)."""

import pytest
import torch

from dtensor_muon_b200.orthogonalize import (
    POLAR_EXPRESS_COEFFS,
    foreach_zeropower,
    foreach_zeropower_3d_fsdp,
    is_fsdp_3d_sharded,
    ns_loop,
    pe_loop,
    zeropower,
)
from testkit import run_distributed

LOOPS = {"newton_schulz": ns_loop, "polar_express": pe_loop}


def _sv(x):
    return torch.linalg.svdvals(x.double())


@pytest.mark.parametrize("strategy", list(LOOPS))
@pytest.mark.parametrize("shape", [(32, 64), (64, 32), (48, 48)])
def test_singular_values_near_one(strategy, shape):
    torch.manual_seed(0)
    g = torch.randn(shape)
    u = LOOPS[strategy](g.double(), 5, eps=1e-7)
    s = _sv(u)
    lo, hi = (0.5, 1.3) if strategy == "newton_schulz" else (0.6, 1.2)
    assert s.min() > lo and s.max() < hi, (s.min().item(), s.max().item())


@pytest.mark.parametrize("strategy", list(LOOPS))
def test_close_to_polar_factor(strategy):
    torch.manual_seed(1)
    g = torch.randn(40, 80, dtype=torch.float64)
    U, _, Vh = torch.linalg.svd(g, full_matrices=False)
    polar = U @ Vh
    u = LOOPS[strategy](g, 5, eps=1e-7)
    cos = (u * polar).sum() / (u.norm() * polar.norm())
    assert cos > 0.97


@pytest.mark.parametrize("strategy", list(LOOPS))
def test_steps0_is_normalized_input(strategy):
    g = torch.randn(8, 12, dtype=torch.float64)
    fac = 1.02 if strategy == "polar_express" else 1.0
    torch.testing.assert_close(LOOPS[strategy](g, 0, eps=1e-7), g / (g.norm() * fac + 1e-7))


@pytest.mark.parametrize("strategy", list(LOOPS))
def test_transpose_symmetry_and_batching(strategy):
    torch.manual_seed(2)
    g = torch.randn(3, 16, 24, dtype=torch.float64)
    loop = LOOPS[strategy]
    torch.testing.assert_close(loop(g.mT, 5, eps=1e-7), loop(g, 5, eps=1e-7).mT)
    torch.testing.assert_close(loop(g[:1], 5, eps=1e-7)[0], loop(g[0], 5, eps=1e-7))


@pytest.mark.parametrize("strategy", list(LOOPS))
def test_scale_invariance_and_zero_input(strategy):
    torch.manual_seed(3)
    g = torch.randn(16, 16, dtype=torch.float64)
    loop = LOOPS[strategy]
    torch.testing.assert_close(loop(g * 1e3, 5, eps=1e-12), loop(g, 5, eps=1e-12), rtol=1e-6, atol=1e-6)
    z = loop(torch.zeros(8, 8, dtype=torch.float64), 5, eps=1e-7)
    assert torch.isfinite(z).all() and z.abs().max() == 0
    r = torch.randn(8, 1, dtype=torch.float64) @ torch.randn(1, 8, dtype=torch.float64)
    assert torch.isfinite(loop(r, 5, eps=1e-7)).all()


def test_orthogonal_input_near_fixed_point():
    q, _ = torch.linalg.qr(torch.randn(32, 32, dtype=torch.float64))
    u = ns_loop(q, 5, eps=1e-12)
    s = _sv(u)
    assert (s - 1).abs().max() < 0.3


def test_pe_coefficient_table():
    assert len(POLAR_EXPRESS_COEFFS) == 5
    assert POLAR_EXPRESS_COEFFS[0] == pytest.approx((8.156554524902461, -22.48329292557795, 15.878769915207462))
    for a, b, c in POLAR_EXPRESS_COEFFS:
        assert a > 0 and b < 0 and c > 0


def test_zeropower_api_returns_bf16_and_validates():
    g = torch.randn(8, 16)
    u = zeropower(g, steps=3, strategy="polar_express")
    assert u.dtype == torch.bfloat16 and u.shape == g.shape
    with pytest.raises(AssertionError, match="only supports up to 5"):
        zeropower(g, steps=6, strategy="polar_express")
    with pytest.raises(ValueError, match="Unknown orthogonalization strategy"):
        zeropower(g, strategy="svd")
    us = foreach_zeropower([g, g * 2], steps=5)
    assert len(us) == 2 and all(x.dtype == torch.bfloat16 for x in us)
    torch.testing.assert_close(us[0].float(), us[1].float(), rtol=2e-2, atol=2e-2)
    # 3-D members are batches of matrices
    us3 = foreach_zeropower([torch.randn(2, 8, 16), torch.randn(2, 8, 16)], steps=5)
    assert us3[0].shape == (2, 8, 16)
    assert zeropower(g, use_triton=False).dtype == torch.bfloat16


def test_is_fsdp_3d_sharded_plain_tensors():
    assert not is_fsdp_3d_sharded([torch.randn(2, 3, 4)])


# ------------------------------------------------------------------ DTensor --
def _dtensor_worker(rank, world):
    import torch
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Replicate, Shard, distribute_tensor

    mesh = init_device_mesh("cpu", (world,))
    torch.manual_seed(0)
    fulls = [torch.randn(10, 12) for _ in range(3)]
    local_ref = [u.float() for u in foreach_zeropower(fulls, steps=5, strategy="polar_express")]
    for placement in (Shard(0), Shard(1), Replicate()):
        ds = [distribute_tensor(f, mesh, [placement]) for f in fulls]
        us = foreach_zeropower(ds, steps=5, strategy="polar_express")
        for u, r in zip(us, local_ref):
            assert u.placements == (placement,)
            torch.testing.assert_close(u.full_tensor().float(), r, rtol=2e-2, atol=2e-2)
        one = zeropower(ds[0], steps=5, strategy="polar_express")
        torch.testing.assert_close(one.full_tensor().float(), local_ref[0], rtol=2e-2, atol=2e-2)
    # 3-D dim-0 sharded stacks: collective-free path, local shards are whole matrices.
    stacks = [torch.randn(4, 6, 8) for _ in range(2)]
    d3 = [distribute_tensor(s, mesh, [Shard(0)]) for s in stacks]
    assert is_fsdp_3d_sharded(d3)
    assert not is_fsdp_3d_sharded([distribute_tensor(stacks[0], mesh, [Shard(1)])])
    u3 = foreach_zeropower_3d_fsdp(d3, steps=5, strategy="newton_schulz")
    ref3 = foreach_zeropower(stacks, steps=5, strategy="newton_schulz")
    for u, r in zip(u3, ref3):
        torch.testing.assert_close(u.full_tensor().float(), r.float(), rtol=2e-2, atol=2e-2)
    with pytest.raises(AssertionError, match="only works for DTensors"):
        foreach_zeropower_3d_fsdp([distribute_tensor(stacks[0], mesh, [Shard(1)])])


def test_dtensor_paths_gloo_two_ranks():
    run_distributed(_dtensor_worker, 2)


def _uneven_worker(rank, world):
    import torch
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Shard, distribute_tensor

    mesh = init_device_mesh("cpu", (world,))
    torch.manual_seed(1)
    fulls = [torch.randn(7, 5) for _ in range(3)]  # 3 matrices over 2 ranks, rows 7 uneven
    ds = [distribute_tensor(f, mesh, [Shard(0)]) for f in fulls]
    us = foreach_zeropower(ds, steps=5, strategy="newton_schulz")
    ref = foreach_zeropower(fulls, steps=5, strategy="newton_schulz")
    for u, r in zip(us, ref):
        torch.testing.assert_close(u.full_tensor().float(), r.float(), rtol=2e-2, atol=2e-2)


def test_dtensor_uneven_shards_gloo():
    run_distributed(_uneven_worker, 2)


def _mesh2d_worker(rank, world):
    import torch
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Replicate, Shard, distribute_tensor

    mesh = init_device_mesh("cpu", (2, 2), mesh_dim_names=("dp", "tp"))
    torch.manual_seed(2)
    fulls = [torch.randn(8, 12) for _ in range(4)]
    ref = foreach_zeropower(fulls, steps=5, strategy="polar_express")
    for pl in ([Replicate(), Shard(0)], [Shard(0), Shard(1)], [Replicate(), Shard(1)]):
        ds = [distribute_tensor(f, mesh, pl) for f in fulls]
        us = foreach_zeropower(ds, steps=5, strategy="polar_express")
        for u, r in zip(us, ref):
            assert list(u.placements) == pl
            torch.testing.assert_close(u.full_tensor().float(), r.float(), rtol=2e-2, atol=2e-2)


def test_dtensor_2d_mesh_gloo_four_ranks():
    run_distributed(_mesh2d_worker, 4)


def test_ns_coefficient_override_changes_the_iteration():
    torch.manual_seed(3)
    g = torch.randn(16, 24)
    default = ns_loop(g.bfloat16(), 5)
    same = ns_loop(g.bfloat16(), 5, a=3.4445, b=-4.7750, c=2.0315)
    cubic = ns_loop(g.bfloat16(), 5, a=1.5, b=-0.5, c=0.0)  # classic cubic Newton-Schulz
    torch.testing.assert_close(default, same)
    assert not torch.equal(default, cubic)
    # the cubic iteration converges monotonically towards singular values 1 from below
    sv = _sv(ns_loop(g.bfloat16(), 12, a=1.5, b=-0.5, c=0.0).float())
    assert float(sv.max()) < 1.05 and float(sv.min()) > 0.0


@pytest.mark.parametrize("strategy", list(LOOPS))
def test_rank_deficient_input_stays_finite(strategy):
    torch.manual_seed(4)
    u = torch.randn(32, 3)
    v = torch.randn(3, 48)
    g = u @ v  # rank 3
    out = zeropower(g, steps=5, strategy=strategy, use_native=False)
    assert torch.isfinite(out.float()).all()
    sv = _sv(out.float())
    # the 3 directions of the input are kept (the bf16 rounding noise in the
    # null space is amplified too, so only the top of the spectrum is checked)
    assert float(sv[:3].min()) > 0.5 and float(sv.max()) < 1.3


def _foreach_sign_worker(rank, world):
    import torch
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Replicate, Shard, distribute_tensor

    import dtensor_muon_b200.optim.optim  # noqa: F401  (registers the strategy)

    mesh = init_device_mesh("cpu", (world,))
    torch.manual_seed(5)
    fulls = [torch.randn(6, 4), torch.randn(5, 3), torch.randn(4, 4)]
    ds = [
        distribute_tensor(fulls[0], mesh, [Shard(0)]),
        distribute_tensor(fulls[1], mesh, [Shard(1)]),
        distribute_tensor(fulls[2], mesh, [Replicate()]),
    ]
    torch._foreach_sign_(ds)
    for d, f, pl in zip(ds, fulls, ([Shard(0)], [Shard(1)], [Replicate()])):
        assert list(d.placements) == pl
        torch.testing.assert_close(d.full_tensor(), f.sign())


def test_dtensor_foreach_sign_strategy_gloo():
    run_distributed(_foreach_sign_worker, 2)


@pytest.mark.parametrize("strategy", ["newton_schulz", "polar_express"])
@pytest.mark.parametrize("splits", [(40, 24), (16, 16, 16, 16), (64, 0)])
def test_sharded_iteration_equals_gathered(strategy, splits):
    """Right-multiplied iteration on row shards with summed partial Grams equals
    the gathered left-multiplied iteration (fp64 on the full matrix)."""
    from dtensor_muon_b200.parallel.sharded_ns import sharded_reference

    torch.manual_seed(9)
    X = torch.randn(sum(splits), 24, dtype=torch.float64)
    want = (ns_loop if strategy == "newton_schulz" else pe_loop)(X, 5, eps=1e-7)
    got = torch.cat(sharded_reference(list(X.split(list(splits))), 5, strategy), dim=0)
    torch.testing.assert_close(got.double(), want, rtol=1e-4, atol=1e-4)
