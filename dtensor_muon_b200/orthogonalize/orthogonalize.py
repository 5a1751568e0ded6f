"""Orthogonalisation entry points and DTensor distribution.

Public-compatible with the reference's ``zeropower`` / ``foreach_zeropower`` /
``foreach_zeropower_3d_fsdp`` / ``is_fsdp_3d_sharded``
(src/muonium/orthogonalize/orthogonalize.py:68-204). The result is always
bf16, like the reference.

Local work goes to the native tcgen05 engine for CUDA tensors
(:func:`dtensor_muon_b200.ops.ortho.orthogonalize_native`) and to the PyTorch
loops otherwise. DTensor inputs keep the reference's distribution contract:

* ``zeropower``: gather the full matrix, orthogonalise, hand back a DTensor
  with the input's placements; on CUDA, row-sharded matrices (fewer than half
  as many as ranks) instead run the sharded iteration of
  :mod:`dtensor_muon_b200.parallel.sharded_ns` with no gather;
* ``foreach_zeropower``: stack the batch, redistribute so that every rank owns
  whole matrices (Shard(0) of the stack), orthogonalise locally, redistribute
  back and unbind;
* ``foreach_zeropower_3d_fsdp``: 3-D tensors sharded only on dim 0 are
  independent matrices on every rank: no communication.
"""

from __future__ import annotations

from typing import Literal, cast

import torch
from torch import Tensor
from torch.distributed.tensor import DTensor, Replicate, Shard

from ..ops import ortho as _native
from .newton_schulz import ns_loop
from .polar_express import pe_loop

OrthogonalizationStrategy = Literal["newton_schulz", "polar_express"]


def get_dtensor_metadata(dtensors: DTensor | list[DTensor], run_check: bool = True) -> dict:
    """Mesh / placements / global shape / stride needed to rebuild a DTensor."""
    first = dtensors if isinstance(dtensors, DTensor) else dtensors[0]
    meta = {
        "device_mesh": first.device_mesh,
        "placements": first.placements,
        "shape": first.shape,
        "stride": first.stride(),
    }
    if run_check and isinstance(dtensors, list) and not torch.compiler.is_compiling():
        for d in dtensors:
            same = (
                d.device_mesh == meta["device_mesh"]
                and d.placements == meta["placements"]
                and d.shape == meta["shape"]
                and d.stride() == meta["stride"]
            )
            assert same, "all DTensors of a batch must share mesh, placements, shape and stride"
    return meta


def _validate_orthogonalization_args(strategy: str, steps: int) -> None:
    if strategy not in ("newton_schulz", "polar_express"):
        raise ValueError(f"Unknown orthogonalization strategy: {strategy}")
    if strategy == "polar_express":
        assert steps <= 5, "polar express orthogonalization only supports up to 5 optimization steps."


def _torch_loop(strategy: str):
    if strategy == "newton_schulz":
        return ns_loop
    if strategy == "polar_express":
        return pe_loop
    raise ValueError(f"Unknown orthogonalization strategy: {strategy}")


def _use_native(x: Tensor, use_native: bool) -> bool:
    return use_native and x.is_cuda


def orthogonalize_local(X: Tensor, steps: int, eps: float, strategy: str, use_native: bool = True) -> Tensor:
    """Orthogonalise a plain tensor [..., N, M] over its last two dims; bf16 out."""
    if X.numel() == 0 or (X.ndim >= 3 and X.size(0) == 0):
        return X.bfloat16()
    if _use_native(X, use_native):
        lead = X.shape[:-2]
        mats = X.reshape(-1, X.shape[-2], X.shape[-1])
        outs = _native.orthogonalize_native(list(mats.unbind(0)), steps, strategy, eps)
        return torch.stack(outs).reshape(*lead, X.shape[-2], X.shape[-1])
    return _torch_loop(strategy)(X.bfloat16(), steps=steps, eps=eps)


def zeropower(
    G: Tensor,
    steps: int = 5,
    eps: float = 1e-7,
    use_native: bool = True,
    strategy: OrthogonalizationStrategy = "newton_schulz",
    *,
    use_triton: bool | None = None,
) -> Tensor:
    """Zero-power (orthogonal polar factor) of one matrix, bf16 out.

    ``use_triton`` is accepted as an alias of ``use_native`` for callers
    written against the reference signature.
    """
    if use_triton is not None:
        use_native = use_triton
    _validate_orthogonalization_args(strategy, steps)
    if isinstance(G, DTensor):
        if use_native and _sharded_ok([G]):
            from ..parallel.sharded_ns import sharded_zeropower

            return sharded_zeropower([G], steps, strategy, eps)[0]
        full = G.full_tensor()
        U = orthogonalize_local(full, steps, eps, strategy, use_native)
        U = DTensor.from_local(U, device_mesh=G.device_mesh, placements=(Replicate(),) * G.device_mesh.ndim)
        return U.redistribute(placements=G.placements, async_op=True)
    return orthogonalize_local(G, steps, eps, strategy, use_native)


def foreach_zeropower(
    Gs: list[Tensor],
    steps: int = 5,
    eps: float = 1e-7,
    use_native: bool = True,
    strategy: OrthogonalizationStrategy = "newton_schulz",
    *,
    use_triton: bool | None = None,
) -> list[Tensor]:
    """Zero-power of a same-shape batch of matrices (2-D or 3-D each), bf16 out."""
    if use_triton is not None:
        use_native = use_triton
    _validate_orthogonalization_args(strategy, steps)
    if len(Gs) == 0:
        return []
    if isinstance(Gs[0], DTensor):
        Gs_d = cast(list[DTensor], Gs)
        meta = get_dtensor_metadata(Gs_d)
        if use_native and _sharded_ok(Gs_d):
            # few row-sharded matrices over many ranks: iterate on the shards
            from ..parallel.sharded_ns import sharded_zeropower

            return cast(list[Tensor], sharded_zeropower(Gs_d, steps, strategy, eps))
        mesh = meta["device_mesh"]
        if _needs_gather_path(meta["placements"]):
            # FSDP over TP-sharded weights (_StridedShard + Shard): gather each
            # full matrix, orthogonalise the batch locally, hand back shards.
            full = torch.stack([g.full_tensor() for g in Gs_d])
            U = _split_over_mesh(full, mesh, lambda x: orthogonalize_local(x, steps, eps, strategy, use_native))
            rep = (Replicate(),) * mesh.ndim
            return [
                DTensor.from_local(u, device_mesh=mesh, placements=rep).redistribute(placements=meta["placements"])
                for u in U.unbind(0)
            ]
        owner_pl = (Shard(0), *([Replicate()] * (mesh.ndim - 1)))
        X = cast(DTensor, torch.stack(list(Gs_d), dim=0).bfloat16())
        X_own = X.redistribute(placements=owner_pl, async_op=True)
        U_own = orthogonalize_local(X_own.to_local(), steps, eps, strategy, use_native)
        U_own = DTensor.from_local(U_own, **get_dtensor_metadata(X_own))
        U = U_own.redistribute(placements=X.placements, async_op=True)
        return [DTensor.from_local(u, **meta) for u in U.to_local().unbind(0)]
    X = torch.stack(list(Gs))
    U = orthogonalize_local(X, steps, eps, strategy, use_native)
    return list(U.unbind(0))


def _sharded_ok(gs: list[DTensor]) -> bool:
    """Row-sharded CUDA matrices that the sharded iteration (no gather) takes."""
    if gs[0].device_mesh.device_type != "cuda":
        return False
    from ..parallel import sharded_ns

    return sharded_ns.zeropower_eligible(gs)


def _split_over_mesh(full: Tensor, mesh, fn) -> Tensor:
    """Apply ``fn`` to a replicated batch with the work split over every rank of ``mesh``:
    rank r handles a contiguous chunk, then one all-gather returns all results."""
    import torch.distributed as dist

    world = mesh.size()
    if world == 1 or world != dist.get_world_size():
        return fn(full)
    rank = dist.get_rank()
    B = full.shape[0]
    chunk = -(-B // world)
    mine = fn(full[rank * chunk : min(B, (rank + 1) * chunk)]) if rank * chunk < B else None
    out = torch.empty((chunk * world, *full.shape[1:]), dtype=torch.bfloat16, device=full.device)
    send = torch.zeros((chunk, *full.shape[1:]), dtype=torch.bfloat16, device=full.device)
    if mine is not None:
        send[: mine.shape[0]].copy_(mine)
    dist.all_gather_into_tensor(out, send)
    return out[:B]


def _needs_gather_path(placements) -> bool:
    """Placements the stacked redistribute cannot express (strided shards from FSDP x TP)."""
    return any(type(p).__name__ == "_StridedShard" for p in placements)


def is_fsdp_3d_sharded(xs: list[Tensor]) -> bool:
    """True when every tensor is a 3-D DTensor sharded on dim 0 exactly once and
    replicated on every other mesh dim (its local shards are whole matrices)."""
    for x in xs:
        if not isinstance(x, DTensor) or x.ndim != 3:
            return False
        pls = x.placements
        if sum(p == Shard(0) for p in pls) != 1:
            return False
        if sum(p == Replicate() for p in pls) != len(pls) - 1:
            return False
    return True


def foreach_zeropower_3d_fsdp(
    Gs: list[DTensor],
    steps: int = 5,
    eps: float = 1e-7,
    use_native: bool = True,
    strategy: OrthogonalizationStrategy = "newton_schulz",
    *,
    use_triton: bool | None = None,
) -> list[DTensor]:
    """Collective-free path for dim-0-sharded 3-D stacks (FSDP / EP experts)."""
    if use_triton is not None:
        use_native = use_triton
    assert is_fsdp_3d_sharded(Gs), (
        "foreach_zeropower_3d_fsdp only works for DTensors that are *only* sharded along the first dimension"
    )
    _validate_orthogonalization_args(strategy, steps)
    meta = get_dtensor_metadata(Gs)
    X = torch.stack([g.to_local() for g in Gs])
    U = orthogonalize_local(X, steps, eps, strategy, use_native)
    return [DTensor.from_local(u, **meta) for u in U.unbind(0)]
