"""Owner-compute Muon for dim-0-sharded (FSDP) 2-D DTensors, fused over NVLink.

Same distribution as the reference's general path (whole matrices assigned
to owner ranks, src/muonium/orthogonalize/orthogonalize.py:140-155), but the
two NCCL all-to-alls are gone: each rank writes its momentum-updated row shard
straight into the owner's workspace (P2P stores inside the momentum kernel),
the owner runs the local tcgen05 engine, and each rank pulls its rows of the
result back (P2P loads inside the apply kernel). Sequence per batch:

    barrier | dist_pack (+ sums push) | barrier | owner: finalize + ortho [+ NorMuon] | barrier | dist_apply

Matrices are assigned in contiguous chunks (matrix b -> rank b // ceil(B/W)),
like a Shard(0) of the stacked batch.
"""

from __future__ import annotations

import math

import torch
from torch import Tensor
from torch.distributed.tensor import DTensor, Shard

from ..ops import _ext
from ..ops.ortho import WORKSPACE, coefficient_table, dtype_code, layout_for, norm_factor
from ..utils.tracing import nvtx
from . import symm

# Cap on one owner's share of the symmetric workspace (two ping-pong buffers).
MAX_OWNER_BYTES = 8 << 30


def _rows(R: int, world: int, rank: int) -> tuple[int, int]:
    chunk = -(-R // world)
    return min(rank * chunk, R), min((rank + 1) * chunk, R)


def eligible(params: list[Tensor], grads: list[Tensor], buffers: list[Tensor], variances=None) -> bool:
    if not params or not symm.available():
        return False
    g0 = grads[0]
    if not isinstance(g0, DTensor) or g0.ndim != 2:
        return False
    mesh = g0.device_mesh
    if mesh.ndim != 1 or tuple(g0.placements) != (Shard(0),) or mesh.device_type != "cuda":
        return False
    world, rank = mesh.size(), mesh.get_local_rank()
    r0, r1 = _rows(g0.shape[0], world, rank)
    tensors = list(params) + list(grads) + list(buffers) + (list(variances) if variances is not None else [])
    for t in tensors:
        if not isinstance(t, DTensor) or t.device_mesh != mesh or tuple(t.placements) != (Shard(0),):
            return False
        loc = t.to_local()
        if not loc.is_cuda or not loc.is_contiguous() or loc.shape[0] != r1 - r0:
            return False
    for p, g, b in zip(params, grads, buffers, strict=True):
        if p.shape != g.shape or b.shape != g.shape or b.dtype != torch.float32:
            return False
        if p.dtype not in (torch.float32, torch.bfloat16) or g.dtype not in (torch.float32, torch.bfloat16):
            return False
    return len({p.dtype for p in params}) == 1 and len({g.dtype for g in grads}) == 1


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


def owner_compute_update(
    params: list[DTensor],
    grads: list[DTensor],
    buffers: list[DTensor],
    lr_effs: list[float],
    *,
    weight_decay: float,
    cautious_wd: bool,
    momentum: float,
    nesterov: bool,
    maximize: bool,
    ns_steps: int,
    strategy: str,
    eps: float = 1e-7,
    variances: list[DTensor] | None = None,
    muon_beta2: float = 0.95,
    momentum_done: bool = False,
) -> None:
    """``momentum_done``: the grads already hold g' (momentum updated in the
    FSDP reduce-scatter), so the pack only casts and scatters them."""
    C_ = _ext.load()
    coeffs = coefficient_table(strategy, ns_steps)
    mesh = grads[0].device_mesh
    group = mesh.get_group()
    world, rank = mesh.size(), mesh.get_local_rank()
    R, C = grads[0].shape
    lay = layout_for(R, C)
    r0, r1 = _rows(R, world, rank)
    g1 = (lay.Mp if lay.transpose else lay.Np) if rank == world - 1 else r1
    device = grads[0].to_local().device
    ws = symm.workspace_for(group, device)
    fac = norm_factor(strategy)
    has_var = variances is not None

    # Batches with a common lr_eff; chunk so one owner's workspace stays bounded.
    per_slot = 2 * lay.Np * lay.Mp * 2
    max_slots = max(1, MAX_OWNER_BYTES // per_slot)
    order: dict[float, list[int]] = {}
    for i, lr in enumerate(lr_effs):
        order.setdefault(float(lr), []).append(i)
    for lr_eff, idxs in order.items():
        step = world * max_slots
        for s in range(0, len(idxs), step):
            sel = idxs[s : s + step]
            _run_batch(
                C_, ws, sel, params, grads, buffers, variances, lr_eff, lay, R, C, r0, r1, g1, rank, world,
                coeffs, fac, eps, weight_decay, cautious_wd, momentum, nesterov, maximize, muon_beta2, has_var,
                device, momentum_done,
            )


def _run_batch(C_, ws, sel, params, grads, buffers, variances, lr_eff, lay, R, C, r0, r1, g1, rank, world, coeffs,
               fac, eps, weight_decay, cautious_wd, momentum, nesterov, maximize, muon_beta2, has_var, device,
               momentum_done=False):
    S = len(sel)
    Bo = math.ceil(S / world)
    steps = coeffs.shape[0]
    # Symmetric layout: sums | vbuf | rowscale | x | x2
    sums_off = 0
    vbuf_off = _align(sums_off + Bo * world * 4)
    rs_off = _align(vbuf_off + (Bo * R * 4 if has_var else 0))
    x_off = _align(rs_off + (Bo * R * 4 if has_var else 0))
    slot_bytes = lay.Np * lay.Mp * 2
    x2_off = _align(x_off + Bo * slot_bytes)
    total = x2_off + Bo * slot_bytes
    buf, peer_base = ws.buffer(total)
    res_off = x_off if steps % 2 == 0 else x2_off

    loc = lambda t: t.to_local()  # noqa: E731
    ptrs = [
        [loc(grads[i]).data_ptr() for i in sel],
        [loc(buffers[i]).data_ptr() for i in sel],
        [loc(params[i]).data_ptr() for i in sel],
        [loc(variances[i]).data_ptr() for i in sel] if has_var else [0] * S,
    ]
    meta64 = torch.tensor(ptrs, dtype=torch.int64).pin_memory().to(device, non_blocking=True)
    owner = [b // Bo for b in range(S)]
    slot = [b % Bo for b in range(S)]
    meta32 = torch.tensor([owner, slot], dtype=torch.int32).pin_memory().to(device, non_blocking=True)
    ints = [
        x_off, res_off, sums_off, vbuf_off, rs_off,
        dtype_code(grads[sel[0]].dtype), dtype_code(params[sel[0]].dtype),
        R, C, int(lay.transpose), lay.Np, lay.Mp, r0, r1, g1, rank, world,
        int(nesterov), 0 if momentum_done else int(maximize), int(cautious_wd), int(has_var),
        int(all(x % 16 == 0 for row in ptrs[:3] for x in row)),
    ]
    floats = [float(momentum), float(lr_eff), float(weight_decay)]

    with nvtx("dmb.owner.pack"):
        ws.barrier()  # every reader of the previous batch's results is done
        C_.dist_pack(meta64, meta32, peer_base, ints, floats, not momentum_done, has_var)
        ws.barrier()  # all shards have landed in the owners' workspaces

    mine = max(0, min(Bo, S - rank * Bo))
    if mine > 0:
        def region(off, n, dtype, shape):
            return buf[off : off + n].view(dtype).view(shape)

        x = region(x_off, mine * slot_bytes, torch.bfloat16, (mine, lay.Np, lay.Mp))
        x2 = region(x2_off, mine * slot_bytes, torch.bfloat16, (mine, lay.Np, lay.Mp))
        sums = region(sums_off, Bo * world * 4, torch.float32, (Bo, world))[:mine].contiguous()
        inv = C_.norm_finalize(sums, fac, eps)
        a_ws = WORKSPACE.get(device, "a", (mine, lay.Np, lay.Np))
        b_ws = WORKSPACE.get(device, "b", (mine, lay.Np, lay.Np))
        res = C_.ortho_iterate(x, x2, a_ws, b_ws, inv, coeffs, 0)
        if has_var:
            rowsq = C_.row_sumsq(res, lay.transpose, R, C)
            vbase = buf.data_ptr() + vbuf_off
            vptrs = torch.tensor([vbase + s * R * 4 for s in range(mine)], dtype=torch.int64).pin_memory()
            rowscale = C_.normuon_finalize(rowsq, vptrs.to(device, non_blocking=True), C, muon_beta2)
            region(rs_off, mine * R * 4, torch.float32, (mine, R)).copy_(rowscale)
    with nvtx("dmb.owner.apply"):
        ws.barrier()  # owners' results are ready
        C_.dist_apply(meta64, meta32, peer_base, ints, floats, has_var)


def fsdp3d_local_eligible(params, grads, buffers) -> bool:
    """3-D DTensors sharded only on dim 0: local shards are whole matrices."""
    from ..orthogonalize import is_fsdp_3d_sharded
    from ..ops import muon_fused

    if not is_fsdp_3d_sharded(list(grads)):
        return False
    return muon_fused.native_eligible(
        [p.to_local() for p in params], [g.to_local() for g in grads], [b.to_local() for b in buffers]
    ) and all(isinstance(t, DTensor) for t in list(params) + list(buffers))
