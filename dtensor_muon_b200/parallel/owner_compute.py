"""Owner-compute Muon for dim-0-sharded (FSDP) 2-D DTensors, fused over NVLink.

Same distribution as the reference's general path (whole matrices assigned
to owner ranks, src/muonium/orthogonalize/orthogonalize.py:140-155), but the
two NCCL all-to-alls are gone: each rank writes its momentum-updated row shard
straight into the owner's workspace (P2P stores inside the momentum kernel),
the owner runs the local tcgen05 engine, and each rank pulls its rows of the
result back (P2P loads inside the apply kernel). Sequence per batch:

    barrier | dist_pack (+ sums push) | barrier | owner: finalize + ortho [+ NorMuon] | barrier | dist_apply

Matrices are assigned in contiguous chunks (matrix b -> rank b // ceil(B/W)),
like a Shard(0) of the stacked batch. Inside :class:`deferred` (the Muon step
uses it) all batches of the step run as one pipeline (:func:`_run_phases`):
one barrier, then per-batch arrival / completion signals.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor
from torch.distributed.tensor import DTensor, Replicate, Shard

from ..ops import _ext
from ..ops.ortho import WORKSPACE, coefficient_table, dtype_code, layout_for, norm_factor
from ..utils.tracing import nvtx
from . import symm

# Cap on one owner's share of the symmetric workspace (two ping-pong buffers).
MAX_OWNER_BYTES = 8 << 30


def _rows(R: int, world: int, rank: int) -> tuple[int, int]:
    chunk = -(-R // world)
    return min(rank * chunk, R), min((rank + 1) * chunk, R)


def shard_dim(placements) -> int | None:
    """Mesh dim that shards tensor dim 0 when every other mesh dim replicates
    (FSDP: ``(Shard(0),)``; HSDP: ``(Replicate(), Shard(0))``), else None."""
    dims = [i for i, pl in enumerate(placements) if pl == Shard(0)]
    if len(dims) != 1 or any(pl != Replicate() for i, pl in enumerate(placements) if i != dims[0]):
        return None
    return dims[0]


@dataclass(frozen=True)
class ShardLayout:
    """Where this rank's local shard sits in the global matrix, and the group of
    ranks that together hold every block of it (owner compute runs over that group).

    * FSDP ``(Shard(0),)`` / HSDP ``(Replicate(), Shard(0))``: row blocks over the
      shard dim's group; the replicas of an HSDP mesh each run their own group.
    * FSDP x TP ``(_StridedShard(0) | Shard(0), Shard(0) | Shard(1))`` on a mesh
      that spans the whole job: every rank holds one rectangle (a row block of a
      column-parallel weight, or a row x column block of a row-parallel one),
      and the group is the whole job.
    """

    group: object
    world: int
    rank: int
    r0: int
    r1: int
    c0: int
    c1: int


def _is_shard(pl) -> bool:
    from torch.distributed.tensor.placement_types import _StridedShard

    return isinstance(pl, (Shard, _StridedShard))


def shard_layout(t: DTensor) -> ShardLayout | None:
    import torch.distributed as dist
    from torch.distributed.tensor._utils import compute_local_shape_and_global_offset

    mesh, pls = t.device_mesh, tuple(t.placements)
    if t.ndim != 2:
        return None
    d = shard_dim(pls)
    R, C = t.shape
    if d is not None and type(pls[d]) is Shard:
        world, rank = mesh.size(d), mesh.get_local_rank(d)
        r0, r1 = _rows(R, world, rank)
        return ShardLayout(mesh.get_group(d), world, rank, r0, r1, 0, C)
    if not all(_is_shard(pl) and pl.dim in (0, 1) for pl in pls) or mesh.size() != dist.get_world_size():
        return None
    shape, off = compute_local_shape_and_global_offset(t.shape, mesh, pls)
    r0, c0 = int(off[0]), int(off[1])
    return ShardLayout(dist.group.WORLD, dist.get_world_size(), dist.get_rank(), r0, r0 + int(shape[0]), c0,
                       c0 + int(shape[1]))


def eligible(params: list[Tensor], grads: list[Tensor], buffers: list[Tensor], variances=None) -> bool:
    """2-D DTensors whose local shards are rectangles of the global matrix
    (:class:`ShardLayout`). With replica dims (HSDP) each replica group runs owner
    compute over its own shard group; the replicas hold identical gradients (FSDP
    reduced them across replicas), so they compute identical updates, as the
    reference's stack + redistribute does (src/muonium/orthogonalize/orthogonalize.py:140-155)."""
    if not params or not symm.available():
        return False
    g0 = grads[0]
    if not isinstance(g0, DTensor) or g0.ndim != 2:
        return False
    mesh = g0.device_mesh
    pls = tuple(g0.placements)
    if mesh.device_type != "cuda":
        return False
    lay = shard_layout(g0)
    if lay is None:
        return False
    shape = (lay.r1 - lay.r0, lay.c1 - lay.c0)
    tensors = list(params) + list(grads) + list(buffers)
    for t in tensors:
        if not isinstance(t, DTensor) or t.device_mesh != mesh or tuple(t.placements) != pls:
            return False
        loc = t.to_local()
        if not loc.is_cuda or not loc.is_contiguous() or tuple(loc.shape) != shape:
            return False
    if variances is not None:
        # NorMuon's per-row variance: one value per global row, sharded like the rows
        for v in variances:
            if not isinstance(v, DTensor) or v.device_mesh != mesh:
                return False
            loc = v.to_local()
            if not loc.is_cuda or not loc.is_contiguous() or loc.numel() != lay.r1 - lay.r0:
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
    sl = shard_layout(grads[0])
    world, rank = sl.world, sl.rank
    R, C = grads[0].shape
    lay = layout_for(R, C)
    device = grads[0].to_local().device
    ws = symm.workspace_for(sl.group, device)
    rpad, cpad = (lay.Mp, lay.Np) if lay.transpose else (lay.Np, lay.Mp)
    grp = _Group(
        C_=_ext.load(), lay=lay, R=R, C=C, rank=rank, world=world, r0=sl.r0, r1=sl.r1,
        g1=rpad if sl.r1 == R else sl.r1, c0=sl.c0, c1=sl.c1, h1=cpad if sl.c1 == C else sl.c1,
        coeffs=coefficient_table(strategy, ns_steps), fac=norm_factor(strategy), eps=eps,
        weight_decay=weight_decay, cautious_wd=cautious_wd, momentum=momentum, nesterov=nesterov,
        maximize=maximize, muon_beta2=muon_beta2, has_var=variances is not None, device=device,
        momentum_done=momentum_done, gdt=dtype_code(grads[0].dtype), pdt=dtype_code(params[0].dtype),
    )

    # Batches with a common lr_eff; chunk so one owner's workspace stays bounded.
    per_slot = 2 * lay.Np * lay.Mp * 2
    step = world * max(1, MAX_OWNER_BYTES // per_slot)
    order: dict[float, list[int]] = {}
    for i, lr in enumerate(lr_effs):
        order.setdefault(float(lr), []).append(i)
    specs = [
        _Spec(grp, idxs[s : s + step], params, grads, buffers, variances, lr_eff)
        for lr_eff, idxs in order.items()
        for s in range(0, len(idxs), step)
    ]
    _enqueue(ws, specs)


# Deferred execution: inside ``deferred()`` every owner-compute batch of the
# optimizer step is queued; at exit all batches share one symmetric buffer and
# run phase by phase (all packs | barrier | all owner GEMMs | barrier | all
# applies), so the step pays three barriers instead of three per batch and the
# packs' NVLink traffic drains together.
_DEFER: dict = {}
MAX_DEFERRED_BYTES = 32 << 30


class deferred:
    def __enter__(self):
        self._prev = _DEFER.get("on", False)
        _DEFER["on"] = True
        return self

    def __exit__(self, exc_type, exc, tb):
        _DEFER["on"] = self._prev
        pending = _DEFER.pop("pending", {}) if not self._prev else {}
        if exc_type is None:
            for ws, specs in pending.values():
                if specs:
                    _run_phases(ws, specs)
        return False


def _enqueue(ws, specs: list) -> None:
    """Queue ``specs`` inside :class:`deferred` (flushing once the queue exceeds
    ``MAX_DEFERRED_BYTES``); outside it, run each batch at once."""
    if _DEFER.get("on"):
        pend = _DEFER.setdefault("pending", {}).setdefault(id(ws), (ws, []))[1]
        pend.extend(specs)
        if sum(sp.nbytes for sp in pend) > MAX_DEFERRED_BYTES:
            flush(ws)
        return
    for sp in specs:
        _run_phases(ws, [sp])


def flush(ws) -> None:
    pend = _DEFER.get("pending", {}).pop(id(ws), None)
    if pend and pend[1]:
        _run_phases(pend[0], pend[1])


@dataclass(frozen=True)
class _Group:
    """What every batch of one owner_compute_update call shares."""

    C_: object
    lay: object
    R: int
    C: int
    rank: int
    world: int
    r0: int
    r1: int
    g1: int
    c0: int
    c1: int
    h1: int
    coeffs: Tensor
    fac: float
    eps: float
    weight_decay: float
    cautious_wd: bool
    momentum: float
    nesterov: bool
    maximize: bool
    muon_beta2: float
    has_var: bool
    device: torch.device
    momentum_done: bool
    gdt: int
    pdt: int


_TABLES: dict[tuple, tuple[Tensor, Tensor]] = {}
_TABLES_MAX = 512


def _tables(ptrs: list[list[int]], S: int, Bo: int, device) -> tuple[Tensor, Tensor]:
    """Device pointer / owner tables of a batch, cached by content: parameters,
    momentum buffers and (usually) gradients keep their addresses from step to
    step, so the steady state makes no host-to-device copy here."""
    key = (str(device), Bo, tuple(x for row in ptrs for x in row))
    hit = _TABLES.get(key)
    if hit is None:
        if len(_TABLES) >= _TABLES_MAX:
            _TABLES.pop(next(iter(_TABLES)))
        meta64 = torch.tensor(ptrs, dtype=torch.int64).pin_memory().to(device, non_blocking=True)
        owner_slot = [[b // Bo for b in range(S)], [b % Bo for b in range(S)]]
        meta32 = torch.tensor(owner_slot, dtype=torch.int32).pin_memory().to(device, non_blocking=True)
        hit = _TABLES[key] = (meta64, meta32)
    return hit


class _Spec:
    """One owner-compute batch: pointer tables, symmetric-buffer layout, kernel arguments."""

    def __init__(self, g: _Group, sel, params, grads, buffers, variances, lr_eff: float):
        self.g = g
        S = len(sel)
        self.Bo = Bo = math.ceil(S / g.world)
        self.mine = max(0, min(Bo, S - g.rank * Bo))
        self.slot_bytes = g.lay.Np * g.lay.Mp * 2
        rows = Bo * g.R * 4 if g.has_var else 0
        # Layout relative to this batch's base: sums | vbuf | rowscale | x | x2
        self.sums_rel = 0
        self.vbuf_rel = _align(Bo * g.world * 4)
        self.rs_rel = _align(self.vbuf_rel + rows)
        self.x_rel = _align(self.rs_rel + rows)
        self.x2_rel = _align(self.x_rel + Bo * self.slot_bytes)
        self.nbytes = _align(self.x2_rel + Bo * self.slot_bytes)
        ptrs = [
            [grads[i].to_local().data_ptr() for i in sel],
            [buffers[i].to_local().data_ptr() for i in sel],
            [params[i].to_local().data_ptr() for i in sel],
            [variances[i].to_local().data_ptr() for i in sel] if g.has_var else [0] * S,
        ]
        self.meta64, self.meta32 = _tables(ptrs, S, Bo, g.device)
        self.floats = [float(g.momentum), float(lr_eff), float(g.weight_decay)]
        self.vec_ok = int(all(x % 16 == 0 for row in ptrs[:3] for x in row))

    def place(self, base: int) -> None:
        g, lay = self.g, self.g.lay
        self.base = base
        x_off, x2_off = base + self.x_rel, base + self.x2_rel
        res_off = x_off if g.coeffs.shape[0] % 2 == 0 else x2_off
        self.ints = [
            x_off, res_off, base + self.sums_rel, base + self.vbuf_rel, base + self.rs_rel,
            g.gdt, g.pdt, g.R, g.C, int(lay.transpose), lay.Np, lay.Mp, g.r0, g.r1, g.g1, g.rank, g.world,
            int(g.nesterov), 0 if g.momentum_done else int(g.maximize), int(g.cautious_wd), int(g.has_var),
            self.vec_ok, g.c0, g.c1, g.h1, g.c1 - g.c0,
        ]

    def pack(self, peer_base):
        g = self.g
        g.C_.dist_pack(self.meta64, self.meta32, peer_base, self.ints, self.floats, not g.momentum_done, g.has_var)

    def compute(self, buf):
        if self.mine == 0:
            return
        g, lay, mine, base = self.g, self.g.lay, self.mine, self.base
        C_ = g.C_

        def region(off, n, dtype, shape):
            return buf[base + off : base + off + n].view(dtype).view(shape)

        x = region(self.x_rel, mine * self.slot_bytes, torch.bfloat16, (mine, lay.Np, lay.Mp))
        x2 = region(self.x2_rel, mine * self.slot_bytes, torch.bfloat16, (mine, lay.Np, lay.Mp))
        sums = region(self.sums_rel, self.Bo * g.world * 4, torch.float32, (self.Bo, g.world))[:mine]
        inv = C_.norm_finalize(sums.contiguous(), g.fac, g.eps)
        a_ws = WORKSPACE.get(g.device, "a", (mine, lay.Np, lay.Np))
        b_ws = WORKSPACE.get(g.device, "b", (mine, lay.Np, lay.Np))
        res = C_.ortho_iterate(x, x2, a_ws, b_ws, inv, g.coeffs, 0)
        if g.has_var:
            R = g.R
            rowsq = C_.row_sumsq(res, lay.transpose, R, g.C)
            vbase = buf.data_ptr() + base + self.vbuf_rel
            vptrs = torch.tensor([vbase + s * R * 4 for s in range(mine)], dtype=torch.int64).pin_memory()
            rowscale = C_.normuon_finalize(rowsq, vptrs.to(g.device, non_blocking=True), g.C, g.muon_beta2)
            region(self.rs_rel, mine * R * 4, torch.float32, (mine, R)).copy_(rowscale)

    def apply(self, peer_base):
        self.g.C_.dist_apply(self.meta64, self.meta32, peer_base, self.ints, self.floats, self.g.has_var)


def _run_phases(ws, specs: list) -> None:
    """All batches of a step, pipelined with per-batch signals instead of
    step-wide barriers: one barrier (every reader of the previous step's results
    is done), then

        pack_j ; signal(arrived_j)                     for every batch j
        wait(arrived_j) ; owner work_j ; signal(done_j) for every batch j
        wait(done_j) ; apply_j                          for every batch j

    An owner starts batch j as soon as every rank's shards of batch j have
    landed, and a rank applies batch j as soon as every owner finished it, so
    skew between ranks is absorbed per batch rather than at whole-step barriers.
    Slots 2j and 2j + 1 of the workspace's signal array are batch j's."""
    total, base = 0, []
    for sp in specs:
        base.append(total)
        total += sp.nbytes
    buf, peer_base = ws.buffer(total)
    for sp, b in zip(specs, base):
        sp.place(b)
    groups = [specs[i : i + ws.SIGNAL_SLOTS // 2] for i in range(0, len(specs), ws.SIGNAL_SLOTS // 2)]
    for grp in groups:
        ws.barrier()  # every reader of the previous results (and of these slots) is done
        epoch = ws.next_signal_epoch()
        with nvtx("dmb.owner.pack"):
            for j, sp in enumerate(grp):
                sp.pack(peer_base)
                ws.signal(2 * j, epoch)
        with nvtx("dmb.owner.compute"):
            for j, sp in enumerate(grp):
                ws.wait(2 * j, epoch)
                sp.compute(buf)
                ws.signal(2 * j + 1, epoch)
        with nvtx("dmb.owner.apply"):
            for j, sp in enumerate(grp):
                ws.wait(2 * j + 1, epoch)
                sp.apply(peer_base)


def fsdp3d_local_eligible(params, grads, buffers) -> bool:
    """3-D DTensors sharded only on dim 0: local shards are whole matrices."""
    from ..orthogonalize import is_fsdp_3d_sharded
    from ..ops import muon_fused

    if not is_fsdp_3d_sharded(list(grads)):
        return False
    return muon_fused.native_eligible(
        [p.to_local() for p in params], [g.to_local() for g in grads], [b.to_local() for b in buffers]
    ) and all(isinstance(t, DTensor) for t in list(params) + list(buffers))
