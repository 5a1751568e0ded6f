"""Sharded orthogonalisation: Newton-Schulz / Polar Express on row-sharded
matrices without gathering them, with the partial-Gram all-reduce over peer memory.

The reference always brings whole matrices to one rank: a full-tensor gather
in ``zeropower`` and a stack + redistribute in ``foreach_zeropower``
(src/muonium/orthogonalize/orthogonalize.py:95-100, :140-155). Owner compute
(:mod:`.owner_compute`) does the same over NVLink and is the right choice when
a batch has at least as many matrices as ranks. When it has far fewer, most
ranks would idle; then this path runs instead. It uses the right-multiplied
form of the iteration, which is identical to the usual one,

    X <- a X + (b A + c A^2) X,  A = X X^T   ==   X <- a X + X (b G + c G^2),  G = X^T X,

because X (X^T X)^k = (X X^T)^k X. With X's rows spread over the ranks,
G = sum_r X_r^T X_r is a sum of per-rank partial Grams, so each iteration is:

    1. partial Gram of the local rows (tcgen05 kernel, epilogue-scaled on step 1)
    2. all-reduce of G over the group, in place in symmetric memory (the Gram
       kernel writes its partial there): NVLS ``multimem`` reduce + broadcast
       through the switch where multicast is available, else P2P loads/stores
    3. B = c G^2 + b G (every rank, replicated; C x C)
    4. X_r <- a X_r + X_r B on the local rows (tcgen05 kernel)

The Frobenius normalisation all-reduces one partial sum of squares per
matrix the same way. No update reduce-scatter is needed: every rank finishes
with exactly its own rows of the orthogonalised matrix and applies them in
place. Per iteration a rank moves (W - 1) C^2 bf16 values over NVLink and does
2 n_r C^2 + 2 C^3 multiply-adds, against 3 R C^2 (R >= C) for one owner.
"""

from __future__ import annotations

import os

import torch
from torch import Tensor
from torch.distributed.tensor import DTensor

from ..ops import _ext
from ..ops.ortho import WORKSPACE, coefficient_table, dtype_code, norm_factor, ptr_tensor, round_up
from . import symm
from .owner_compute import shard_layout

# Force the sharded path for every eligible batch ("1"), never ("0"), or let the
# cost rule decide (unset).
_FORCE = os.environ.get("DMB_SHARDED_NS")
COMM_CTAS = int(os.environ.get("DMB_COMM_CTAS", "64"))


def eligible(params, grads, buffers, variances=None) -> bool:
    """Row-sharded 2-D Muon batches (each rank holds full rows) with R >= 2 C
    (R >= C when forced)."""
    if _FORCE == "0" or variances is not None or not params or not symm.available():
        return False
    g0 = grads[0]
    if not isinstance(g0, DTensor) or g0.ndim != 2 or g0.device_mesh.device_type != "cuda":
        return False
    lay = shard_layout(g0)
    if lay is None or lay.c0 != 0 or lay.c1 != g0.shape[1] or lay.world < 2:
        return False
    R, C = g0.shape
    # every rank repeats the C x C polynomial (2 C^3 per iteration) and the
    # Gram all-reduce; splitting the 4 R C^2 of the other two GEMMs pays for
    # that only for tall matrices (measured at W = 2: 14336 x 4096 sharded
    # 2.45 ms vs 3.30 ms on one GPU; 4096 x 4096 sharded 1.59 ms vs 1.2 ms)
    if R < (C if _FORCE == "1" else 2 * C):
        return False
    if _FORCE != "1" and 2 * len(params) > lay.world:  # enough matrices for owner compute
        return False
    shape = (lay.r1 - lay.r0, C)
    for t in list(params) + list(grads) + list(buffers):
        if not isinstance(t, DTensor) or tuple(t.placements) != tuple(g0.placements):
            return False
        loc = t.to_local()
        if not loc.is_cuda or not loc.is_contiguous() or tuple(loc.shape) != shape:
            return False
    if any(b.dtype != torch.float32 for b in buffers):
        return False
    dts = (torch.float32, torch.bfloat16)
    return (all(p.dtype in dts for p in params) and all(g.dtype in dts for g in grads)
            and len({p.dtype for p in params}) == 1 and len({g.dtype for g in grads}) == 1)


class _Region:
    """The batch's Gram and norm buffers placed in symmetric memory, so the
    partial Gram kernel writes straight into the memory the all-reduce reads.

    The all-reduce is in place: one bounded barrier (every partial written),
    ``allreduce_inplace`` (rank r sums chunk r over all ranks and writes the sum
    to every rank: NVLS ``multimem.ld_reduce`` / ``multimem.st`` when the buffer
    has an NVSwitch multicast address, P2P loads and stores otherwise), and a
    second barrier (every sum visible; nobody rewrites a chunk a peer still reads).
    """

    def __init__(self, ws, B: int, Cp: int):
        self.ws = ws
        self.a_bytes = B * Cp * Cp * 2
        self.s_bytes = 256
        buf, self.peers = ws.buffer(self.a_bytes + self.s_bytes)
        self.a = buf[: self.a_bytes].view(torch.bfloat16).view(B, Cp, Cp)
        self.sums = buf[self.a_bytes : self.a_bytes + self.s_bytes].view(torch.float32)

    def allreduce(self, off: int, nbytes: int, dtype_code: int) -> None:
        ws = self.ws
        ws.barrier()
        _ext.load().allreduce_inplace(self.peers, off, nbytes, dtype_code, ws.rank, ws.world, ws.mc_base,
                                      2 * COMM_CTAS)
        ws.barrier()



def _iterate(C_, region, x, x2, b_ws, sumsq, B, coeffs, ns_steps, strategy, eps):
    """The all-reduced normalisation and ``ns_steps`` sharded iterations on the
    packed local rows ``x`` (X_r^T); returns the result buffer and 1/||X||."""
    a_ws = region.a
    region.sums.zero_()
    region.sums[:B] = sumsq
    region.allreduce(region.a_bytes, region.s_bytes, 0)
    inv = 1.0 / (region.sums[:B].sqrt() * norm_factor(strategy) + eps)
    c = coeffs.tolist()
    cur, nxt = x, x2
    for s in range(ns_steps):
        first = s == 0
        sc = inv if first else None
        C_.gram_sym2(cur, a_ws, None, sc, 1.0, 0.0, 2 if first else 0, 0)  # partial G = s^2 X_r^T X_r
        region.allreduce(0, region.a_bytes, 1)
        C_.gram_sym2(a_ws, b_ws, a_ws, None, c[s][2], c[s][1], 0, 0)  # B = c G^2 + b G
        C_.gemm_ax2(b_ws, cur, nxt, cur, sc, 1.0, c[s][0], 1 if first else 0, 1 if first else 0)
        cur, nxt = nxt, cur
    return cur, inv


def sharded_update(
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
    momentum_done: bool = False,
) -> None:
    """One Muon step of a row-sharded batch; every rank updates its own rows in place."""
    C_ = _ext.load()
    coeffs = coefficient_table(strategy, ns_steps)
    sl = shard_layout(grads[0])
    R, C = grads[0].shape
    n_r = sl.r1 - sl.r0
    device = grads[0].to_local().device
    ws = symm.workspace_for(sl.group, device, "sharded_ns")
    B = len(params)
    if B > 64:
        raise ValueError("sharded orthogonalisation takes at most 64 matrices per batch")
    Cp, Mp = round_up(C, 256), round_up(max(n_r, 1), 256)
    region = _Region(ws, B, Cp)
    x = WORKSPACE.get(device, "shx", (B, Cp, Mp))
    x2 = WORKSPACE.get(device, "shx2", (B, Cp, Mp))
    a_ws = region.a
    b_ws = WORKSPACE.get(device, "shb", (B, Cp, Cp))
    loc = [(p.to_local(), g.to_local(), b.to_local()) for p, g, b in zip(params, grads, buffers, strict=True)]
    vec_ok = all(t.data_ptr() % 16 == 0 for trip in loc for t in trip)
    ptrs = ptr_tensor([t[1].data_ptr() for t in loc] + [t[2].data_ptr() for t in loc]
                      + [t[0].data_ptr() for t in loc], device)
    gptrs, bptrs, pptrs = ptrs[:B], ptrs[B : 2 * B], ptrs[2 * B :]
    gdt, pdt = dtype_code(loc[0][1].dtype), dtype_code(loc[0][0].dtype)
    if n_r > 0:
        # local rows, transposed: x[b] = X_r^T (C x n_r), zero-padded
        if momentum_done:
            partial = C_.muon_pack_ex(gptrs, None, gdt, n_r, C, C, True, x, 0.0, False, False, vec_ok)
        else:
            partial = C_.muon_pack_ex(gptrs, bptrs, gdt, n_r, C, C, True, x, momentum, nesterov, maximize, vec_ok)
        sumsq = partial.sum(dim=1)
    else:
        x.zero_()
        sumsq = torch.zeros(B, dtype=torch.float32, device=device)
    cur, inv = _iterate(C_, region, x, x2, b_ws, sumsq, B, coeffs, ns_steps, strategy, eps)
    if n_r == 0:
        return
    mat_scale = inv if ns_steps == 0 else None
    for lr in sorted(set(float(e) for e in lr_effs)):
        idx = [i for i, e in enumerate(lr_effs) if float(e) == lr]
        if len(idx) == B:
            res, pp = cur, pptrs
        else:
            sel = torch.tensor(idx, device=device)
            res, pp = cur.index_select(0, sel), pptrs.index_select(0, sel)
        ms = mat_scale.index_select(0, torch.tensor(idx, device=device)) if mat_scale is not None and len(idx) != B \
            else mat_scale
        C_.muon_apply_ex(res, True, n_r, C, C, pp, pdt, None, ms, lr, float(weight_decay), bool(cautious_wd),
                         vec_ok)


def zeropower_eligible(gs: list) -> bool:
    """A batch of row-sharded 2-D CUDA DTensors the orthogonalisation-only
    entry (:func:`sharded_zeropower`) takes: same rule as the optimizer path."""
    if not gs or not all(isinstance(g, DTensor) for g in gs):
        return False
    return eligible(gs, gs, [], None) and all(g.to_local().dtype in (torch.float32, torch.bfloat16) for g in gs)


def sharded_zeropower(gs: list[DTensor], steps: int, strategy: str, eps: float = 1e-7) -> list[DTensor]:
    """Orthogonalise row-sharded matrices without gathering them; returns bf16
    DTensors with the inputs' placements (each rank computes its own rows)."""
    C_ = _ext.load()
    coeffs = coefficient_table(strategy, steps)
    sl = shard_layout(gs[0])
    R, C = gs[0].shape
    n_r = sl.r1 - sl.r0
    device = gs[0].to_local().device
    ws = symm.workspace_for(sl.group, device, "sharded_ns")
    B = len(gs)
    if B > 64:
        raise ValueError("sharded orthogonalisation takes at most 64 matrices per batch")
    Cp, Mp = round_up(C, 256), round_up(max(n_r, 1), 256)
    region = _Region(ws, B, Cp)
    x = WORKSPACE.get(device, "shx", (B, Cp, Mp))
    x2 = WORKSPACE.get(device, "shx2", (B, Cp, Mp))
    b_ws = WORKSPACE.get(device, "shb", (B, Cp, Cp))
    loc = [g.to_local().contiguous() for g in gs]
    if len({t.dtype for t in loc}) != 1:
        loc = [t.float() for t in loc]
    if n_r > 0:
        ptrs = ptr_tensor([t.data_ptr() for t in loc], device)
        vec_ok = all(t.data_ptr() % 16 == 0 for t in loc)
        sumsq = C_.muon_pack_ex(ptrs, None, dtype_code(loc[0].dtype), n_r, C, C, True, x, 0.0, False, False,
                                vec_ok).sum(dim=1)
    else:
        x.zero_()
        sumsq = torch.zeros(B, dtype=torch.float32, device=device)
    cur, inv = _iterate(C_, region, x, x2, b_ws, sumsq, B, coeffs, steps, strategy, eps)
    if n_r > 0:
        out = C_.muon_unpack(cur, True, n_r, C, inv if steps == 0 else None)
    else:
        out = torch.empty(B, 0, C, dtype=torch.bfloat16, device=device)
    meta = dict(device_mesh=gs[0].device_mesh, placements=gs[0].placements, shape=gs[0].shape,
                stride=gs[0].stride(), run_check=False)
    return [DTensor.from_local(o, **meta) for o in out.unbind(0)]


def sharded_reference(shards: list[Tensor], steps: int, strategy: str, eps: float = 1e-7) -> list[Tensor]:
    """PyTorch statement of the sharded iteration (fp32, no communication): the
    row blocks ``shards`` of one matrix in, their orthogonalised blocks out. Used
    as the CPU oracle for the algorithm; equals the gathered iteration up to rounding."""
    coeffs = coefficient_table(strategy, steps).tolist()
    xs = [s.float() for s in shards]
    norm = torch.sqrt(sum((x * x).sum() for x in xs))
    xs = [x / (norm * norm_factor(strategy) + eps) for x in xs]
    for a, b, c in coeffs:
        G = sum(x.mT @ x for x in xs)  # the all-reduced partial Grams
        Bm = b * G + c * (G @ G)
        xs = [a * x + x @ Bm for x in xs]
    return xs
