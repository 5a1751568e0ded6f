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
    2. all-reduce of G over the group: P2P push of the partial into every
       peer's staging slot, one bounded device barrier, fp32 sum of the W slots
    3. B = c G^2 + b G (every rank, replicated; C x C)
    4. X_r <- a X_r + X_r B on the local rows (tcgen05 kernel)

The Frobenius normalisation all-reduces one partial sum of squares per
matrix the same way. No update reduce-scatter is needed: every rank finishes
with exactly its own rows of the orthogonalised matrix and applies them in
place. Per iteration a rank moves (W - 1) C^2 bf16 values over NVLink and does
2 n_r C^2 + 2 C^3 multiply-adds, against 3 R C^2 (R >= C) for one owner.
"""

from __future__ import annotations

import math
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
    """Row-sharded 2-D Muon batches (each rank holds full rows) with R >= C."""
    if _FORCE == "0" or variances is not None or not params or not symm.available():
        return False
    g0 = grads[0]
    if not isinstance(g0, DTensor) or g0.ndim != 2 or g0.device_mesh.device_type != "cuda":
        return False
    lay = shard_layout(g0)
    if lay is None or lay.c0 != 0 or lay.c1 != g0.shape[1] or lay.world < 2:
        return False
    R, C = g0.shape
    if R < C:
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


class _AllReduce:
    """Sum of a device tensor over the group through a double-buffered staging
    region in symmetric memory (push, barrier, local fp32 slot sum)."""

    def __init__(self, ws):
        self.ws = ws
        self.calls = 0

    def __call__(self, t: Tensor) -> None:
        ws = self.ws
        flat = t.view(-1)
        nbytes = flat.numel() * flat.element_size()
        assert nbytes % 16 == 0 and flat.numel() % 8 == 0
        half = ws.world * nbytes
        buf, peers = ws.buffer(2 * half)
        off = (self.calls % 2) * half
        self.calls += 1
        C = _ext.load()
        C.push_slots(flat, peers, off, nbytes, ws.rank, ws.world, False, COMM_CTAS)
        ws.barrier()  # every rank's partial has landed in every staging
        C.local_slot_sum(flat, buf, off, ws.world, 1.0, 2 * COMM_CTAS)


_REDUCERS: dict[int, _AllReduce] = {}


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
    reduce_ = _REDUCERS.setdefault(id(ws), _AllReduce(ws))
    B = len(params)
    Cp, Mp = round_up(C, 256), round_up(max(n_r, 1), 256)
    x = WORKSPACE.get(device, "shx", (B, Cp, Mp))
    x2 = WORKSPACE.get(device, "shx2", (B, Cp, Mp))
    a_ws = WORKSPACE.get(device, "sha", (B, Cp, Cp))
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
    sums = torch.zeros(8 * math.ceil(B / 8), dtype=torch.float32, device=device)
    sums[:B] = sumsq
    reduce_(sums)
    inv = 1.0 / (sums[:B].sqrt() * norm_factor(strategy) + eps)
    c = coeffs.tolist()
    cur, nxt = x, x2
    for s in range(ns_steps):
        first = s == 0
        sc = inv if first else None
        C_.gram_sym2(cur, a_ws, None, sc, 1.0, 0.0, 2 if first else 0, 0)  # partial G = s^2 X_r^T X_r
        reduce_(a_ws)
        C_.gram_sym2(a_ws, b_ws, a_ws, None, c[s][2], c[s][1], 0, 0)  # B = c G^2 + b G
        C_.gemm_ax2(b_ws, cur, nxt, cur, sc, 1.0, c[s][0], 1 if first else 0, 1 if first else 0)
        cur, nxt = nxt, cur
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
