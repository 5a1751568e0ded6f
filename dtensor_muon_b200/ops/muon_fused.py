"""Fused native Muon / NorMuon update for a batch of same-shape CUDA tensors.

One step of the reference's ``MuonBaseline.foreach_update`` /
``NorMuon.foreach_update`` (src/muonium/optim/algorithms/muon.py:79-140,
normuon.py:147-203) as a short fixed sequence of sm_100a kernels:

    muon_pack       buf = m buf + g ; g' = g + m buf  -> bf16 workspace (+ sum of squares)
    norm_finalize   1 / (||g'|| fac + eps)
    ortho_iterate   steps x (Gram, polynomial, B X) tcgen05 GEMMs
    [row_sumsq + normuon_finalize   NorMuon only]
    muon_apply      cautious / plain WD and p -= lr * lr_ratio * u, in place

Nothing is materialised in the parameter layout between the momentum update
and the parameter write: g' and u live only in the padded workspace.
"""

from __future__ import annotations

from collections import defaultdict

import torch
from torch import Tensor
from torch.distributed.tensor import DTensor

from ..utils.tracing import nvtx
from . import _ext
from .ortho import (
    WORKSPACE,
    batch_chunk,
    coefficient_table,
    dtype_code,
    layout_for,
    norm_factor,
    ptr_tensor,
    run_iteration,
)

_FLOAT_DTYPES = (torch.float32, torch.bfloat16)


def native_eligible(params: list[Tensor], grads: list[Tensor], buffers: list[Tensor]) -> bool:
    """Whether a batch can take the fused kernel path."""
    if not params or not _ext.available():
        return False
    for p, g, b in zip(params, grads, buffers, strict=True):
        if isinstance(p, DTensor) or isinstance(g, DTensor) or isinstance(b, DTensor):
            return False
        if not (p.is_cuda and g.is_cuda and b.is_cuda):
            return False
        if p.dtype not in _FLOAT_DTYPES or g.dtype not in _FLOAT_DTYPES or b.dtype != torch.float32:
            return False
        if not (p.is_contiguous() and g.is_contiguous() and b.is_contiguous()):
            return False
        if g.ndim < 2 or p.numel() != g.numel() or b.shape != g.shape:
            return False
    return True


def _matrix_ptrs(t: Tensor, R: int, C: int) -> list[int]:
    n = t.numel() // (R * C)
    step = R * C * t.element_size()
    base = t.data_ptr()
    return [base + i * step for i in range(n)]


def fused_muon_update(
    params: list[Tensor],
    grads: list[Tensor],
    buffers: list[Tensor],
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
    variances: list[Tensor] | None = None,
    muon_beta2: float = 0.95,
    momentum_done: bool = False,
) -> None:
    """Run one fused Muon (or NorMuon, when ``variances`` is given) step in place.

    ``grads`` are the (possibly flattened) gradient views [..., R, C];
    ``params`` have the same number of elements in the same order. With
    ``momentum_done`` the ``grads`` already hold the orthogonalisation input
    g' (e.g. written by the quantised-state momentum kernel) and ``buffers``
    are ignored.
    """
    C_ = _ext.load()
    coefficient_table(strategy, ns_steps)  # validate
    R, C = grads[0].shape[-2], grads[0].shape[-1]
    if R == 0 or C == 0:
        return
    device = grads[0].device
    lay = layout_for(R, C)
    fac = norm_factor(strategy)

    # Flatten to per-matrix entries, grouped by (lr_eff, param dtype, grad dtype).
    groups: dict[tuple, list[tuple[int, int, int, int | None]]] = defaultdict(list)
    if momentum_done:
        buffers = list(grads)
    for i, (p, g, b) in enumerate(zip(params, grads, buffers, strict=True)):
        key = (float(lr_effs[i]), p.dtype, g.dtype)
        vp = _matrix_ptrs(variances[i], R, 1) if variances is not None else None
        for j, (pp, gp, bp) in enumerate(
            zip(_matrix_ptrs(p, R, C), _matrix_ptrs(g, R, C), _matrix_ptrs(b, R, C), strict=True)
        ):
            groups[key].append((pp, gp, bp, vp[j] if vp is not None else None))

    with nvtx(f"dmb.muon_fused[{R}x{C}]"):
        _run_groups(C_, groups, lay, R, C, device, fac, eps, ns_steps, strategy, momentum, nesterov, maximize,
                    weight_decay, cautious_wd, variances, muon_beta2, momentum_done)


def _run_groups(C_, groups, lay, R, C, device, fac, eps, ns_steps, strategy, momentum, nesterov, maximize,
                weight_decay, cautious_wd, variances, muon_beta2, momentum_done):
    for (lr_eff, pdt, gdt), entries in groups.items():
        chunk = batch_chunk(lay, len(entries))
        for s in range(0, len(entries), chunk):
            part = entries[s : s + chunk]
            B = len(part)
            x = WORKSPACE.get(device, "x", (B, lay.Np, lay.Mp))
            packed = ptr_tensor([e[1] for e in part] + [e[2] for e in part] + [e[0] for e in part], device)
            gptrs, bptrs, pptrs = packed[:B], packed[B : 2 * B], packed[2 * B :]
            # 16-byte vector I/O only when every matrix pointer is aligned
            # (views into sharded / flat storage need not be).
            vec_ok = all(e[i] % 16 == 0 for e in part for i in range(3))
            if momentum_done:
                partial = C_.muon_pack_ex(
                    gptrs, None, dtype_code(gdt), R, C, C, lay.transpose, x, 0.0, False, False, vec_ok
                )
            else:
                partial = C_.muon_pack_ex(
                    gptrs, bptrs, dtype_code(gdt), R, C, C, lay.transpose, x, momentum, nesterov, maximize, vec_ok
                )
            inv = C_.norm_finalize(partial, fac, eps)
            res = run_iteration(x, inv, lay, ns_steps, strategy)
            mat_scale = inv if ns_steps == 0 else None
            rowscale = None
            if variances is not None:
                rowsq = C_.row_sumsq(res, lay.transpose, R, C)
                if mat_scale is not None:
                    rowsq.mul_(mat_scale.view(-1, 1).square())
                vptrs = ptr_tensor([e[3] for e in part], device)
                rowscale = C_.normuon_finalize(rowsq, vptrs, C, muon_beta2)
            C_.muon_apply_ex(
                res,
                lay.transpose,
                R,
                C,
                C,
                pptrs,
                dtype_code(pdt),
                rowscale,
                mat_scale,
                lr_eff,
                float(weight_decay),
                bool(cautious_wd),
                vec_ok,
            )
