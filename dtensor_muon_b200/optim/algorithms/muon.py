"""Baseline Muon (Keller Jordan's Muon) with cautious weight decay.

Math of the reference's ``MuonBaseline`` (src/muonium/optim/algorithms/muon.py:15-140):

    buf = momentum * buf + g            (g negated when maximize)
    g'  = g + momentum * buf            (Nesterov) or buf
    u   = orthogonalize(g')             (bf16 result)
    u  += wd * p * [u * p > 0]          (cautious) or wd * p (plain)
    p  -= lr_ratio * lr * u

CUDA batches whose orthogonaliser is the built-in one run as the fused kernel
sequence of :mod:`dtensor_muon_b200.ops.muon_fused`; everything else (CPU,
DTensors, ``split_sizes``, a substituted orthogonaliser) runs the PyTorch
formulation below.
"""

from __future__ import annotations

import torch
from torch import Tensor

from ...ops import muon_fused
from . import base
from .base import MuonAlgorithm, orthogonalize_batch, orthogonalize_single, register_muon_algorithm


def fused_path_ok(params, grads, buffers, split_sizes) -> bool:
    return split_sizes is None and base._seams_are_builtin() and muon_fused.native_eligible(params, grads, buffers)


def distributed_fused(params, grads, buffers, lr_ratios, lr, split_sizes, ns_steps, kw, variances=None) -> bool:
    """Run the fused distributed path when the batch qualifies; returns whether it ran.

    * 2-D row-sharded DTensors with fewer matrices than ranks: sharded
      Newton-Schulz / Polar Express (:mod:`...parallel.sharded_ns`).
    * other 2-D DTensors whose shards are rectangles (FSDP, HSDP, FSDP x TP):
      owner compute over symmetric memory.
    * 3-D DTensors sharded only on dim 0: the local shards are whole matrices,
      so the single-GPU fused kernels run on them with no communication.
    """
    if split_sizes is not None or ns_steps < 1 or not base._seams_are_builtin():
        return False
    if not params or not hasattr(grads[0], "device_mesh"):
        return False
    from ...parallel import owner_compute

    from ...parallel.fsdp_comm import FUSED_GRADS

    effs = lr_effs(lr, lr_ratios)
    fused = [id(p) in FUSED_GRADS for p in params]
    from ...parallel import sharded_ns

    if sharded_ns.eligible(params, grads, buffers, variances):
        # Few matrices for many ranks: orthogonalise the row shards in place with
        # an all-reduced partial Gram per iteration instead of idling owners.
        for done in (False, True):
            idx = [i for i, f in enumerate(fused) if f == done]
            if idx:
                sharded_ns.sharded_update(
                    [params[i] for i in idx], [grads[i] for i in idx], [buffers[i] for i in idx],
                    [effs[i] for i in idx], ns_steps=ns_steps, momentum_done=done, **kw,
                )
        FUSED_GRADS.difference_update(id(p) for p in params)
        return True
    if owner_compute.eligible(params, grads, buffers, variances):
        # Grads whose momentum was applied inside the FSDP reduce-scatter hold g'.
        for done in (False, True):
            idx = [i for i, f in enumerate(fused) if f == done]
            if not idx:
                continue
            pick = lambda xs: [xs[i] for i in idx] if xs is not None else None  # noqa: E731
            owner_compute.owner_compute_update(
                pick(params), pick(grads), pick(buffers), pick(effs), ns_steps=ns_steps, variances=pick(variances),
                momentum_done=done, **kw,
            )
        FUSED_GRADS.difference_update(id(p) for p in params)
        return True
    if any(fused):
        raise RuntimeError("gradients with fused momentum reached a non-fused Muon path")
    if owner_compute.fsdp3d_local_eligible(params, grads, buffers) and (
        variances is None or all(hasattr(v, "to_local") for v in variances)
    ):
        muon_fused.fused_muon_update(
            [p.to_local() for p in params],
            [g.to_local() for g in grads],
            [b.to_local() for b in buffers],
            effs,
            ns_steps=ns_steps,
            variances=[v.to_local() for v in variances] if variances is not None else None,
            **kw,
        )
        return True
    return False


def lr_effs(lr: Tensor, lr_ratios: list[Tensor]) -> list[float]:
    lr_f = float(lr)
    return [float(r) * lr_f for r in lr_ratios]


def apply_weight_decay_and_step(p: Tensor, u: Tensor, lr_ratio, lr, weight_decay: float, cautious_wd: bool) -> None:
    """Per-tensor fp32 tail shared by the built-in algorithms."""
    p32 = p.to(torch.float32)
    if weight_decay != 0:
        decay = p32 * (u * p32 > 0) if cautious_wd else p32
        u = u + weight_decay * decay
    p.copy_(p32 - (lr_ratio * lr) * u)


def foreach_weight_decay_and_step(p: list[Tensor], u: list[Tensor], lr_ratios, lr, weight_decay, cautious_wd):
    """Batched tail in the parameter dtype (the reference's foreach semantics)."""
    scale = torch._foreach_mul(lr_ratios, lr)
    if weight_decay != 0:
        if cautious_wd:
            masked = [p_ * (u_ * p_ > 0).to(p_.dtype) for u_, p_ in zip(u, p, strict=True)]
            torch._foreach_add_(u, masked, alpha=weight_decay)
        else:
            torch._foreach_add_(u, p, alpha=weight_decay)
    torch._foreach_mul_(u, scale)
    torch._foreach_sub_(p, u)


@register_muon_algorithm
class MuonBaseline(MuonAlgorithm):
    """The original Muon update: momentum, orthogonalise, shape-scaled apply."""

    name = "muon"

    def update(
        self,
        param,
        grad,
        state,
        lr_ratio,
        *,
        lr,
        weight_decay,
        cautious_wd,
        momentum,
        nesterov,
        maximize,
        ns_steps,
        orthogonalization_strategy,
        split_sizes,
        **opts,
    ) -> None:
        buf = state["momentum_buffer"]
        if fused_path_ok([param], [grad], [buf], split_sizes):
            muon_fused.fused_muon_update(
                [param],
                [grad],
                [buf],
                lr_effs(lr, [lr_ratio]),
                weight_decay=weight_decay,
                cautious_wd=cautious_wd,
                momentum=momentum,
                nesterov=nesterov,
                maximize=maximize,
                ns_steps=ns_steps,
                strategy=orthogonalization_strategy,
            )
            return
        kw = dict(weight_decay=weight_decay, cautious_wd=cautious_wd, momentum=momentum, nesterov=nesterov,
                  maximize=maximize, strategy=orthogonalization_strategy)
        if distributed_fused([param], [grad], [buf], [lr_ratio], lr, split_sizes, ns_steps, kw):
            return
        g32 = (-grad if maximize else grad).to(torch.float32)
        new_buf = buf.to(torch.float32) * momentum + g32
        buf.copy_(new_buf)
        g_eff = g32 + momentum * new_buf if nesterov else new_buf
        u = orthogonalize_single(
            g_eff, ns_steps=ns_steps, strategy=orthogonalization_strategy, split_sizes=split_sizes
        )
        u = u.view_as(param)
        apply_weight_decay_and_step(param, u, lr_ratio, lr, weight_decay, cautious_wd)

    def foreach_update(
        self,
        params,
        grads,
        state,
        lr_ratios,
        *,
        lr,
        weight_decay,
        cautious_wd,
        momentum,
        nesterov,
        maximize,
        ns_steps,
        orthogonalization_strategy,
        split_sizes,
        **opts,
    ) -> None:
        bufs = state["momentum_buffer"]
        if fused_path_ok(params, grads, bufs, split_sizes):
            muon_fused.fused_muon_update(
                params,
                grads,
                bufs,
                lr_effs(lr, lr_ratios),
                weight_decay=weight_decay,
                cautious_wd=cautious_wd,
                momentum=momentum,
                nesterov=nesterov,
                maximize=maximize,
                ns_steps=ns_steps,
                strategy=orthogonalization_strategy,
            )
            return
        kw = dict(weight_decay=weight_decay, cautious_wd=cautious_wd, momentum=momentum, nesterov=nesterov,
                  maximize=maximize, strategy=orthogonalization_strategy)
        if distributed_fused(params, grads, bufs, lr_ratios, lr, split_sizes, ns_steps, kw):
            return
        g = list(torch._foreach_neg(grads)) if maximize else list(grads)
        torch._foreach_mul_(bufs, momentum)
        torch._foreach_add_(bufs, g)
        g_eff = torch._foreach_add(g, bufs, alpha=momentum) if nesterov else bufs
        u = orthogonalize_batch(
            list(g_eff), ns_steps=ns_steps, strategy=orthogonalization_strategy, split_sizes=split_sizes
        )
        u = [u_.view_as(p_) for u_, p_ in zip(u, params, strict=True)]
        u = [u_.to(p_.dtype) if u_.dtype != p_.dtype else u_ for u_, p_ in zip(u, params, strict=True)]
        foreach_weight_decay_and_step(params, u, lr_ratios, lr, weight_decay, cautious_wd)
