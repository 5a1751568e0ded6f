"""NorMuon: Muon with neuron-wise update normalisation (arXiv:2510.05491).

Math of the reference's ``NorMuon`` (src/muonium/optim/algorithms/normuon.py:16-203):
after orthogonalisation, keep ``||u||_F``, update the per-row second moment
``v = lerp(v, mean(u^2, -1), 1 - beta2)``, divide rows by ``sqrt(v) + 1e-8``
and rescale to the original Frobenius norm. With ``split_sizes`` each row
block is normalised on its own.

CUDA batches run fused (row sums of squares and the per-row scale are two
small kernels between the last GEMM and the parameter write).
"""

from __future__ import annotations

import torch
from torch import Tensor

from ...ops import muon_fused
from .base import (
    BufferSpec,
    MuonAlgorithm,
    orthogonalize_batch,
    orthogonalize_single,
    register_muon_algorithm,
)
from .muon import (
    apply_weight_decay_and_step,
    distributed_fused,
    foreach_weight_decay_and_step,
    fused_path_ok,
    lr_effs,
)


def _normuon_normalize(
    u: Tensor, v: Tensor, muon_beta2: float, split_sizes: tuple[int, ...] | None = None
) -> tuple[Tensor, Tensor]:
    """Return ``(normalised u, new v)`` out of place."""
    if split_sizes is not None:
        parts = [
            _normuon_normalize(ub, vb, muon_beta2)
            for ub, vb in zip(u.split(list(split_sizes), dim=-2), v.split(list(split_sizes), dim=-2), strict=True)
        ]
        return torch.cat([a for a, _ in parts], dim=-2), torch.cat([b for _, b in parts], dim=-2)
    u = u.to(v.dtype)
    fro = u.norm(p=2, dim=(-2, -1), keepdim=True)
    row_ms = (u * u).mean(dim=-1, keepdim=True)
    v_new = torch.lerp(v, row_ms, 1 - muon_beta2)
    u = u / (v_new.sqrt() + 1e-8)
    fro_new = u.norm(p=2, dim=(-2, -1), keepdim=True).clamp(min=1e-8)
    return u * (fro / fro_new), v_new


def _fused_ok(params, grads, bufs, variances, split_sizes) -> bool:
    if not fused_path_ok(params, grads, bufs, split_sizes):
        return False
    return all(
        v.is_cuda and v.dtype == torch.float32 and v.is_contiguous() and not hasattr(v, "device_mesh")
        for v in variances
    )


@register_muon_algorithm
class NorMuon(MuonAlgorithm):
    """Muon plus a neuron-wise (row-wise) second-moment normalisation of the update."""

    name = "normuon"
    options = {"muon_beta2": 0.95}
    state_spec = {
        "momentum_buffer": BufferSpec(like="grad", signed=True),
        "variance_neuron": BufferSpec(like="grad_rows", signed=False),
    }

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
        muon_beta2: float = 0.95,
        **opts,
    ) -> None:
        buf, var = state["momentum_buffer"], state["variance_neuron"]
        if _fused_ok([param], [grad], [buf], [var], split_sizes):
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
                variances=[var],
                muon_beta2=muon_beta2,
            )
            return
        kw = dict(weight_decay=weight_decay, cautious_wd=cautious_wd, momentum=momentum, nesterov=nesterov,
                  maximize=maximize, strategy=orthogonalization_strategy, muon_beta2=muon_beta2)
        if distributed_fused([param], [grad], [buf], [lr_ratio], lr, split_sizes, ns_steps, kw, variances=[var]):
            return
        g32 = (-grad if maximize else grad).to(torch.float32)
        new_buf = buf.to(torch.float32) * momentum + g32
        buf.copy_(new_buf)
        g_eff = g32 + momentum * new_buf if nesterov else new_buf
        u = orthogonalize_single(
            g_eff, ns_steps=ns_steps, strategy=orthogonalization_strategy, split_sizes=split_sizes
        )
        u, v_new = _normuon_normalize(u, var.to(torch.float32), muon_beta2, split_sizes)
        var.copy_(v_new)
        apply_weight_decay_and_step(param, u.view_as(param), lr_ratio, lr, weight_decay, cautious_wd)

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
        muon_beta2: float = 0.95,
        **opts,
    ) -> None:
        bufs, variances = state["momentum_buffer"], state["variance_neuron"]
        if _fused_ok(params, grads, bufs, variances, split_sizes):
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
                variances=variances,
                muon_beta2=muon_beta2,
            )
            return
        kw = dict(weight_decay=weight_decay, cautious_wd=cautious_wd, momentum=momentum, nesterov=nesterov,
                  maximize=maximize, strategy=orthogonalization_strategy, muon_beta2=muon_beta2)
        if distributed_fused(params, grads, bufs, lr_ratios, lr, split_sizes, ns_steps, kw, variances=variances):
            return
        g = list(torch._foreach_neg(grads)) if maximize else list(grads)
        torch._foreach_mul_(bufs, momentum)
        torch._foreach_add_(bufs, g)
        g_eff = torch._foreach_add(g, bufs, alpha=momentum) if nesterov else bufs
        u = orthogonalize_batch(
            list(g_eff), ns_steps=ns_steps, strategy=orthogonalization_strategy, split_sizes=split_sizes
        )
        normed = []
        for u_, v in zip(u, variances, strict=True):
            u_n, v_new = _normuon_normalize(u_, v.to(torch.float32), muon_beta2, split_sizes)
            v.copy_(v_new)
            normed.append(u_n)
        u = [u_.view_as(p_).to(p_.dtype) for u_, p_ in zip(normed, params, strict=True)]
        foreach_weight_decay_and_step(params, u, lr_ratios, lr, weight_decay, cautious_wd)
