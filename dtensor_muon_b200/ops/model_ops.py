"""Autograd wrappers for the fused decoder-block kernels (``ops/csrc/model_ops.cu``).

``rope`` and ``swiglu`` run the native kernels for contiguous bf16 CUDA inputs
and the equivalent PyTorch composition otherwise (CPU, fp32).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _ext


def _native(*ts: Tensor) -> bool:
    return all(t.is_cuda and t.dtype == torch.bfloat16 for t in ts) and _ext.available()


def rope_reference(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """Rotate interleaved pairs of the last dim of x [B, S, H, D] (fp32 math)."""
    xf = x.float().unflatten(-1, (-1, 2))
    x0, x1 = xf[..., 0], xf[..., 1]
    c = cos[None, : x.shape[1], None, :]
    s = sin[None, : x.shape[1], None, :]
    return torch.stack((x0 * c - x1 * s, x0 * s + x1 * c), dim=-1).flatten(-2).to(x.dtype)


class _Rope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cos, sin):
        ctx.save_for_backward(cos, sin)
        return _ext.load().rope(x.contiguous(), cos, sin, 1.0)

    @staticmethod
    def backward(ctx, g):
        cos, sin = ctx.saved_tensors
        return _ext.load().rope(g.contiguous(), cos, sin, -1.0), None, None


def rope(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    if _native(x) and x.shape[-1] % 8 == 0:
        return _Rope.apply(x, cos.contiguous(), sin.contiguous())
    return rope_reference(x, cos, sin)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        a, b = a.contiguous(), b.contiguous()
        ctx.save_for_backward(a, b)
        return _ext.load().swiglu_fwd(a, b)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        da, db = _ext.load().swiglu_bwd(a, b, g.contiguous())
        return da, db


def swiglu(a: Tensor, b: Tensor) -> Tensor:
    """silu(a) * b."""
    if _native(a, b) and a.numel() % 8 == 0:
        return _SwiGLU.apply(a, b)
    return F.silu(a) * b


class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets):
        loss_rows, lse = _ext.load().cross_entropy_fwd(logits, targets)
        ctx.save_for_backward(logits, targets, lse)
        return loss_rows.mean()

    @staticmethod
    def backward(ctx, g):
        logits, targets, lse = ctx.saved_tensors
        # the upstream scalar is read by the kernel on the device: no host sync
        gs = g.reshape(1).to(torch.float32).contiguous()
        return _ext.load().cross_entropy_bwd(logits, targets, lse, 1.0 / logits.shape[0], gs), None


def cross_entropy(logits: Tensor, targets: Tensor) -> Tensor:
    """Mean next-token cross entropy; fp32 math, bf16 logits read once per pass on CUDA."""
    flat = logits.reshape(-1, logits.shape[-1])
    t = targets.reshape(-1)
    if _native(flat) and flat.shape[-1] % 8 == 0 and t.dtype == torch.int64:
        return _CrossEntropy.apply(flat.contiguous(), t.contiguous())
    return F.cross_entropy(flat.float(), t)
