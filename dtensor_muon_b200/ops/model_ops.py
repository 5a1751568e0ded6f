"""Entry points for the fused decoder-block kernels (``ops/csrc/model_ops.cu``).

``rope``, ``swiglu`` and ``cross_entropy`` run the native kernels, registered
as ``torch.library`` ops with their autograd formulas (``ops/library.py``), for
bf16 CUDA inputs and the equivalent PyTorch composition otherwise (CPU, fp32).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _ext, library


def _native(*ts: Tensor) -> bool:
    return all(t.is_cuda and t.dtype == torch.bfloat16 for t in ts) and _ext.available()


def rope_reference(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """Rotate interleaved pairs of the last dim of x [B, S, H, D] (fp32 math)."""
    xf = x.float().unflatten(-1, (-1, 2))
    x0, x1 = xf[..., 0], xf[..., 1]
    c = cos[None, : x.shape[1], None, :]
    s = sin[None, : x.shape[1], None, :]
    return torch.stack((x0 * c - x1 * s, x0 * s + x1 * c), dim=-1).flatten(-2).to(x.dtype)


def rope(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    if _native(x) and x.shape[-1] % 8 == 0:
        return library.rope(x, cos, sin, 1.0)
    return rope_reference(x, cos, sin)


def swiglu(a: Tensor, b: Tensor) -> Tensor:
    """silu(a) * b."""
    if _native(a, b) and a.numel() % 8 == 0:
        return library.swiglu(a, b)
    return F.silu(a) * b


def cross_entropy(logits: Tensor, targets: Tensor) -> Tensor:
    """Mean next-token cross entropy; fp32 math, bf16 logits read once per pass on CUDA."""
    flat = logits.reshape(-1, logits.shape[-1])
    t = targets.reshape(-1)
    if _native(flat) and flat.shape[-1] % 8 == 0 and t.dtype == torch.int64:
        return library.cross_entropy(flat, t)[0]
    return F.cross_entropy(flat.float(), t)
