"""``torch.library`` registrations of the native kernels (namespace ``dmb``).

Registering the kernels as custom ops makes them visible to ``torch.compile``
and other tracers. A region that calls them traces as one graph: the fake
kernels give output shapes, and the autograd formulas are registered with the
ops. Each op has a CUDA kernel (the sm_100a extension) and a CPU kernel (the
PyTorch composition of the same math). The CPU kernel is the fallback and the
oracle.

Ops:

* ``dmb::rope(x, cos, sin, sign)``: rotates interleaved pairs of the last dim
  of ``x`` [B, S, H, D] by ``sign * angle``.
* ``dmb::swiglu(a, b)`` and ``dmb::swiglu_backward(a, b, g)``.
* ``dmb::cross_entropy(logits, targets) -> (mean loss, lse)`` and
  ``dmb::cross_entropy_backward``.
* ``dmb::gram(x)``: ``x @ x.mT`` over the last two dims, in bf16.
* ``dmb::zeropower(x, steps, strategy, eps)``: orthogonalises the last two
  dims (Newton-Schulz or Polar Express), in bf16.

The reference compiles its update math with ``torch.compile``
(``src/muonium/optim/optim.py:224-229``). Its Triton Gram kernel
(``src/muonium/kernels/gram.py:109-165``) is the op that ``dmb::gram`` stands
in for.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _ext

# ---------------------------------------------------------------- rope


@torch.library.custom_op("dmb::rope", mutates_args=(), device_types="cuda")
def rope(x: Tensor, cos: Tensor, sin: Tensor, sign: float) -> Tensor:
    return _ext.load().rope(x.contiguous(), cos.contiguous(), sin.contiguous(), sign)


@rope.register_kernel("cpu")
def _rope_cpu(x: Tensor, cos: Tensor, sin: Tensor, sign: float) -> Tensor:
    xf = x.float().unflatten(-1, (-1, 2))
    x0, x1 = xf[..., 0], xf[..., 1]
    c = cos[None, : x.shape[1], None, :].float()
    s = sign * sin[None, : x.shape[1], None, :].float()
    return torch.stack((x0 * c - x1 * s, x0 * s + x1 * c), dim=-1).flatten(-2).to(x.dtype)


@rope.register_fake
def _rope_fake(x, cos, sin, sign):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


def _rope_setup(ctx, inputs, output):
    _, cos, sin, sign = inputs
    ctx.save_for_backward(cos, sin)
    ctx.sign = sign


def _rope_backward(ctx, g):
    cos, sin = ctx.saved_tensors
    # the inverse of a rotation is the rotation by the negated angle
    return rope(g, cos, sin, -ctx.sign), None, None, None


rope.register_autograd(_rope_backward, setup_context=_rope_setup)

# ---------------------------------------------------------------- swiglu


@torch.library.custom_op("dmb::swiglu", mutates_args=(), device_types="cuda")
def swiglu(a: Tensor, b: Tensor) -> Tensor:
    return _ext.load().swiglu_fwd(a.contiguous(), b.contiguous())


@swiglu.register_kernel("cpu")
def _swiglu_cpu(a: Tensor, b: Tensor) -> Tensor:
    return (F.silu(a.float()) * b.float()).to(a.dtype)


@swiglu.register_fake
def _swiglu_fake(a, b):
    return torch.empty_like(a, memory_format=torch.contiguous_format)


@torch.library.custom_op("dmb::swiglu_backward", mutates_args=(), device_types="cuda")
def swiglu_backward(a: Tensor, b: Tensor, g: Tensor) -> tuple[Tensor, Tensor]:
    da, db = _ext.load().swiglu_bwd(a.contiguous(), b.contiguous(), g.contiguous())
    return da, db


@swiglu_backward.register_kernel("cpu")
def _swiglu_backward_cpu(a: Tensor, b: Tensor, g: Tensor) -> tuple[Tensor, Tensor]:
    af, bf, gf = a.float(), b.float(), g.float()
    sig = torch.sigmoid(af)
    da = gf * bf * sig * (1 + af * (1 - sig))
    db = gf * af * sig
    return da.to(a.dtype), db.to(b.dtype)


@swiglu_backward.register_fake
def _swiglu_backward_fake(a, b, g):
    return (torch.empty_like(a, memory_format=torch.contiguous_format),
            torch.empty_like(b, memory_format=torch.contiguous_format))


def _swiglu_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _swiglu_grad(ctx, g):
    a, b = ctx.saved_tensors
    return swiglu_backward(a, b, g)


swiglu.register_autograd(_swiglu_grad, setup_context=_swiglu_setup)

# ---------------------------------------------------------------- cross entropy


@torch.library.custom_op("dmb::cross_entropy", mutates_args=(), device_types="cuda")
def cross_entropy(logits: Tensor, targets: Tensor) -> tuple[Tensor, Tensor]:
    """Mean cross entropy of ``logits`` [T, V] against ``targets`` [T]; also returns the row log-sum-exp."""
    rows, lse = _ext.load().cross_entropy_fwd(logits.contiguous(), targets.contiguous())
    return rows.mean(), lse


@cross_entropy.register_kernel("cpu")
def _cross_entropy_cpu(logits: Tensor, targets: Tensor) -> tuple[Tensor, Tensor]:
    lf = logits.float()
    lse = torch.logsumexp(lf, dim=-1)
    rows = lse - lf.gather(-1, targets[:, None]).squeeze(-1)
    return rows.mean(), lse


@cross_entropy.register_fake
def _cross_entropy_fake(logits, targets):
    return logits.new_empty((), dtype=torch.float32), logits.new_empty(logits.shape[:1], dtype=torch.float32)


@torch.library.custom_op("dmb::cross_entropy_backward", mutates_args=(), device_types="cuda")
def cross_entropy_backward(logits: Tensor, targets: Tensor, lse: Tensor, g: Tensor) -> Tensor:
    """d(mean loss)/d(logits) times the upstream scalar ``g`` (read on the device: no host sync)."""
    gs = g.reshape(1).to(torch.float32).contiguous()
    return _ext.load().cross_entropy_bwd(logits.contiguous(), targets.contiguous(), lse, 1.0 / logits.shape[0], gs)


@cross_entropy_backward.register_kernel("cpu")
def _cross_entropy_backward_cpu(logits: Tensor, targets: Tensor, lse: Tensor, g: Tensor) -> Tensor:
    p = torch.exp(logits.float() - lse[:, None])
    p[torch.arange(logits.shape[0]), targets] -= 1.0
    return (p * (g.float() / logits.shape[0])).to(logits.dtype)


@cross_entropy_backward.register_fake
def _cross_entropy_backward_fake(logits, targets, lse, g):
    return torch.empty_like(logits, memory_format=torch.contiguous_format)


def _ce_setup(ctx, inputs, output):
    logits, targets = inputs
    ctx.save_for_backward(logits, targets, output[1])


def _ce_grad(ctx, g_loss, g_lse):
    logits, targets, lse = ctx.saved_tensors
    return cross_entropy_backward(logits, targets, lse, g_loss), None


cross_entropy.register_autograd(_ce_grad, setup_context=_ce_setup)

# ---------------------------------------------------------------- orthogonalisation


@torch.library.custom_op("dmb::gram", mutates_args=(), device_types="cuda")
def gram(x: Tensor) -> Tensor:
    from .ortho import gram as native_gram

    return native_gram(x.bfloat16())


@gram.register_kernel("cpu")
def _gram_cpu(x: Tensor) -> Tensor:
    xf = x.float()
    return (xf @ xf.mT).bfloat16()


@gram.register_fake
def _gram_fake(x):
    return x.new_empty((*x.shape[:-1], x.shape[-2]), dtype=torch.bfloat16)


@torch.library.custom_op("dmb::zeropower", mutates_args=(), device_types="cuda")
def zeropower(x: Tensor, steps: int, strategy: str, eps: float) -> Tensor:
    from ..orthogonalize.orthogonalize import orthogonalize_local

    return orthogonalize_local(x, steps, eps, strategy, use_native=True).clone()


@zeropower.register_kernel("cpu")
def _zeropower_cpu(x: Tensor, steps: int, strategy: str, eps: float) -> Tensor:
    from ..orthogonalize.orthogonalize import orthogonalize_local

    return orthogonalize_local(x, steps, eps, strategy, use_native=False).clone()


@zeropower.register_fake
def _zeropower_fake(x, steps, strategy, eps):
    return x.new_empty(x.shape, dtype=torch.bfloat16)


__all__ = ["cross_entropy", "cross_entropy_backward", "gram", "rope", "swiglu", "swiglu_backward", "zeropower"]
