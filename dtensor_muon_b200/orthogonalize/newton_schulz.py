"""Newton-Schulz orthogonalisation: PyTorch oracle loop.

Same iteration as the reference's ``ns_loop``
(src/muonium/orthogonalize/newton_schulz.py:15-57): transpose so rows <= cols,
normalise by ``||X||_F + eps``, then ``A = X X^T; B = b A + c A^2; X = a X + B X``.
This loop is the CPU path and the numerical oracle; CUDA inputs go to the
native engine in :mod:`dtensor_muon_b200.ops.ortho`.
"""

from __future__ import annotations

import torch
from torch import Tensor

from ..ops.ortho import NS_COEFFS


def ns_loop(
    X: Tensor,
    steps: int = 5,
    *,
    a: float = NS_COEFFS[0],
    b: float = NS_COEFFS[1],
    c: float = NS_COEFFS[2],
    eps: float = 1e-7,
) -> Tensor:
    """Newton-Schulz iteration over the last two dims of ``X`` ([..., N, M])."""
    if X.ndim >= 3 and X.size(0) == 0:
        return X
    transpose = X.size(-2) > X.size(-1)
    if transpose:
        X = X.transpose(-2, -1)
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + eps)
    for _ in range(steps):
        A = torch.matmul(X, X.transpose(-1, -2))
        B = b * A + c * torch.matmul(A, A)
        X = a * X + torch.matmul(B, X)
    if transpose:
        X = X.transpose(-2, -1)
    return X
