"""Polar Express orthogonalisation (arXiv:2505.16932): PyTorch oracle loop.

Same iteration as the reference's ``pe_loop``
(src/muonium/orthogonalize/polar_express.py:28-66): per-step coefficient
triples, normalisation by ``1.02 * ||X||_F + eps``. CUDA inputs go to the
native engine in :mod:`dtensor_muon_b200.ops.ortho`.
"""

from __future__ import annotations

import torch
from torch import Tensor

from ..ops.ortho import POLAR_EXPRESS_COEFFS


def pe_loop(X: Tensor, steps: int = 5, *, eps: float = 1e-6) -> Tensor:
    """Polar Express iteration over the last two dims of ``X`` ([..., N, M])."""
    if X.ndim >= 3 and X.size(0) == 0:
        return X
    transpose = X.size(-2) > X.size(-1)
    if transpose:
        X = X.transpose(-2, -1)
    X = X / (X.norm(dim=(-2, -1), keepdim=True) * 1.02 + eps)
    for a, b, c in POLAR_EXPRESS_COEFFS[:steps]:
        A = torch.matmul(X, X.transpose(-1, -2))
        B = b * A + c * torch.matmul(A, A)
        X = a * X + B @ X
    if transpose:
        X = X.transpose(-2, -1)
    return X


__all__ = ["POLAR_EXPRESS_COEFFS", "pe_loop"]
