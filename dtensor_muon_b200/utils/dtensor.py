"""DTensor helpers (reference: src/muonium/utils/dtensor.py:5-9)."""

from __future__ import annotations

from torch import Tensor
from torch.distributed.tensor import DTensor


def to_local(tensor: Tensor, full_tensor: bool = False) -> Tensor:
    """Local shard of a DTensor (or the full gathered tensor); plain tensors pass through."""
    if not isinstance(tensor, DTensor):
        return tensor
    return tensor.full_tensor() if full_tensor else tensor.to_local()
