"""Grouping / device-move helpers for the batched driver
(reference: src/muonium/utils/foreach.py:8-40)."""

from __future__ import annotations

from typing import Sequence

import torch
from torch import Tensor


def group_tensors_by_shape(tensorlist: list[Tensor]) -> dict[tuple[int, ...], tuple[list[Tensor], list[int]]]:
    """Map each distinct shape to (tensors of that shape, their indices).

    Insertion order of first appearance is kept; dtype and device are ignored
    (callers group by those first).
    """
    groups: dict[tuple[int, ...], tuple[list[Tensor], list[int]]] = {}
    for idx, t in enumerate(tensorlist):
        entry = groups.setdefault(tuple(t.shape), ([], []))
        entry[0].append(t)
        entry[1].append(idx)
    return groups


def move_tensors_to_device(
    tensors: Sequence[Tensor | None], device_in: torch.device, device_out: torch.device
) -> list[Tensor | None]:
    """Copy tensors to ``device_out`` unless ``device_in`` already has the same device *type*.

    Same-type moves (e.g. cuda:0 -> cuda:1) are deliberately a no-op, like the
    reference; the input sequence object itself is returned in that case.
    """
    if device_in.type == device_out.type:
        return tensors  # type: ignore[return-value]
    return [t.to(device_out, non_blocking=True) if t is not None else None for t in tensors]
