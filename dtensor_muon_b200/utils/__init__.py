"""DTensor and batching helpers (reference: ``src/muonium/utils/dtensor.py:5-9``,
``src/muonium/utils/foreach.py:8-40``)."""

from .dtensor import to_local
from .foreach import group_tensors_by_shape, move_tensors_to_device

__all__ = ["to_local", "group_tensors_by_shape", "move_tensors_to_device"]
