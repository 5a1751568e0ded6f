"""Loader for the in-tree sm_100a extension ``dtensor_muon_b200._C``.

The CUDA paths of this package always go through the compiled extension. If a
CUDA tensor reaches an op while the extension cannot be imported, the op raises
instead of silently running a PyTorch fallback.
"""

from __future__ import annotations

import importlib

_C = None
_IMPORT_ERROR: Exception | None = None


def load():
    """Return the compiled extension module, importing it on first use."""
    global _C, _IMPORT_ERROR
    if _C is not None:
        return _C
    if _IMPORT_ERROR is not None:
        raise RuntimeError(
            "dtensor_muon_b200 native extension is not built "
            "(run `python setup.py build_ext --inplace`)"
        ) from _IMPORT_ERROR
    try:
        _C = importlib.import_module("dtensor_muon_b200._C")
    except Exception as exc:  # pragma: no cover - depends on the build
        _IMPORT_ERROR = exc
        raise RuntimeError(
            "dtensor_muon_b200 native extension is not built "
            "(run `python setup.py build_ext --inplace`)"
        ) from exc
    return _C


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def check_device_errors(device) -> None:
    """Raise if a kernel on ``device`` recorded a timed-out wait since the last check."""
    import torch

    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    code = load().take_device_error(idx)
    if code:
        raise RuntimeError(f"dtensor_muon_b200 kernel reported error code {code} on cuda:{idx}")
