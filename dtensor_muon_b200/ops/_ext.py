"""Loader for the in-tree sm_100a extension ``dtensor_muon_b200._C``.

The CUDA paths of this package always go through the compiled extension. If a
CUDA tensor reaches an op while the extension cannot be imported, the op raises
instead of silently running a PyTorch fallback.
"""

from __future__ import annotations

import importlib

_C = None
_IMPORT_ERROR: Exception | None = None

# Kernel launches issued by each binding (ortho_iterate: three per step).
_LAUNCHES = {
    "gram_sym": 1,
    "gemm_ax": 1,
    "gram_sym2": 1,
    "gemm_ax2": 1,
    "muon_pack": 1,
    "muon_pack_ex": 1,
    "muon_apply_ex": 1,
    "norm_finalize": 1,
    "muon_apply": 1,
    "muon_unpack": 1,
    "row_sumsq": 1,
    "normuon_finalize": 1,
    "adamw_multi": 1,
    "lp_momentum_step": 1,
    "lp_dequantize": 1,
    "lp_quantize": 1,
    "dist_pack": 2,
    "dist_apply": 1,
    "dist_barrier": 1,
    "push_slots": 1,
    "local_slot_sum": 1,
    "rs_sum_momentum": 1,
    "ag_gemm": 1,
    "ep_scatter_rows": 1,
    "ep_gather_rows": 1,
    "rope": 1,
    "swiglu_fwd": 1,
    "swiglu_bwd": 1,
    "cross_entropy_fwd": 1,
    "cross_entropy_bwd": 1,
}
launch_count = 0


class _Counted:
    """Thin proxy over the extension that counts the kernels each call launches."""

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def call(*args, **kwargs):
            global launch_count
            if name == "ortho_iterate":
                launch_count += 3 * int(args[5].shape[0])
            else:
                launch_count += _LAUNCHES.get(name, 0)
            return fn(*args, **kwargs)

        return call


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
        _C = _Counted(importlib.import_module("dtensor_muon_b200._C"))
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
