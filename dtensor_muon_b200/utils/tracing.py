"""NVTX ranges around the fused phases (visible in Nsight Systems / ncu).

Enabled by default; set ``DMB_NVTX=0`` to turn the markers off. The ranges cost
a few microseconds of host time each and nothing on the device.
"""

from __future__ import annotations

import contextlib
import os

import torch

_ON = os.environ.get("DMB_NVTX", "1") != "0"


@contextlib.contextmanager
def nvtx(name: str):
    if _ON and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield
