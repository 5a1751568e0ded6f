"""Native fused multi-tensor Adam / AdamW (one sm_100a launch per param group).

Matches ``torch.optim.adam``'s math, which the reference uses for its
"adam"/"adamw" groups (src/muonium/optim/optim.py:642-694). Step counters stay
on the CPU (torch's default placement); per-tensor bias corrections are
computed on the host in double precision and handed to the kernel.
"""

from __future__ import annotations

import math
import struct

import torch
from torch import Tensor

from . import _ext

_CODE = {torch.float32: 0, torch.bfloat16: 1}


def native_eligible(params: list[Tensor], grads, exp_avgs, exp_avg_sqs, max_exp_avg_sqs, amsgrad: bool) -> bool:
    if not params or not _ext.available():
        return False
    lists = [params, grads, exp_avgs, exp_avg_sqs] + ([max_exp_avg_sqs] if amsgrad else [])
    for ts in lists:
        for t in ts:
            if not t.is_cuda or t.dtype not in _CODE or not t.is_contiguous() or hasattr(t, "device_mesh"):
                return False
    dev = params[0].device
    return all(p.device == dev for p in params)


def _f32_bits(x: float) -> int:
    return struct.unpack("<i", struct.pack("<f", x))[0]


def fused_adam(
    params: list[Tensor],
    grads: list[Tensor],
    exp_avgs: list[Tensor],
    exp_avg_sqs: list[Tensor],
    max_exp_avg_sqs: list[Tensor],
    state_steps: list[Tensor],
    *,
    amsgrad: bool,
    beta1: float,
    beta2: float,
    lr: float,
    weight_decay: float,
    eps: float,
    maximize: bool,
    decoupled_weight_decay: bool,
) -> None:
    C = _ext.load()
    rows = []
    for i, (p, g, m, v) in enumerate(zip(params, grads, exp_avgs, exp_avg_sqs, strict=True)):
        step_t = state_steps[i]
        step_t += 1
        step = float(step_t)
        bc1 = 1.0 - beta1**step
        bc2 = 1.0 - beta2**step
        vmax = max_exp_avg_sqs[i] if amsgrad else v
        dts = _CODE[p.dtype] | (_CODE[g.dtype] << 4) | (_CODE[m.dtype] << 8) | (_CODE[v.dtype] << 12) | (
            _CODE[vmax.dtype] << 16
        )
        if p.numel() % 8 == 0 and all(t.data_ptr() % 16 == 0 for t in (p, g, m, v, vmax)):
            dts |= 1 << 20  # 16-byte vector path
        rows.append(
            [
                p.data_ptr(),
                g.data_ptr(),
                m.data_ptr(),
                v.data_ptr(),
                vmax.data_ptr(),
                p.numel(),
                dts,
                0,
                _f32_bits(lr / bc1),
                _f32_bits(1.0 / math.sqrt(bc2)),
            ]
        )
    meta = torch.tensor(rows, dtype=torch.int64)
    C.adamw_multi(
        meta, float(lr), beta1, beta2, eps, float(weight_decay), decoupled_weight_decay, amsgrad, maximize,
        params[0].device,
    )
