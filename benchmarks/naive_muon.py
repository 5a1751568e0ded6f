"""Blog-post style Muon: eager bf16 Newton-Schulz, plain decoupled weight decay,
one parameter at a time. The floor every optimised path is compared against
(the reference keeps the same baseline in benchmark/naive_muon.py)."""

from __future__ import annotations

import math

import torch


def newton_schulz_bf16(g: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    a, b, c = 3.4445, -4.7750, 2.0315
    x = g.bfloat16()
    tall = x.size(-2) > x.size(-1)
    if tall:
        x = x.mT
    x = x / (x.norm() + eps)
    for _ in range(steps):
        A = x @ x.mT
        B = b * A + c * (A @ A)
        x = a * x + B @ x
    return x.mT if tall else x


class NaiveMuon(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-3, wd=0.1, momentum=0.95, nesterov=True, ns_steps=5):
        super().__init__(params, dict(lr=lr, wd=wd, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps))

    @torch.no_grad()
    def step(self):
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if not st:
                    st["momentum_buffer"] = torch.zeros_like(p, dtype=torch.float32)
                buf = st["momentum_buffer"]
                buf.mul_(group["momentum"]).add_(p.grad)
                g = p.grad + group["momentum"] * buf if group["nesterov"] else buf
                u = newton_schulz_bf16(g, group["ns_steps"]).to(p.dtype)
                scale = math.sqrt(max(1.0, p.size(-2) / p.size(-1)))
                p.mul_(1 - group["lr"] * group["wd"])
                p.add_(u, alpha=-group["lr"] * scale)
