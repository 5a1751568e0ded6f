"""Mixtral-style sparse MoE decoder (top-2 routing, stacked 3-D experts).

Expert weights are stacked ``[E, F, D]`` / ``[E, D, F]`` parameters: with
expert parallelism they are DTensors sharded on dim 0 across the EP group, so
the optimizer sees 3-D tensors sharded only on dim 0 and orthogonalises every
local expert matrix with no communication (the reference's collective-free
path, src/muonium/orthogonalize/orthogonalize.py:165-204). Tokens reach their
experts through :mod:`dtensor_muon_b200.parallel.expert_parallel`
(dispatch / combine over NVLink peer memory, or NCCL all-to-all).
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch
from torch import Tensor, nn

from ..ops import model_ops as _model_ops
from .llama import Block, Llama, LlamaConfig


@dataclass(frozen=True)
class MixtralConfig(LlamaConfig):
    n_experts: int = 8
    top_k: int = 2


MIXTRAL_PRESETS = {
    "mixtral-8x7b": MixtralConfig(vocab_size=32000, dim=4096, n_layers=32, n_heads=32, n_kv_heads=8,
                                  ffn_dim=14336, rope_theta=1e6, n_experts=8, top_k=2),
    "mixtral-tiny": MixtralConfig(vocab_size=1024, dim=256, n_layers=2, n_heads=4, n_kv_heads=4, ffn_dim=512,
                                  rope_theta=10000.0, max_seq_len=512, n_experts=4, top_k=2),
}


def mixtral_preset(name: str, **overrides) -> MixtralConfig:
    return replace(MIXTRAL_PRESETS[name], **overrides)


def _grouped(x: Tensor, w: Tensor, counts: Tensor) -> Tensor:
    """rows of ``x`` grouped by expert (``counts`` per expert) times ``w[e].T``."""
    if x.is_cuda and x.dtype == torch.bfloat16 and x.shape[0] > 0:
        offs = torch.cumsum(counts, 0).to(torch.int32)
        try:
            return torch._grouped_mm(x, w.transpose(-2, -1), offs=offs)
        except (RuntimeError, NotImplementedError):
            pass
    outs = []
    for e, xe in enumerate(torch.split(x, counts.tolist())):
        outs.append(xe @ w[e].t())
    return torch.cat(outs) if outs else x.new_zeros(0, w.shape[1])


def expert_ffn(x: Tensor, counts: Tensor, w1: Tensor, w3: Tensor, w2: Tensor) -> Tensor:
    """SwiGLU experts over expert-grouped rows."""
    h = _model_ops.swiglu(_grouped(x, w1, counts), _grouped(x, w3, counts))
    return _grouped(h, w2, counts)


class MoEFeedForward(nn.Module):
    def __init__(self, cfg: MixtralConfig, ep=None):
        super().__init__()
        self.n_experts = cfg.n_experts
        self.top_k = cfg.top_k
        self.router = nn.Linear(cfg.dim, cfg.n_experts, bias=False)
        self.w1 = nn.Parameter(torch.empty(cfg.n_experts, cfg.ffn_dim, cfg.dim))  # gate
        self.w3 = nn.Parameter(torch.empty(cfg.n_experts, cfg.ffn_dim, cfg.dim))  # up
        self.w2 = nn.Parameter(torch.empty(cfg.n_experts, cfg.dim, cfg.ffn_dim))  # down
        self.ep = ep  # ExpertParallel or None (all experts local)

    def route(self, x: Tensor) -> tuple[Tensor, Tensor]:
        logits = self.router(x)
        top, idx = torch.topk(logits, self.top_k, dim=-1)
        return idx, torch.softmax(top.float(), dim=-1).to(x.dtype)

    def forward(self, x: Tensor) -> Tensor:
        B, S, D = x.shape
        flat = x.reshape(-1, D)
        idx, gates = self.route(flat)
        w1, w3, w2 = (w.to_local() if hasattr(w, "to_local") else w for w in (self.w1, self.w3, self.w2))
        if self.ep is None:
            expert = idx.reshape(-1)
            order = torch.argsort(expert, stable=True)
            counts = torch.bincount(expert, minlength=self.n_experts)
            rows = flat.repeat_interleave(self.top_k, dim=0)[order]
            y = expert_ffn(rows, counts, w1, w3, w2)
            out = torch.empty_like(y)
            out[order] = y
        else:
            out = self.ep.run(flat, idx, lambda rows, counts: expert_ffn(rows, counts, w1, w3, w2))
        out = out.view(-1, self.top_k, D) * gates.unsqueeze(-1)
        return out.sum(dim=1).view(B, S, D)


class Mixtral(Llama):
    """Llama attention blocks with MoE feed-forward layers."""

    def __init__(self, cfg: MixtralConfig, ep=None):
        super().__init__(cfg, block_factory=lambda: Block(cfg, ffn=MoEFeedForward(cfg, ep)))


__all__ = ["MIXTRAL_PRESETS", "MixtralConfig", "Mixtral", "MoEFeedForward", "expert_ffn", "mixtral_preset"]
