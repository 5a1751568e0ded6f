"""Llama-style decoder (RMSNorm, RoPE, GQA attention, SwiGLU), random init.

The reference ships no model; this is the training workload its optimizer is
benchmarked on (Llama-3-8B / Llama-2-13B shapes, plus the tiny 2-layer model
of the CPU parity config). Attention goes through
``F.scaled_dot_product_attention`` (flash / cuDNN kernels on B200); weights
are plain ``nn.Linear`` / ``nn.Embedding`` so FSDP2 ``fully_shard`` and
DTensor tensor-parallel plans apply without adapters.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..ops import model_ops as _model_ops


@dataclass(frozen=True)
class LlamaConfig:
    vocab_size: int = 128256
    dim: int = 4096
    n_layers: int = 32
    n_heads: int = 32
    n_kv_heads: int = 8
    ffn_dim: int = 14336
    norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    max_seq_len: int = 4096
    init_std: float = 0.02

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads


PRESETS = {
    "llama3-8b": LlamaConfig(),
    "llama2-13b": LlamaConfig(
        vocab_size=32000, dim=5120, n_layers=40, n_heads=40, n_kv_heads=40, ffn_dim=13824, rope_theta=10000.0
    ),
    # 2-layer CPU parity model (d 256, 4 heads, SwiGLU 1024, vocab 1024).
    "tiny": LlamaConfig(vocab_size=1024, dim=256, n_layers=2, n_heads=4, n_kv_heads=4, ffn_dim=1024,
                        rope_theta=10000.0, max_seq_len=512),
}


def preset(name: str, **overrides) -> LlamaConfig:
    return replace(PRESETS[name], **overrides)


def rope_tables(head_dim: int, seq_len: int, theta: float, device=None) -> tuple[Tensor, Tensor]:
    """cos / sin tables [seq, head_dim // 2] for rotary embeddings (fp32)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))
    t = torch.arange(seq_len, dtype=torch.float32, device=device)
    freqs = torch.outer(t, inv)
    return freqs.cos(), freqs.sin()


def apply_rope(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """Rotate interleaved pairs of the last dim. x: [B, S, H, D] (fused kernel on CUDA bf16)."""
    return _model_ops.rope(x, cos, sin)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: Tensor) -> Tensor:
        return F.rms_norm(x, (x.size(-1),), self.weight, self.eps)


class Attention(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.n_heads = cfg.n_heads
        self.n_kv_heads = cfg.n_kv_heads
        self.head_dim = cfg.head_dim
        self.wq = nn.Linear(cfg.dim, cfg.n_heads * cfg.head_dim, bias=False)
        self.wk = nn.Linear(cfg.dim, cfg.n_kv_heads * cfg.head_dim, bias=False)
        self.wv = nn.Linear(cfg.dim, cfg.n_kv_heads * cfg.head_dim, bias=False)
        self.wo = nn.Linear(cfg.n_heads * cfg.head_dim, cfg.dim, bias=False)
        # set by train.build_llama(fused_gather=True): q/k/v through the fused
        # parameter all-gather + GEMM kernel (parallel.ag_gemm.GatherLinear)
        self.gather = None
        self.gather_out = None  # wo through the fused gather (one-weight GatherLinear)

    def forward(self, x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
        B, S, _ = x.shape
        if self.gather is not None:
            q, k, v = (t.view(B, S, -1, self.head_dim) for t in self.gather(x))
        else:
            q = self.wq(x).view(B, S, -1, self.head_dim)
            k = self.wk(x).view(B, S, -1, self.head_dim)
            v = self.wv(x).view(B, S, -1, self.head_dim)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=self.n_kv_heads != self.n_heads)
        o = o.transpose(1, 2).reshape(B, S, -1)
        if self.gather_out is not None:
            return self.gather_out(o)[0]
        return self.wo(o)


class FeedForward(nn.Module):
    def __init__(self, dim: int, hidden: int):
        super().__init__()
        self.w1 = nn.Linear(dim, hidden, bias=False)  # gate
        self.w3 = nn.Linear(dim, hidden, bias=False)  # up
        self.w2 = nn.Linear(hidden, dim, bias=False)  # down
        self.gather = None  # gate/up through the fused all-gather + GEMM (see Attention)
        self.gather_out = None  # w2 likewise

    def forward(self, x: Tensor) -> Tensor:
        if self.gather is not None:
            gate, up = self.gather(x)
            h = _model_ops.swiglu(gate, up)
            return self.gather_out(h)[0] if self.gather_out is not None else self.w2(h)
        return self.w2(_model_ops.swiglu(self.w1(x), self.w3(x)))


class Block(nn.Module):
    def __init__(self, cfg: LlamaConfig, ffn: nn.Module | None = None):
        super().__init__()
        self.attention_norm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.attention = Attention(cfg)
        self.ffn_norm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.feed_forward = ffn if ffn is not None else FeedForward(cfg.dim, cfg.ffn_dim)

    def forward(self, x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
        x = x + self.attention(self.attention_norm(x), cos, sin)
        return x + self.feed_forward(self.ffn_norm(x))


class Llama(nn.Module):
    def __init__(self, cfg: LlamaConfig, block_factory=None):
        super().__init__()
        self.cfg = cfg
        self.tok_embeddings = nn.Embedding(cfg.vocab_size, cfg.dim)
        make = block_factory or (lambda: Block(cfg))
        self.layers = nn.ModuleList([make() for _ in range(cfg.n_layers)])
        self.norm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.output = nn.Linear(cfg.dim, cfg.vocab_size, bias=False)
        self._rope_cache: dict = {}

    def rope(self, seq_len: int, device) -> tuple[Tensor, Tensor]:
        key = (seq_len, str(device))
        if key not in self._rope_cache:
            self._rope_cache[key] = rope_tables(self.cfg.head_dim, seq_len, self.cfg.rope_theta, device)
        return self._rope_cache[key]

    @torch.no_grad()
    def init_weights(self, seed: int | None = None, generator: torch.Generator | None = None) -> None:
        """N(0, init_std) for every Linear / Embedding weight (router included), ones for norms."""
        gen = generator
        if gen is None and seed is not None:
            gen = torch.Generator(device="cpu").manual_seed(seed)
        for name, p in self.named_parameters():
            local = p.to_local() if hasattr(p, "to_local") else p
            if name.endswith("norm.weight") or "_norm." in name:
                local.fill_(1.0)
            elif gen is not None and local.device.type == "cpu":
                local.copy_(torch.randn(local.shape, generator=gen, dtype=torch.float32) * self.cfg.init_std)
            else:
                local.normal_(0.0, self.cfg.init_std)

    def forward(self, tokens: Tensor) -> Tensor:
        h = self.tok_embeddings(tokens)
        cos, sin = self.rope(tokens.size(1), tokens.device)
        for layer in self.layers:
            h = layer(h, cos, sin)
        return self.output(self.norm(h))


def lm_loss(logits: Tensor, targets: Tensor) -> Tensor:
    """Next-token cross entropy in fp32 (fused kernel for bf16 CUDA logits)."""
    return _model_ops.cross_entropy(logits, targets)


def muon_and_adam_params(model: nn.Module) -> tuple[list[nn.Parameter], list[nn.Parameter]]:
    """Muon for the 2-D (and stacked 3-D expert) weights inside the decoder
    blocks; AdamW for embeddings, norms, the LM head and MoE routers."""
    muon, adam = [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        hidden = name.startswith("layers.")
        if hidden and p.ndim >= 2 and "router" not in name:
            muon.append(p)
        else:
            adam.append(p)
    return muon, adam


def param_count(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())


def flops_per_token(cfg: LlamaConfig, seq_len: int) -> float:
    """Training FLOPs per token: 6 * matmul params + attention (causal, fwd+bwd)."""
    n = cfg.n_layers * (2 * cfg.dim * cfg.dim + 2 * cfg.dim * cfg.n_kv_heads * cfg.head_dim + 3 * cfg.dim * cfg.ffn_dim)
    n += cfg.dim * cfg.vocab_size
    attn = cfg.n_layers * 6 * seq_len * cfg.dim  # 12 * L * S * d / 2 (causal)
    return 6.0 * n + attn


__all__ = [
    "Block",
    "FeedForward",
    "Llama",
    "LlamaConfig",
    "PRESETS",
    "RMSNorm",
    "apply_rope",
    "flops_per_token",
    "lm_loss",
    "muon_and_adam_params",
    "param_count",
    "preset",
    "rope_tables",
]
