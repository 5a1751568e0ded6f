"""Training harness: model construction (optionally FSDP2-sharded), the Muon +
AdamW optimizer split, synthetic data and one training step.

This is the public entry point a user calls to train with the framework:

    model = build_llama(preset("llama3-8b"), device)
    opt = build_optimizer(model)
    trainer = Trainer(model, opt)
    loss = trainer.step(tokens, targets)
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor, nn

from .models.llama import Llama, LlamaConfig, lm_loss, muon_and_adam_params
from .optim import Muon


def build_llama(
    cfg: LlamaConfig,
    device: torch.device,
    dtype: torch.dtype = torch.bfloat16,
    mesh=None,
    seed: int | None = 0,
    block_factory=None,
    reshard_after_forward: bool = False,
    fsdp_comm: str = "p2p",
    fused_gather: bool | str = False,
) -> Llama:
    """Build a randomly initialised Llama on ``device`` without a host copy.

    With ``mesh`` (a 1-D DeviceMesh) every decoder block and the root are
    wrapped with FSDP2 ``fully_shard`` (dim-0 sharding of every parameter).
    ``reshard_after_forward=False`` (default) keeps each block's gathered
    weights until its backward: with 180 GB of HBM per GPU the extra bf16 copy
    of an 8B model (16 GB) is cheap, and it removes the backward re-gather.
    ``fsdp_comm="p2p"`` runs FSDP's all-gather / reduce-scatter on the NVLink
    peer-memory kernels of :mod:`dtensor_muon_b200.parallel.fsdp_comm`;
    ``"nccl"`` keeps FSDP2's NCCL collectives.
    ``fused_gather=True`` (with ``mesh``) takes the q/k/v and gate/up weights out
    of FSDP: they become ``Shard(0)`` DTensors applied by the fused parameter
    all-gather + GEMM kernel (:class:`dtensor_muon_b200.parallel.ag_gemm.GatherLinear`),
    whose gather runs inside the GEMM instead of ahead of it; ``fused_gather="all"``
    does the same for wo and w2 (only the norms stay in FSDP2).
    """
    with torch.device("meta"):
        model = Llama(cfg, block_factory=block_factory).to(dtype)
    if mesh is not None:
        from torch.distributed.fsdp import fully_shard

        ignored: set = set()
        if fused_gather:
            from .parallel.ag_gemm import GatherLinear

            world = mesh.size()

            def make(linears):
                # groups the kernel's layout rules exclude stay on FSDP2
                if not GatherLinear.eligible(linears, world):
                    return None
                g = GatherLinear(linears, mesh)
                ignored.update(g.params)
                return g

            for layer in model.layers:
                att, ffn = layer.attention, layer.feed_forward
                att.gather = make([att.wq, att.wk, att.wv])
                if fused_gather == "all":
                    att.gather_out = make([att.wo])
                if hasattr(ffn, "w1") and hasattr(ffn, "w3"):
                    ffn.gather = make([ffn.w1, ffn.w3])
                    if fused_gather == "all" and ffn.gather is not None:
                        ffn.gather_out = make([ffn.w2])
        kw = dict(ignored_params=ignored) if ignored else {}
        for layer in model.layers:
            fully_shard(layer, mesh=mesh, reshard_after_forward=reshard_after_forward, **kw)
        fully_shard(model, mesh=mesh, reshard_after_forward=reshard_after_forward, **kw)
        # Issue each block's parameter all-gather two blocks ahead of its forward.
        layers = list(model.layers)
        for i, layer in enumerate(layers):
            nxt = layers[i + 1 : i + 3]
            if nxt:
                layer.set_modules_to_forward_prefetch(nxt)
        if fsdp_comm == "p2p" and mesh.size() > 1:
            from .parallel.fsdp_comm import use_p2p_collectives

            use_p2p_collectives(model)
    model.to_empty(device=device)
    if seed is not None:
        torch.manual_seed(seed + (dist.get_rank() if dist.is_initialized() else 0))
    model.init_weights()
    return model


def build_optimizer(model: nn.Module, optimizer_cls=Muon, lr: float = 1e-3, wd: float = 0.1,
                    adam_lr: float | None = None, muon_group: dict | None = None, fuse_momentum: bool = False,
                    **kwargs):
    """Muon on the 2-D / 3-D decoder weights, AdamW on embeddings, norms and head.

    ``fuse_momentum=True`` (FSDP models on the P2P collectives) moves the Muon
    momentum / Nesterov update into FSDP's gradient reduce-scatter, so it runs
    during backward; requires one backward per optimizer step.
    """
    muon, adam = muon_and_adam_params(model)
    groups = [dict(params=muon, **(muon_group or {}))]
    if adam:
        g = {"params": adam, "algorithm": "adamw"}
        if adam_lr is not None:
            g["lr"] = adam_lr
        groups.append(g)
    opt = optimizer_cls(groups, lr=lr, wd=wd, **kwargs)
    if fuse_momentum:
        from .parallel.fsdp_comm import use_p2p_collectives

        use_p2p_collectives(model, opt)
    return opt


def synthetic_batch(batch: int, seq: int, vocab: int, generator: torch.Generator | None = None,
                    pin: bool = False) -> tuple[Tensor, Tensor]:
    """Uniform random token ids; targets are the next token."""
    ids = torch.randint(0, vocab, (batch, seq + 1), generator=generator)
    if pin:
        ids = ids.pin_memory()
    return ids[:, :-1], ids[:, 1:]


class Trainer:
    """forward -> loss -> backward -> optimizer.step -> zero_grad."""

    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer):
        self.model = model
        self.optimizer = optimizer

    def forward_backward(self, tokens: Tensor, targets: Tensor) -> Tensor:
        loss = lm_loss(self.model(tokens), targets)
        loss.backward()
        return loss.detach()

    def step(self, tokens: Tensor, targets: Tensor) -> Tensor:
        loss = self.forward_backward(tokens, targets)
        self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)
        return loss
