"""Tensor parallelism (Megatron-style) for the Llama / Mixtral attention and MLP,
composed with FSDP2 on a 2-D (dp, tp) mesh.

Column-parallel: wq, wk, wv, w1 (gate), w3 (up) -> weights Shard(0) on tp.
Row-parallel:    wo, w2 (down)                   -> weights Shard(1) on tp.
Heads are split across tp ranks (the attention module infers local head
counts from the projected width). The optimizer sees 2-D-mesh DTensors and
orthogonalises full matrices gathered across the TP group, as the reference
does (src/muonium/orthogonalize/orthogonalize.py:140-155).
"""

from __future__ import annotations

from torch import nn


def tp_plan(block: nn.Module) -> dict:
    from torch.distributed.tensor.parallel import ColwiseParallel, RowwiseParallel

    plan = {
        "attention.wq": ColwiseParallel(),
        "attention.wk": ColwiseParallel(),
        "attention.wv": ColwiseParallel(),
        "attention.wo": RowwiseParallel(),
    }
    if hasattr(block.feed_forward, "w1") and isinstance(block.feed_forward.w1, nn.Linear):
        plan.update(
            {
                "feed_forward.w1": ColwiseParallel(),
                "feed_forward.w3": ColwiseParallel(),
                "feed_forward.w2": RowwiseParallel(),
            }
        )
    return plan


def apply_tensor_parallel(model: nn.Module, tp_mesh) -> nn.Module:
    """Shard every decoder block's projections over ``tp_mesh`` (1-D)."""
    from torch.distributed.tensor.parallel import parallelize_module

    tp = tp_mesh.size()
    for block in model.layers:
        att = block.attention
        if att.n_heads % tp or att.n_kv_heads % tp:
            raise ValueError(f"{att.n_heads} heads / {att.n_kv_heads} kv heads do not split over tp={tp}")
        parallelize_module(block, tp_mesh, tp_plan(block))
    return model


def apply_fsdp_tp(model: nn.Module, mesh) -> nn.Module:
    """TP over ``mesh['tp']`` then FSDP2 over ``mesh['dp']`` (every block and the root)."""
    from torch.distributed.fsdp import fully_shard

    apply_tensor_parallel(model, mesh["tp"])
    for block in model.layers:
        fully_shard(block, mesh=mesh["dp"])
    fully_shard(model, mesh=mesh["dp"])
    return model
