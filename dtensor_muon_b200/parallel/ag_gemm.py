"""Parameter all-gather fused into the first forward GEMM (``y = x @ W^T`` with W
row-sharded over a process group), and the FSDP-style linear built on it.

``AllGatherGemm`` owns the symmetric slot buffer, the ready flags and the
parity-indexed work counters of the fused kernel (``ops/csrc/ag_gemm.cu``):
one call gathers every rank's shard of W into a local ``wg`` and multiplies, the
gather overlapping the tcgen05 GEMM tile by tile. ``wg`` is returned so the
backward can reuse it (no second all-gather).

``AllGatherLinear`` is the autograd function: forward is the fused kernel,
backward computes ``dx = dy @ wg`` and the local weight gradient
``dW_shard = reduce_scatter(dy^T @ x)``.

The reference has no model or forward pass; its FSDP all-gather is FSDP2's
(NCCL) ahead of cuBLAS, which is the unfused baseline this replaces.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import _ext
from . import symm

_COUNTER_INTS = 2 * (2 + 1024)


class AllGatherGemm:
    """Fused all-gather + GEMM over ``group`` (all calls on one CUDA stream, SPMD order)."""

    def __init__(self, group: dist.ProcessGroup | None, device: torch.device):
        self.device = torch.device(device)
        self.group = group
        if group is None:
            self.rank, self.world = 0, 1
            self.ws = None
        else:
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
            self.ws = symm.workspace_for(group, self.device, "ag_gemm") if self.world > 1 else None
        self.counters = torch.zeros(_COUNTER_INTS, dtype=torch.int32, device=self.device)
        self._cap = 0
        self._epoch = 0
        self._empty = torch.empty(0, dtype=torch.int64, device=self.device)

    def __call__(self, x: torch.Tensor, shard: torch.Tensor, wg: torch.Tensor | None = None,
                 out: torch.Tensor | None = None, max_pairs: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        assert x.dtype == torch.bfloat16 and shard.dtype == torch.bfloat16
        x = x.contiguous()
        shard = shard.contiguous()
        n = shard.shape[0] * self.world
        if wg is None:
            wg = torch.empty(n, shard.shape[1], dtype=shard.dtype, device=self.device)
        if out is None:
            out = torch.empty(x.shape[0], n, dtype=x.dtype, device=self.device)
        if self.ws is None:
            self._epoch += 1
            _ext.load().ag_gemm(x, shard, wg, out, self._empty, 0, self._empty, self.counters,
                                0, 1, self._epoch, max_pairs)
            return out, wg
        nbytes = shard.numel() * shard.element_size()
        if nbytes > self._cap:
            # every previous call on every rank has finished before the slot layout changes
            if self._cap:
                self.ws.barrier()
            self._cap = (nbytes + 4095) // 4096 * 4096
        _, peer_base = self.ws.buffer(2 * self._cap)
        flag_ptrs = self.ws._signal_ptrs()
        epoch = self.ws.next_signal_epoch()
        _ext.load().ag_gemm(x, shard, wg, out, peer_base, (epoch & 1) * self._cap, flag_ptrs, self.counters,
                            self.rank, self.world, epoch, max_pairs)
        return out, wg

    def check(self) -> None:
        _ext.check_device_errors(self.device)


_ENGINES: dict[tuple, AllGatherGemm] = {}


def engine_for(group: dist.ProcessGroup | None, device: torch.device) -> AllGatherGemm:
    key = (None if group is None else group.group_name, torch.device(device).index)
    eng = _ENGINES.get(key)
    if eng is None:
        eng = AllGatherGemm(group, device)
        _ENGINES[key] = eng
    return eng


class AllGatherLinear(torch.autograd.Function):
    """``y = x @ all_gather(W_shard)^T`` with the gather fused into the GEMM."""

    @staticmethod
    def forward(ctx, x, shard, group):
        eng = engine_for(group, x.device)
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        y, wg = eng(x2, shard)
        ctx.save_for_backward(x2, wg)
        ctx.group = group
        ctx.lead = lead
        return y.view(*lead, wg.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, wg = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1])
        dx = (dy2 @ wg).view(*ctx.lead, wg.shape[1])
        dw = dy2.t() @ x2
        group = ctx.group
        if group is not None and dist.get_world_size(group) > 1:
            world = dist.get_world_size(group)
            dshard = torch.empty(dw.shape[0] // world, dw.shape[1], dtype=dw.dtype, device=dw.device)
            dist.reduce_scatter_tensor(dshard, dw, group=group)
        else:
            dshard = dw
        return dx, dshard, None


def all_gather_linear(x: torch.Tensor, shard: torch.Tensor, group: dist.ProcessGroup | None) -> torch.Tensor:
    return AllGatherLinear.apply(x, shard, group)
