"""FSDP2 parameter all-gather and gradient reduce-scatter on our NVLink P2P kernels.

FSDP2 (``torch.distributed.fsdp.fully_shard``) keeps its scheduling (prefetch,
streams, copy-in / copy-out); only the two collectives are replaced, through
``FSDPModule.set_custom_all_gather`` / ``set_custom_reduce_scatter``:

* all-gather: ``push_slots`` stores this rank's shard into slot ``rank`` of
  every rank's symmetric staging (posted NVLink stores), one bounded device
  barrier, then a local copy of the W slots into FSDP's output.
* reduce-scatter: ``push_slots`` stores chunk ``k`` of the local gradient into
  slot ``rank`` of rank k's staging, one barrier, then ``local_slot_sum`` adds
  the W slots in fp32 (one bf16 rounding instead of one per hop).
Staging is double-buffered, so one barrier per collective suffices.

Each collective has its own symmetric workspace (own barrier sequence)
because FSDP issues them on different streams. Output buffers are ordinary
caching-allocator memory, so FSDP's buffer lifetimes are unchanged.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch.distributed.fsdp._fully_shard._fsdp_api import AllGather, ReduceScatter

from ..ops import _ext
from . import symm

# Grid cap of the copy kernels (they overlap with compute on other streams).
COMM_CTAS = int(os.environ.get("DMB_COMM_CTAS", "64"))


def _ws(group, device, purpose):
    return symm.workspace_for(group, device, purpose)


class _PushStaging:
    """Double-buffered staging in one symmetric buffer: call i uses half i % 2.

    A call pushes into every peer's current half, passes one barrier and then
    reads only its own half. The barrier of call i + 1 orders every rank's
    reads of half i % 2 (call i) before anyone pushes into it again (call i + 2).
    """

    def __init__(self, purpose: str):
        self.purpose = purpose
        self.calls = 0

    def half(self, group, device, nbytes):
        ws = _ws(group, device, self.purpose)
        half = (nbytes + 255) // 256 * 256
        buf, peers = ws.buffer(2 * half)
        off = (self.calls % 2) * half
        self.calls += 1
        return ws, buf, peers, off


class P2PAllGather(AllGather):
    """All-gather by P2P stores: shard -> slot ``rank`` of every peer's staging."""

    def __init__(self):
        self._stage = _PushStaging("fsdp_ag")

    def allocate(self, size, *, dtype, device):
        return torch.empty(*size, dtype=dtype, device=device)

    def __call__(self, output_tensor, input_tensor, group, async_op=False):
        nbytes = input_tensor.numel() * input_tensor.element_size()
        if nbytes % 16 or not output_tensor.is_contiguous() or not input_tensor.is_contiguous():
            return dist.all_gather_into_tensor(output_tensor, input_tensor, group=group, async_op=async_op)
        world = dist.get_world_size(group)
        ws, buf, peers, off = self._stage.half(group, output_tensor.device, nbytes * world)
        C = _ext.load()
        C.push_slots(input_tensor, peers, off, nbytes, ws.rank, world, False, COMM_CTAS)
        ws.barrier()  # every shard has landed in every rank's staging
        output_tensor.view(-1).view(torch.uint8).copy_(buf[off : off + nbytes * world])
        return None


class P2PReduceScatter(ReduceScatter):
    """Reduce-scatter by P2P stores: chunk k -> slot ``rank`` of peer k, then a local fp32 sum."""

    def __init__(self):
        self._stage = _PushStaging("fsdp_rs")

    def allocate(self, size, *, dtype, device):
        return torch.empty(*size, dtype=dtype, device=device)

    def __call__(self, output_tensor, input_tensor, group, op, async_op=False):
        world = dist.get_world_size(group)
        scale = {dist.ReduceOp.SUM: 1.0, dist.ReduceOp.AVG: 1.0 / world}.get(op)
        ok = (
            scale is not None
            and output_tensor.dtype in (torch.float32, torch.bfloat16)
            and output_tensor.numel() % 8 == 0
            and output_tensor.is_contiguous()
            and input_tensor.is_contiguous()
            and input_tensor.dtype == output_tensor.dtype
        )
        if not ok:
            return dist.reduce_scatter_tensor(output_tensor, input_tensor, op=op, group=group, async_op=async_op)
        slot = output_tensor.numel() * output_tensor.element_size()
        ws, buf, peers, off = self._stage.half(group, output_tensor.device, slot * world)
        C = _ext.load()
        C.push_slots(input_tensor, peers, off, slot, ws.rank, world, True, COMM_CTAS)
        ws.barrier()  # every rank's chunk for me has landed
        C.local_slot_sum(output_tensor, buf, off, world, scale, 2 * COMM_CTAS)
        return None


def use_p2p_collectives(model: torch.nn.Module) -> int:
    """Install the P2P all-gather / reduce-scatter on every FSDP module of ``model``.

    Returns the number of FSDP modules configured (0 when symmetric memory is unavailable).
    """
    from torch.distributed.fsdp import FSDPModule

    if not symm.available():
        return 0
    ag, rs = P2PAllGather(), P2PReduceScatter()
    n = 0
    for m in model.modules():
        if isinstance(m, FSDPModule):
            m.set_custom_all_gather(ag)
            m.set_custom_reduce_scatter(rs)
            n += 1
    return n
