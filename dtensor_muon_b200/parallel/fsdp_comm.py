"""FSDP2 parameter all-gather and gradient reduce-scatter on our NVLink P2P kernels.

FSDP2 (``torch.distributed.fsdp.fully_shard``) keeps its scheduling (prefetch,
streams, copy-in / copy-out); only the two collectives are replaced, through
``FSDPModule.set_custom_all_gather`` / ``set_custom_reduce_scatter``:

* all-gather: the local shard is staged in this rank's symmetric buffer,
  bounded device barrier, then ``fsdp_all_gather_pull`` reads every rank's
  shard straight from its buffer (16-byte P2P loads) into the output, barrier.
* reduce-scatter: the local full gradient is staged, barrier, then
  ``fsdp_reduce_scatter_pull`` reads this rank's chunk from every peer and
  sums in fp32 (one bf16 rounding instead of one per hop), barrier.

Each collective has its own symmetric workspace (own barrier sequence)
because FSDP issues them on different streams. Output buffers are ordinary
caching-allocator memory, so FSDP's buffer lifetimes are unchanged.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch.distributed.fsdp._fully_shard._fsdp_api import AllGather, ReduceScatter

from ..ops import _ext
from . import symm

# Grid cap of the copy kernels: leave most SMs to the overlapped compute.
COMM_CTAS = 32


def _ws(group, device, purpose):
    return symm.workspace_for(group, device, purpose)


class P2PAllGather(AllGather):
    def allocate(self, size, *, dtype, device):
        return torch.empty(*size, dtype=dtype, device=device)

    def __call__(self, output_tensor, input_tensor, group, async_op=False):
        ws = _ws(group, output_tensor.device, "fsdp_ag")
        nbytes = input_tensor.numel() * input_tensor.element_size()
        if nbytes % 16 or not output_tensor.is_contiguous():
            return dist.all_gather_into_tensor(output_tensor, input_tensor, group=group, async_op=async_op)
        buf, peers = ws.buffer(nbytes)
        buf[:nbytes].view(input_tensor.dtype).copy_(input_tensor.reshape(-1))
        ws.barrier()  # every rank's shard is staged
        _ext.load().fsdp_all_gather_pull(output_tensor, peers, 0, nbytes, ws.world, COMM_CTAS)
        ws.barrier()  # every peer has read my staged shard
        return None


class P2PReduceScatter(ReduceScatter):
    def allocate(self, size, *, dtype, device):
        return torch.empty(*size, dtype=dtype, device=device)

    def __call__(self, output_tensor, input_tensor, group, op, async_op=False):
        world = dist.get_world_size(group)
        if op == dist.ReduceOp.SUM:
            scale = 1.0
        elif op == dist.ReduceOp.AVG:
            scale = 1.0 / world
        else:
            scale = None
        ok = (
            scale is not None
            and output_tensor.dtype in (torch.float32, torch.bfloat16)
            and output_tensor.numel() % 8 == 0
            and output_tensor.is_contiguous()
            and input_tensor.dtype == output_tensor.dtype
        )
        if not ok:
            return dist.reduce_scatter_tensor(output_tensor, input_tensor, op=op, group=group, async_op=async_op)
        ws = _ws(group, output_tensor.device, "fsdp_rs")
        nbytes = input_tensor.numel() * input_tensor.element_size()
        buf, peers = ws.buffer(nbytes)
        buf[:nbytes].view(input_tensor.dtype).copy_(input_tensor.reshape(-1))
        ws.barrier()
        _ext.load().fsdp_reduce_scatter_pull(output_tensor, peers, 0, ws.rank, world, scale, COMM_CTAS)
        ws.barrier()
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
