"""FSDP2 parameter all-gather and gradient reduce-scatter on our NVLink P2P kernels.

FSDP2 (``torch.distributed.fsdp.fully_shard``) keeps its scheduling (prefetch,
streams, copy-in / copy-out); only the two collectives are replaced, through
``FSDPModule.set_custom_all_gather`` / ``set_custom_reduce_scatter``:

* all-gather (default, pull): this rank's shard goes into slot ``rank`` of its
  own symmetric staging, one bounded device barrier, then ``pull_slots`` loads
  every peer's slot over NVLink straight into FSDP's output. (Push variant:
  ``push_slots`` stores the shard into every peer's staging, barrier, local copy.)
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

    A push call stores into every peer's current half, passes one barrier and
    then reads only its own half; a pull call writes only its own slot of its
    own half, passes the barrier and reads every peer's half. Either way the
    barrier of call i + 1 orders every rank's reads of half i % 2 (call i)
    before anyone writes into it again (call i + 2).
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


_STAGING: dict[str, _PushStaging] = {}


def _staging(purpose: str) -> _PushStaging:
    # One staging (one double-buffer parity) per purpose, shared by every FSDP module.
    if purpose not in _STAGING:
        _STAGING[purpose] = _PushStaging(purpose)
    return _STAGING[purpose]


# All-gather scheme. Every scheme puts this rank's shard into its own staging
# slot (or every peer's), passes one bounded barrier and then fills FSDP's output:
#  "ce" (default): W - 1 device copies from the peers' slots straight into the
#       output, executed by the copy engines: no SM is taken from the model
#       GEMMs that overlap the all-gather (W = 2, 436 MB: 0.49 ms alone vs
#       NCCL 0.67 ms; under a concurrent GEMM loop 1.13 ms and +0.09 ms on the
#       GEMMs, vs NCCL 1.59 ms and +0.50 ms);
#  "pull": the same transfer by the pull_slots kernel (P2P loads on SMs);
#  "push": push_slots stores the shard into every peer's staging, then one
#       local copy of the W slots into the output.
AG_MODE = os.environ.get("DMB_AG_MODE", "ce")
# Reduce-scatter scheme: "ce" (default): the W chunks go to their owners'
# staging by copy-engine copies, barrier, local fp32 slot sum; "push": the same
# with the push_slots kernel; "nvls": this rank's full input goes into its own
# staging by a copy-engine copy, barrier, then one multimem.ld_reduce kernel
# reads the sum of its own chunk through the switch (needs a multicast
# address); "auto" = "ce". Measured at W = 2 on a 436 MB layer
# (benchmarks/bench_fsdp_comm.py): ce 0.90 ms alone and 2.17 ms under a
# concurrent GEMM loop that it slows by 0.22 ms; NCCL 0.72 / 2.39 ms, +1.06 ms;
# push 0.83 / 2.46, +0.68; nvls 2.24 / 2.68, +0.36 (the full-size local copy
# into staging dominates it).
RS_MODE = os.environ.get("DMB_RS_MODE", "ce")


class P2PAllGather(AllGather):
    """All-gather over peer memory (see ``AG_MODE``)."""

    def __init__(self):
        self._stage = _staging("fsdp_ag")

    def allocate(self, size, *, dtype, device):
        return torch.empty(*size, dtype=dtype, device=device)

    def __call__(self, output_tensor, input_tensor, group, async_op=False):
        nbytes = input_tensor.numel() * input_tensor.element_size()
        if nbytes % 16 or not output_tensor.is_contiguous() or not input_tensor.is_contiguous():
            return dist.all_gather_into_tensor(output_tensor, input_tensor, group=group, async_op=async_op)
        world = dist.get_world_size(group)
        ws, buf, peers, off = self._stage.half(group, output_tensor.device, nbytes * world)
        C = _ext.load()
        if AG_MODE in ("ce", "pull"):
            mine = off + ws.rank * nbytes
            src = input_tensor.view(-1).view(torch.uint8)
            buf[mine : mine + nbytes].copy_(src)
            ws.barrier()  # every rank's shard is in its own staging slot
            if AG_MODE == "pull":
                C.pull_slots(output_tensor.view(-1), peers, off, nbytes, ws.rank, world, COMM_CTAS)
                return None
            out = output_tensor.view(-1).view(torch.uint8)
            if src.data_ptr() != out.data_ptr() + ws.rank * nbytes:  # FSDP's input is normally this slot
                out[ws.rank * nbytes : (ws.rank + 1) * nbytes].copy_(src)
            for j in range(1, world):
                k = (ws.rank + j) % world
                out[k * nbytes : (k + 1) * nbytes].copy_(ws.peer_bytes(k, off + k * nbytes, nbytes))
            return None
        C.push_slots(input_tensor, peers, off, nbytes, ws.rank, world, False, COMM_CTAS)
        ws.barrier()  # every shard has landed in every rank's staging
        output_tensor.view(-1).view(torch.uint8).copy_(buf[off : off + nbytes * world])
        return None


class P2PReduceScatter(ReduceScatter):
    """Reduce-scatter by P2P stores: chunk k -> slot ``rank`` of peer k, then a local fp32 sum.

    With a :class:`FusedMomentum` attached (one instance per FSDP module), the
    local sum also applies the Muon momentum / Nesterov update of that module's
    Muon parameters (``rs_sum_momentum``) and leaves g' as their gradient.
    """

    def __init__(self, module=None, fused=None, purpose: str = "fsdp_rs"):
        # callers that issue reduce-scatters on another stream pass their own purpose
        # (own symmetric workspace, own barrier sequence)
        self._stage = _staging(purpose)
        self._module = module
        self._fused = fused

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
        segs = self._fused.segments(self._module, output_tensor, world) if self._fused is not None else None
        mode = RS_MODE
        if mode == "auto":
            mode = "ce"
        if mode == "nvls" and ws.mc_base and segs is None:
            # my full input at my staging offset; the switch sums chunk `rank` over all ranks
            buf[off : off + slot * world].copy_(input_tensor.view(-1).view(torch.uint8))
            ws.barrier()  # every rank's input is in its staging
            C.multimem_reduce_to_local(output_tensor, ws.mc_base + off + ws.rank * slot, scale, COMM_CTAS)
            return None
        if mode == "ce":
            src = input_tensor.view(-1).view(torch.uint8)
            for j in range(world):
                k = (ws.rank + j) % world
                dst = off + ws.rank * slot  # slot `rank` of peer k's staging
                piece = src[k * slot : (k + 1) * slot]
                if k == ws.rank:
                    buf[dst : dst + slot].copy_(piece)
                else:
                    ws.peer_bytes(k, dst, slot).copy_(piece)
        else:
            C.push_slots(input_tensor, peers, off, slot, ws.rank, world, True, COMM_CTAS)
        ws.barrier()  # every rank's chunk for me has landed
        if segs is not None:
            C.rs_sum_momentum(output_tensor, buf, off, world, scale, segs, 2 * COMM_CTAS)
        else:
            C.local_slot_sum(output_tensor, buf, off, world, scale, 2 * COMM_CTAS)
        return None


# Parameters whose current .grad already holds the Nesterov input g' (their
# momentum buffer was updated inside the reduce-scatter). The optimizer consumes
# and clears the marks in its next step.
FUSED_GRADS: set[int] = set()


class FusedMomentum:
    """Maps each FSDP module's reduce-scatter output to its Muon parameters' momentum buffers.

    Fusion applies to 2-D, dim-0-sharded Muon parameters on a 1-D mesh whose
    momentum buffer already exists (from the first optimizer step on) and
    whose gradient is not being accumulated (no ``.grad`` when the reduce-
    scatter runs). Every other parameter gets the plain reduced gradient.
    """

    def __init__(self, optimizer):
        self.opt = optimizer
        self.group_of = {id(p): g for g in optimizer.param_groups for p in g["params"]}

    def segments(self, module, output: torch.Tensor, world: int):
        try:
            fsdp_params = module._get_fsdp_state()._fsdp_param_group.fsdp_params
        except AttributeError:  # private FSDP2 layout changed: no fusion
            return None
        rows, off, fused_ids = [], 0, []
        for fp in fsdp_params:
            p = fp.sharded_param
            shape = tuple(p.shape)
            padded0 = -(-shape[0] // world) * world
            rest = 1
            for d in shape[1:]:
                rest *= d
            seg = padded0 * rest // world
            local = p.to_local()
            buf_ptr, flags, mom = 0, 0, 0.0
            g = self.group_of.get(id(p))
            st = self.opt.state.get(p, {})
            mb = st.get("momentum_buffer") if st else None
            if (
                g is not None and g.get("use_muon") and mb is not None and p.grad is None and len(shape) == 2
                and not g.get("flatten") and g.get("split_sizes") is None and hasattr(mb, "to_local")
                and mb.to_local().dtype == torch.float32 and mb.to_local().is_contiguous()
                and mb.to_local().numel() == local.numel() and local.numel() % 8 == 0 and off % 8 == 0
                and output.dtype == p.dtype and mb.to_local().data_ptr() % 16 == 0
            ):
                buf_ptr = mb.to_local().data_ptr()
                flags = int(bool(g["nesterov"])) | (int(bool(g["maximize"])) << 1)
                mom = float(g["momentum"])
                fused_ids.append(id(p))
            import struct

            rows.append([off, local.numel(), buf_ptr, flags, struct.unpack("<i", struct.pack("<f", mom))[0]])
            off += seg
        if not fused_ids or off != output.numel() or len(rows) > 64 or any(r[0] % 8 for r in rows):
            return None
        FUSED_GRADS.update(fused_ids)
        return torch.tensor(rows, dtype=torch.int64).pin_memory().to(output.device, non_blocking=True)


def use_p2p_collectives(model: torch.nn.Module, optimizer=None) -> int:
    """Install the P2P all-gather / reduce-scatter on every FSDP module of ``model``.

    With ``optimizer`` (a Muon), the reduce-scatter also runs the momentum
    update of the module's Muon parameters (see :class:`FusedMomentum`).
    Returns the number of FSDP modules configured (0 when symmetric memory is unavailable).
    """
    from torch.distributed.fsdp import FSDPModule

    if not symm.available():
        return 0
    ag = P2PAllGather()
    fused = FusedMomentum(optimizer) if optimizer is not None else None
    n = 0
    for m in model.modules():
        if isinstance(m, FSDPModule):
            m.set_custom_all_gather(ag)
            m.set_custom_reduce_scatter(P2PReduceScatter(m, fused))
            n += 1
    return n
