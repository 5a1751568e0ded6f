"""Expert parallelism: top-k token dispatch to the rank owning each expert and
the matching combine, over NVLink peer memory (``backend="p2p"``) or an NCCL
all-to-all (``backend="nccl"``, the baseline).

The reference has no token exchange (it ships no model). Its EP support is the
collective-free orthogonalisation of dim-0-sharded expert stacks
(``src/muonium/orthogonalize/orthogonalize.py:177-204``, ``README.md:10-11``),
which ``foreach_zeropower_3d_fsdp`` here keeps.

Layout. With ``W`` ranks and ``E`` experts, rank ``r`` owns experts
``[r*E/W, (r+1)*E/W)``. A rank's receive region holds its tokens grouped by
local expert, and within an expert by source rank, so the expert GEMMs consume
it directly. Every rank learns the full [W, E] count matrix with one small
all-gather, from which each source row's destination rank and row follow
without further communication.

P2P path, per layer:
  dispatch  forward: ep_scatter_rows into the owners' regions, barrier, copy out
            backward: grads into my region, barrier, ep_gather_rows
  combine   forward: results into my region, barrier, ep_gather_rows
            backward: ep_scatter_rows into the owners' regions, barrier, copy out
Each exchange ends with a second barrier before the region can be reused.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor

from ..ops import _ext
from . import symm


class _Plan:
    """Destination of every (sorted) source row and the local receive layout.

    Built from the [W, E] count matrix with vectorised tensor ops on the
    tokens' device: per-row destinations (rank, row) and the NCCL receive
    permutation never pass through Python loops. The only host transfer is the
    W x E count matrix itself (one small copy per layer), which sizes the
    receive buffers and the expert GEMMs.
    """

    def __init__(self, counts_all: Tensor, sorted_experts: Tensor, rank: int, world: int, n_experts: int):
        # counts_all: int64 [W, E] on the device = rows source rank s sends to expert e
        # sorted_experts: this rank's expert id per sorted row (ascending)
        self.world, self.rank = world, rank
        el = n_experts // world
        self.local_experts = el
        dev = counts_all.device
        # Receive layout of owner d: (local expert, source) blocks in order.
        # off[s, e] = rows of owner(e) before block (e, s).
        blocks = counts_all.t().reshape(world, el, world)  # [owner, local e, source]
        flat = blocks.reshape(world, el * world)
        before = torch.cumsum(flat, dim=1) - flat  # exclusive, within owner
        off = before.reshape(world, el, world).permute(2, 0, 1).reshape(world, n_experts)  # [s, e]
        # Destination of each of my sorted rows: owner of its expert, off + rank within its expert run
        mine = counts_all[rank]
        start = torch.cumsum(mine, 0) - mine
        e = sorted_experts.long()
        pos = torch.arange(e.numel(), device=dev)
        self.dst_rank_d = (e // el).to(torch.int32)
        self.dst_row_d = (off[rank].index_select(0, e) + pos - start.index_select(0, e)).to(torch.int32)
        # Host-side sizes: one [W, E] copy.
        host = counts_all.cpu()
        self.recv_rows = host.t().reshape(world, el * world).sum(1).tolist()
        self.local_counts = host[:, rank * el:(rank + 1) * el].sum(0)  # per local expert
        self.send_split = host[rank].reshape(world, el).sum(1).tolist()
        self.recv_split = host[:, rank * el:(rank + 1) * el].sum(1).tolist()
        # NCCL receives (source, local expert) blocks; permutation to (local expert, source).
        c_se = counts_all[:, rank * el:(rank + 1) * el]  # [s, e_local]
        old_start = (torch.cumsum(c_se.reshape(-1), 0) - c_se.reshape(-1)).reshape(world, el)
        c_es = c_se.t().reshape(-1)  # blocks in (e, s) order
        new_start = torch.cumsum(c_es, 0) - c_es
        total = int(self.recv_rows[rank])
        idx = torch.arange(total, device=dev)
        blk_old = torch.repeat_interleave(old_start.t().reshape(-1), c_es, output_size=total)
        blk_new = torch.repeat_interleave(new_start, c_es, output_size=total)
        self.nccl_perm_d = blk_old + (idx - blk_new)

    @property
    def n_send(self) -> int:
        return int(self.dst_rank_d.numel())


class _P2PExchange:
    def __init__(self, ws: symm.SymmetricWorkspace):
        self.ws = ws

    def region(self, rows: int, dim: int, dtype) -> tuple[Tensor, Tensor]:
        nbytes = max(rows, 1) * dim * torch.tensor([], dtype=dtype).element_size()
        buf, peers = self.ws.buffer(nbytes)
        return buf[:nbytes].view(dtype).view(max(rows, 1), dim)[:rows], peers

    def scatter(self, src: Tensor, plan: _Plan, out_rows: int) -> Tensor:
        C = _ext.load()
        region, peers = self.region(max(plan.recv_rows), src.shape[1], src.dtype)
        self.ws.barrier()  # previous users of the region are done
        C.ep_scatter_rows(src.contiguous(), plan.dst_rank_d, plan.dst_row_d, peers, 0)
        self.ws.barrier()  # every row has landed
        return region[:out_rows].clone()

    def gather(self, local: Tensor, plan: _Plan) -> Tensor:
        C = _ext.load()
        region, peers = self.region(max(plan.recv_rows), local.shape[1], local.dtype)
        self.ws.barrier()
        region[: local.shape[0]].copy_(local)
        self.ws.barrier()  # every owner's results are in place
        out = torch.empty(plan.n_send, local.shape[1], dtype=local.dtype, device=local.device)
        C.ep_gather_rows(out, plan.dst_rank_d, plan.dst_row_d, peers, 0)
        return out


class _Dispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, rows, ep, plan):
        ctx.ep, ctx.plan = ep, plan
        return ep._send(rows, plan)

    @staticmethod
    def backward(ctx, grad):
        return ctx.ep._recv_back(grad.contiguous(), ctx.plan), None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, ep, plan):
        ctx.ep, ctx.plan = ep, plan
        return ep._recv_back(y.contiguous(), plan)

    @staticmethod
    def backward(ctx, grad):
        return ctx.ep._send(grad.contiguous(), ctx.plan), None, None


class ExpertParallel:
    """Routes top-k token copies to expert owners and back across ``group``."""

    def __init__(self, group: dist.ProcessGroup, n_experts: int, backend: str = "p2p"):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split over {self.world} ranks")
        self.n_experts = n_experts
        self.local_experts = n_experts // self.world
        if backend == "p2p" and not symm.available():
            backend = "nccl"
        self.backend = backend
        self._p2p = None

    def _exchange(self, device) -> _P2PExchange:
        if self._p2p is None:
            self._p2p = _P2PExchange(symm.workspace_for(self.group, device, "ep"))
        return self._p2p

    def plan(self, expert_ids: Tensor) -> tuple[_Plan, Tensor, Tensor]:
        counts = torch.bincount(expert_ids, minlength=self.n_experts)
        counts_all = torch.empty(self.world * self.n_experts, dtype=counts.dtype, device=counts.device)
        dist.all_gather_into_tensor(counts_all, counts, group=self.group)
        counts_all = counts_all.view(self.world, self.n_experts)
        order = torch.argsort(expert_ids, stable=True)
        plan = _Plan(counts_all, expert_ids.index_select(0, order), self.rank, self.world, self.n_experts)
        return plan, order, counts

    # -- transport: sorted source rows -> my expert-grouped rows, and back
    def _send(self, rows: Tensor, plan: _Plan) -> Tensor:
        if self.backend == "p2p":
            return self._exchange(rows.device).scatter(rows, plan, plan.recv_rows[self.rank])
        out = rows.new_empty(sum(plan.recv_split), rows.shape[1])
        dist.all_to_all_single(out, rows.contiguous(), plan.recv_split, plan.send_split, group=self.group)
        return out.index_select(0, plan.nccl_perm_d)

    def _recv_back(self, y: Tensor, plan: _Plan) -> Tensor:
        if self.backend == "p2p":
            return self._exchange(y.device).gather(y, plan)
        src_order = torch.empty_like(y)
        src_order.index_copy_(0, plan.nccl_perm_d, y)
        out = y.new_empty(sum(plan.send_split), y.shape[1])
        dist.all_to_all_single(out, src_order, plan.send_split, plan.recv_split, group=self.group)
        return out

    def run(self, x: Tensor, idx: Tensor, expert_fn) -> Tensor:
        """x: [T, D]; idx: [T, k] global expert ids. Returns [T*k, D] expert outputs
        in (token, slot) order; ``expert_fn(rows, counts)`` runs the local experts."""
        k = idx.shape[1]
        expert = idx.reshape(-1)
        plan, order, _ = self.plan(expert)
        rows = x.repeat_interleave(k, dim=0)[order]
        recv = _Dispatch.apply(rows, self, plan)
        y = expert_fn(recv, plan.local_counts.to(x.device))
        back = _Combine.apply(y, self, plan)
        out = torch.empty_like(back)
        out[order] = back
        return out


def reduce_dense_grads(params, group: dist.ProcessGroup, expert_params=()) -> None:
    """Data-parallel reduction for an EP model: average the replicated (non-expert)
    grads over the group; expert grads already hold every rank's tokens, so they
    are scaled by 1/W to match the averaged loss."""
    world = dist.get_world_size(group)
    ex = {id(p) for p in expert_params}
    dense = [p.grad for p in params if p.grad is not None and id(p) not in ex]
    if dense:
        flat = torch.cat([g.reshape(-1).float() for g in dense])
        dist.all_reduce(flat, group=group)
        flat.div_(world)
        off = 0
        for g in dense:
            n = g.numel()
            g.copy_(flat[off:off + n].view_as(g))
            off += n
    for p in expert_params:
        if p.grad is not None:
            p.grad.div_(world)


def shard_experts(model: torch.nn.Module, mesh, ep: ExpertParallel) -> list[torch.nn.Parameter]:
    """Turn every MoE layer's stacked expert weights into DTensors sharded on dim 0
    over the 1-D ``mesh`` (each rank keeps its local experts) and attach ``ep``.
    Returns the new expert parameters."""
    from torch.distributed.tensor import Shard, distribute_tensor

    from ..models.mixtral import MoEFeedForward

    out = []
    for mod in model.modules():
        if isinstance(mod, MoEFeedForward):
            for name in ("w1", "w2", "w3"):
                full = getattr(mod, name).detach()
                p = torch.nn.Parameter(distribute_tensor(full, mesh, [Shard(0)]))
                setattr(mod, name, p)
                out.append(p)
            mod.ep = ep
    return out
