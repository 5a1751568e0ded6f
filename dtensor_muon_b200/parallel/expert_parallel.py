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
    """Destination of every (sorted) source row and the local receive layout."""

    def __init__(self, counts_all: Tensor, rank: int, world: int, n_experts: int):
        # counts_all: CPU int64 [W, E] = rows source rank s sends to expert e
        self.world, self.rank = world, rank
        el = n_experts // world
        self.local_experts = el
        # receive offsets: owner d, local expert e, source s -> row
        off = torch.zeros(world, n_experts, dtype=torch.int64)
        for d in range(world):
            cur = 0
            for e in range(d * el, (d + 1) * el):
                for s in range(world):
                    off[s, e] = cur
                    cur += int(counts_all[s, e])
        self.recv_rows = [int(counts_all[:, d * el:(d + 1) * el].sum()) for d in range(world)]
        mine = counts_all[rank]  # rows I send per expert, in expert order (rows are pre-sorted)
        dst_rank, dst_row = [], []
        for e in range(n_experts):
            n = int(mine[e])
            if n:
                dst_rank += [e // el] * n
                base = int(off[rank, e])
                dst_row += list(range(base, base + n))
        self.dst_rank = torch.tensor(dst_rank, dtype=torch.int32)
        self.dst_row = torch.tensor(dst_row, dtype=torch.int32)
        self.local_counts = counts_all[:, rank * el:(rank + 1) * el].sum(0)  # per local expert
        self.send_split = [int(mine[d * el:(d + 1) * el].sum()) for d in range(world)]
        self.recv_split = [int(counts_all[s, rank * el:(rank + 1) * el].sum()) for s in range(world)]
        # NCCL receive order is (source, local expert); permutation to (local expert, source)
        perm = []
        src_base = torch.tensor([0] + self.recv_split).cumsum(0)
        for e in range(el):
            for s in range(world):
                n = int(counts_all[s, rank * el + e])
                start = int(src_base[s]) + int(counts_all[s, rank * el:rank * el + e].sum())
                perm += list(range(start, start + n))
        self.nccl_perm = torch.tensor(perm, dtype=torch.int64)

    def to(self, device):
        self.dst_rank_d = self.dst_rank.to(device, non_blocking=True)
        self.dst_row_d = self.dst_row.to(device, non_blocking=True)
        self.nccl_perm_d = self.nccl_perm.to(device, non_blocking=True)
        return self


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
        out = torch.empty(plan.dst_rank.numel(), local.shape[1], dtype=local.dtype, device=local.device)
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
        gathered = [torch.empty_like(counts) for _ in range(self.world)]
        dist.all_gather(gathered, counts, group=self.group)
        counts_all = torch.stack(gathered).cpu()
        order = torch.argsort(expert_ids, stable=True)
        return _Plan(counts_all, self.rank, self.world, self.n_experts).to(expert_ids.device), order, counts

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
