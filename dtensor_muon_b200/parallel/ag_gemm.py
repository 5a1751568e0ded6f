"""Parameter all-gather fused into the first forward GEMM (``y = x @ W^T`` with W
row-sharded over a process group), and the FSDP-style linear built on it.

``AllGatherGemm`` owns the symmetric slot buffer, the ready flags and the
parity-indexed work counters of the fused kernel (``ops/csrc/ag_gemm.cu``):
one call gathers every rank's shard of W into a local ``wg`` and multiplies, the
gather overlapping the tcgen05 GEMM tile by tile. ``wg`` is returned so the
backward can reuse it (no second all-gather).

``GatherLinear`` applies several linears that share an input (q/k/v, gate/up)
with one fused call; their weights are ``Shard(0)`` DTensors (FSDP layout).
Backward: ``dx = dy @ wg`` on the current stream, ``dW = reduce_scatter(dy^T x)``
on a side stream, delivered at the end of the backward.

The reference has no model or forward pass; its FSDP all-gather is FSDP2's
(NCCL) ahead of cuBLAS, which is the unfused baseline this replaces.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import _ext
from . import symm

_COUNTER_INTS = 2 * (2 + 2048)
CHUNK_ROWS = 128


def gather_plan(rows: list[int], rank: int, world: int) -> tuple[list[int], list[int], int]:
    """Order of the 128-row chunks of ``wg`` for ``rank`` (its own chunks first, then
    rank + 1's, ...) and the processing order of the 256-row N tiles (by the
    gather position of their later chunk). Returns (gather_order, tile_order,
    number of local chunks)."""
    keys = []
    for n in rows:
        rpr = n // world
        for r in range(0, n, CHUNK_ROWS):
            keys.append(((r // rpr - rank) % world, len(keys)))
    order = [c for _, c in sorted(keys)]
    pos = [0] * len(order)
    for i, c in enumerate(order):
        pos[c] = i
    tiles = sorted(range(len(order) // 2), key=lambda tn: (max(pos[2 * tn], pos[2 * tn + 1]), tn))
    local = sum(1 for k, _ in keys if k == 0)
    return order, tiles, local


class AllGatherGemm:
    """Fused all-gather + GEMM over ``group`` (all calls on one CUDA stream, SPMD order).

    ``eng(x, [shard_0, ...])`` returns ``([x @ W_0^T, ...], wg)`` where W_s is the
    row-concatenation of every rank's ``shard_s`` and ``wg`` holds all W_s stacked
    by rows. Every shard has a multiple of 128 rows; every W_s a multiple of 256.
    """

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
        self._plans: dict[tuple, tuple[torch.Tensor, int]] = {}
        self._empty = torch.empty(0, dtype=torch.int64, device=self.device)

    def _plan(self, rows: tuple[int, ...]) -> tuple[torch.Tensor, int]:
        plan = self._plans.get(rows)
        if plan is None:
            order, tiles, local = gather_plan(list(rows), self.rank, self.world)
            plan = (torch.tensor(order + tiles, dtype=torch.int32).to(self.device), local)
            self._plans[rows] = plan
        return plan

    def __call__(self, x: torch.Tensor, shards, wg: torch.Tensor | None = None, outs=None,
                 max_pairs: int = 0) -> tuple[list[torch.Tensor], torch.Tensor]:
        if isinstance(shards, torch.Tensor):
            shards = [shards]
        assert x.dtype == torch.bfloat16 and all(s.dtype == torch.bfloat16 for s in shards)
        x = x.contiguous()
        shards = [s.contiguous() for s in shards]
        rows = tuple(s.shape[0] * self.world for s in shards)
        if wg is None:
            wg = torch.empty(sum(rows), x.shape[1], dtype=x.dtype, device=self.device)
        if outs is None:
            outs = [torch.empty(x.shape[0], n, dtype=x.dtype, device=self.device) for n in rows]
        elif isinstance(outs, torch.Tensor):
            outs = [outs]
        order, local = self._plan(rows)
        slot_offs, off = [], 0
        for s in shards:
            slot_offs.append(off)
            off += s.numel() * s.element_size()
        if self.ws is None:
            self._epoch += 1
            _ext.load().ag_gemm(x, shards, wg, outs, order, local, slot_offs, self._empty, 0, self._empty,
                                self.counters, 0, 1, self._epoch, max_pairs)
            return outs, wg
        if off > self._cap:
            # every previous call on every rank has finished before the slot layout changes
            if self._cap:
                self.ws.barrier()
            self._cap = (off + 4095) // 4096 * 4096
        _, peer_base = self.ws.buffer(2 * self._cap)
        flag_ptrs = self.ws._signal_ptrs()
        epoch = self.ws.next_signal_epoch()
        _ext.load().ag_gemm(x, shards, wg, outs, order, local, slot_offs, peer_base, (epoch & 1) * self._cap,
                            flag_ptrs, self.counters, self.rank, self.world, epoch, max_pairs)
        return outs, wg

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


class _GatherLinearFn(torch.autograd.Function):
    """outs_s = x @ all_gather(shard_s)^T; the weight gradients go out of band
    (``GatherLinear._reduce_grads``) so their reduce-scatter overlaps the rest of
    the backward instead of blocking it."""

    @staticmethod
    def forward(ctx, x, owner, *shards):
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        outs, wg = engine_for(owner.group, x.device)(x2, list(shards))
        ctx.save_for_backward(x2, wg)
        ctx.owner = owner
        ctx.lead = lead
        ctx.rows = [o.shape[1] for o in outs]
        return tuple(o.view(*lead, o.shape[1]) for o in outs)

    @staticmethod
    def backward(ctx, *dys):
        x2, wg = ctx.saved_tensors
        dys2 = [dy.reshape(-1, dy.shape[-1]) for dy in dys]
        dx = None
        row0 = 0
        for dy, n in zip(dys2, ctx.rows):
            w = wg[row0:row0 + n]
            dx = dy @ w if dx is None else dx.addmm_(dy, w)
            row0 += n
        ctx.owner._reduce_grads(dys2, x2)
        return (dx.view(*ctx.lead, wg.shape[1]), None) + (None,) * len(dys)


_RS: dict = {}


def _reduce_scatter(group):
    """Reduce-scatter used for the weight gradients: the copy-engine scatter + fp32
    local sum over peer memory (``fsdp_comm.P2PReduceScatter``, its own workspace
    because it runs on the side stream), or NCCL when symmetric memory is
    unavailable or ``DMB_GATHER_RS=nccl``."""
    import os

    key = group.group_name
    rs = _RS.get(key)
    if rs is None:
        if os.environ.get("DMB_GATHER_RS", "p2p") == "p2p" and symm.available():
            from .fsdp_comm import P2PReduceScatter

            rs = P2PReduceScatter(purpose="gather_linear_rs")
        else:
            def rs(out, inp, grp, op):
                dist.reduce_scatter_tensor(out, inp, op=op, group=grp)
        _RS[key] = rs
    return rs


class GatherLinear:
    """Up to four ``nn.Linear`` layers that read the same input (q/k/v, gate/up),
    their weights kept as ``Shard(0)`` DTensors over a 1-D mesh (FSDP layout, so
    the Muon optimizer's owner compute handles them like FSDP parameters) and
    applied with the fused all-gather + GEMM kernel.

    Backward: ``dx`` on the current stream from the gathered weights the forward
    kept; each rank's slice of ``dW_s = dy_s^T x`` is computed on a side stream
    straight into a rank-major buffer, reduce-scattered there (mean over ranks,
    as FSDP does), and assigned to ``weight.grad`` at the end of the backward
    after the current stream has waited for the side stream.
    """

    _pending: list = []
    _side: dict = {}

    def __init__(self, linears, mesh):
        from torch.distributed.tensor import DTensor, Shard

        self.linears = list(linears)
        self.mesh = mesh
        self.group = mesh.get_group() if mesh is not None and mesh.size() > 1 else None
        world = mesh.size() if mesh is not None else 1
        for lin in self.linears:
            w = lin.weight
            n, k = w.shape
            assert n % (world * CHUNK_ROWS) == 0 and n % 256 == 0 and k % 64 == 0, (n, k, world)
            if mesh is not None and not isinstance(w, DTensor):
                rank = mesh.get_local_rank()
                local = w.detach()[rank * (n // world):(rank + 1) * (n // world)]
                lin.weight = torch.nn.Parameter(
                    DTensor.from_local(local, mesh, [Shard(0)], run_check=False, shape=(n, k), stride=(k, 1)))

    @staticmethod
    def eligible(linears, world: int) -> bool:
        """The kernel's layout rules: every weight has a multiple of 256 rows and of
        128 rows per rank, K a multiple of 64 shared by all, at most four weights."""
        ks = {lin.weight.shape[1] for lin in linears}
        return (
            1 <= len(linears) <= 4 and len(ks) == 1 and ks.pop() % 64 == 0
            and all(lin.weight.shape[0] % 256 == 0 and lin.weight.shape[0] % (world * CHUNK_ROWS) == 0
                    for lin in linears)
        )

    @property
    def params(self):
        return [lin.weight for lin in self.linears]

    def __call__(self, x: torch.Tensor):
        shards = [w._local_tensor if hasattr(w, "_local_tensor") else w.detach() for w in self.params]
        return _GatherLinearFn.apply(x, self, *shards)

    @staticmethod
    def _side_stream(device):
        s = GatherLinear._side.get(device)
        if s is None:
            s = GatherLinear._side[device] = torch.cuda.Stream(device)
        return s

    def _reduce_grads(self, dys, x2):
        cur = torch.cuda.current_stream(x2.device)
        side = self._side_stream(x2.device)
        side.wait_stream(cur)
        world = 1 if self.group is None else dist.get_world_size(self.group)
        with torch.cuda.stream(side):
            for t in (*dys, x2):
                t.record_stream(side)
            if world == 1:
                grads = [dy.t() @ x2 for dy in dys]
            else:
                rpr = [dy.shape[1] // world for dy in dys]
                tot = sum(rpr)
                packed = torch.empty(world, tot, x2.shape[1], dtype=x2.dtype, device=x2.device)
                for r in range(world):
                    off = 0
                    for dy, n in zip(dys, rpr):
                        torch.matmul(dy[:, r * n:(r + 1) * n].t(), x2, out=packed[r, off:off + n])
                        off += n
                red = torch.empty(tot, x2.shape[1], dtype=x2.dtype, device=x2.device)
                _reduce_scatter(self.group)(red, packed.view(world * tot, -1), self.group, dist.ReduceOp.AVG)
                grads, off = [], 0
                for n in rpr:
                    grads.append(red[off:off + n])
                    off += n
        GatherLinear._pending.append((self, grads, side))
        # one callback per call: the first to run delivers every pending gradient, the
        # rest find the list empty (a backward that raised leaves nothing queued behind)
        torch.autograd.Variable._execution_engine.queue_callback(GatherLinear._finish)

    @staticmethod
    def _finish():
        from torch.distributed.tensor import DTensor, Shard

        pending, GatherLinear._pending = GatherLinear._pending, []
        for owner, grads, side in pending:
            cur = torch.cuda.current_stream(grads[0].device)
            cur.wait_stream(side)
            for p, g in zip(owner.params, grads):
                g.record_stream(cur)  # allocated on the side stream, consumed on this one
                if isinstance(p, DTensor):
                    g = DTensor.from_local(g, owner.mesh, [Shard(0)], run_check=False, shape=p.shape,
                                           stride=p.stride())
                if p.grad is None:
                    p.grad = g
                else:
                    p.grad += g


def all_gather_linear(x: torch.Tensor, shard: torch.Tensor, group: dist.ProcessGroup | None) -> torch.Tensor:
    """Functional single-weight form: ``x @ all_gather(shard)^T`` (autograd: ``dx``
    and the reduce-scattered shard gradient, returned synchronously)."""
    return _SingleFn.apply(x, shard, group)


class _SingleFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, shard, group):
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        (y,), wg = engine_for(group, x.device)(x2, [shard])
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
