"""Algorithm registry, state specs and the shared orthogonalisation helpers.

Public contract of the reference's ``muonium.optim.algorithms.base``
(src/muonium/optim/algorithms/base.py:1-310): algorithms own the update math;
the optimizer owns everything around it (group building, state allocation
from ``state_spec``, batching, offload, quantised state). The module-level
names ``zeropower`` / ``foreach_zeropower`` are the seam through which every
algorithm orthogonalises, so tests (and users) can substitute them.
"""

from __future__ import annotations

import math
from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Any, ClassVar, Literal

import torch
from torch import Tensor
from torch.distributed.tensor import DTensor, Replicate

from ...orthogonalize import (
    OrthogonalizationStrategy,
    foreach_zeropower,
    foreach_zeropower_3d_fsdp,
    is_fsdp_3d_sharded,
    zeropower,
)
from ...orthogonalize import orthogonalize as _ortho_module

# Keys the optimizer owns; algorithm options may not reuse them.
RESERVED_GROUP_KEYS = frozenset(
    {
        "params",
        "algorithm",
        "use_muon",
        "lr",
        "wd",
        "use_cautious_wd",
        "momentum",
        "nesterov",
        "ns_steps",
        "orthogonalization_strategy",
        "maximize",
        "flatten",
        "foreach",
        "split_sizes",
    }
)

# Names that select the Adam path in the optimizer and can never be registered.
ADAM_ALGORITHMS = ("adam", "adamw")


@dataclass(frozen=True)
class BufferSpec:
    """Declares one per-parameter state buffer.

    ``like="grad"``: fp32, shaped like the (possibly flattened) gradient.
    ``like="grad_rows"``: fp32, shaped like ``grad[..., :1]`` (one value per row).
    ``signed`` tells quantised-state optimizers whether negative values occur.
    """

    like: Literal["grad", "grad_rows"]
    signed: bool = True


def split_lr_scales(shape, split_sizes: tuple[int, ...]) -> tuple[float, ...]:
    """Per-block LR corrections for a fused 2-D weight split into row blocks.

    The whole update is later scaled by ``sqrt(max(1, rows/cols))`` of the full
    matrix; each block should instead get its own ratio, so it is pre-scaled
    by ``ratio(block) / ratio(full)``.
    """
    rows, cols = shape[-2], shape[-1]
    full = math.sqrt(max(1.0, rows / cols))
    return tuple(math.sqrt(max(1.0, h / cols)) / full for h in split_sizes)


def _orthogonalize_row_blocks(
    mats: list[Tensor],
    split_sizes: tuple[int, ...],
    *,
    ns_steps: int,
    strategy: OrthogonalizationStrategy,
) -> list[Tensor]:
    """Orthogonalise the row blocks of every (plain, same-shape) matrix of a batch.

    Blocks are collected across the WHOLE batch and grouped by height, so a batch
    of B fused QKV weights under GQA costs two engine calls (B query blocks, 2B
    key/value blocks) rather than 2B. Each result block is scaled by its
    :func:`split_lr_scales` factor and written in place into one preallocated
    bf16 output per matrix (no concatenation). Same semantics as the reference's
    per-tensor split (src/muonium/optim/algorithms/base.py:73-99).
    """
    if not mats:
        return []
    scales = split_lr_scales(mats[0].shape, split_sizes)
    starts = [0]
    for h in split_sizes[:-1]:
        starts.append(starts[-1] + h)
    outs = [torch.empty(m.shape, dtype=torch.bfloat16, device=m.device) for m in mats]
    for height in sorted(set(split_sizes)):
        jobs = [(k, starts[j], scales[j]) for k in range(len(mats)) for j, h in enumerate(split_sizes) if h == height]
        us = foreach_zeropower([mats[k].narrow(-2, r0, height) for k, r0, _ in jobs], steps=ns_steps, strategy=strategy)
        for (k, r0, sc), u in zip(jobs, us, strict=True):
            outs[k].narrow(-2, r0, height).copy_(u * sc)
    return outs


def _gather_batch(gs: list[DTensor]) -> list[Tensor]:
    """Full (replicated) local copies of a batch of DTensors with common metadata:
    one stacked gather for the batch instead of one per tensor."""
    try:
        stacked = torch.stack(list(gs), dim=0)
        return list(stacked.full_tensor().unbind(0))
    except (RuntimeError, NotImplementedError):  # placements the stacked form cannot express
        return [g.full_tensor() for g in gs]


def _reshard_like(u: Tensor, like: DTensor) -> DTensor:
    """Hand a replicated result back with ``like``'s placements; Replicate -> Shard
    is a local slice on every rank, so no collective runs."""
    mesh = like.device_mesh
    rep = DTensor.from_local(u, device_mesh=mesh, placements=(Replicate(),) * mesh.ndim, run_check=False)
    return rep.redistribute(placements=like.placements)


def _seams_are_builtin() -> bool:
    """True while ``zeropower`` / ``foreach_zeropower`` of this module are the
    library's own functions (the fused kernel path computes the same thing)."""
    mod = globals()
    return mod["zeropower"] is _ortho_module.zeropower and mod["foreach_zeropower"] is _ortho_module.foreach_zeropower


def orthogonalize_single(
    g: Tensor,
    *,
    ns_steps: int,
    strategy: OrthogonalizationStrategy,
    split_sizes: tuple[int, ...] | None = None,
) -> Tensor:
    """Orthogonalise one tensor: a batch of one (DTensor handling lives in
    ``zeropower`` and :func:`orthogonalize_batch`). With ``split_sizes`` each row
    block is orthogonalised on its own and rescaled (:func:`split_lr_scales`)."""
    if split_sizes is None:
        return zeropower(g, steps=ns_steps, strategy=strategy)
    return orthogonalize_batch([g], ns_steps=ns_steps, strategy=strategy, split_sizes=split_sizes)[0]


def orthogonalize_batch(
    gs: list[Tensor],
    *,
    ns_steps: int,
    strategy: OrthogonalizationStrategy,
    split_sizes: tuple[int, ...] | None = None,
) -> list[Tensor]:
    """Orthogonalise a same-shape batch; the only place algorithms meet distribution.

    * ``split_sizes``: every row block of every matrix goes through
      :func:`_orthogonalize_row_blocks` (one engine call per block height). A
      DTensor batch is gathered once as a stack and its results are sliced back
      to each rank's shard locally, so any placement works.
    * 3-D stacks sharded only on dim 0 (FSDP / EP experts): local, collective-free.
    * everything else: the batched ``foreach_zeropower``.

    Reference behaviour: src/muonium/optim/algorithms/base.py:134-168.
    """
    if not gs:
        return []
    if split_sizes is not None:
        if isinstance(gs[0], DTensor):
            us = _orthogonalize_row_blocks(_gather_batch(gs), split_sizes, ns_steps=ns_steps, strategy=strategy)
            return [_reshard_like(u, g) for u, g in zip(us, gs, strict=True)]
        return _orthogonalize_row_blocks(list(gs), split_sizes, ns_steps=ns_steps, strategy=strategy)
    if is_fsdp_3d_sharded(gs):
        return foreach_zeropower_3d_fsdp(gs, steps=ns_steps, strategy=strategy)
    return foreach_zeropower(gs, steps=ns_steps, strategy=strategy)


class MuonAlgorithm(ABC):
    """A Muon-family update rule, selected per param group by ``"algorithm"``.

    Subclasses define ``name``, optionally ``options`` (per-group
    hyperparameters with defaults) and ``state_spec`` (extra per-parameter
    buffers), and implement :meth:`update`. Register with
    :func:`register_muon_algorithm`.
    """

    name: ClassVar[str]
    options: ClassVar[dict[str, Any]] = {}
    state_spec: ClassVar[dict[str, BufferSpec]] = {"momentum_buffer": BufferSpec(like="grad", signed=True)}

    def validate_param(self, p: Tensor) -> None:
        """Reject parameters the algorithm cannot update (called when groups are built)."""
        if p.ndim < 2:
            raise ValueError("Muon only supports 2D+ parameters; found a 1D tensor in a Muon group")
        if torch.is_complex(p):
            raise NotImplementedError(
                "Complex parameters are not supported in Muon. Add these parameters "
                "to the Adam group or use a different optimizer."
            )

    @abstractmethod
    def update(
        self,
        param: Tensor,
        grad: Tensor,
        state: dict[str, Tensor],
        lr_ratio: Tensor,
        *,
        lr: Tensor,
        weight_decay: float,
        cautious_wd: bool,
        momentum: float,
        nesterov: bool,
        maximize: bool,
        ns_steps: int,
        orthogonalization_strategy: OrthogonalizationStrategy,
        split_sizes: tuple[int, ...] | None,
        **opts,
    ) -> None:
        """Per-tensor fp32 update; mutates ``param`` and ``state`` in place."""

    def foreach_update(
        self,
        params: list[Tensor],
        grads: list[Tensor],
        state: dict[str, list[Tensor]],
        lr_ratios: list[Tensor],
        *,
        lr: Tensor,
        weight_decay: float,
        cautious_wd: bool,
        momentum: float,
        nesterov: bool,
        maximize: bool,
        ns_steps: int,
        orthogonalization_strategy: OrthogonalizationStrategy,
        split_sizes: tuple[int, ...] | None,
        **opts,
    ) -> None:
        """Batched update over same-(device, dtype, shape) tensors; defaults to a
        loop over :meth:`update`."""
        for i, (p, g, r) in enumerate(zip(params, grads, lr_ratios, strict=True)):
            self.update(
                p,
                g,
                {k: v[i] for k, v in state.items()},
                r,
                lr=lr,
                weight_decay=weight_decay,
                cautious_wd=cautious_wd,
                momentum=momentum,
                nesterov=nesterov,
                maximize=maximize,
                ns_steps=ns_steps,
                orthogonalization_strategy=orthogonalization_strategy,
                split_sizes=split_sizes,
                **opts,
            )


_REGISTRY: dict[str, MuonAlgorithm] = {}


def register_muon_algorithm(cls: type[MuonAlgorithm]) -> type[MuonAlgorithm]:
    """Register ``cls`` under ``cls.name`` (case-insensitive); usable as a decorator.

    Re-registering the same class (same ``__qualname__``) replaces the
    instance; a different class under an existing name is an error.
    """
    name = getattr(cls, "name", None)
    if not isinstance(name, str) or not name:
        raise ValueError(f"{cls.__qualname__} must define a non-empty string `name`")
    key = name.lower()
    if key in ADAM_ALGORITHMS:
        raise ValueError(f"'{key}' is reserved for the Adam path")
    existing = _REGISTRY.get(key)
    if existing is not None and type(existing).__qualname__ != cls.__qualname__:
        raise ValueError(f"Muon algorithm '{key}' is already registered")
    clash = sorted(RESERVED_GROUP_KEYS.intersection(cls.options))
    if clash:
        raise ValueError(f"{cls.__qualname__}.options shadow reserved group keys: {clash}")
    _REGISTRY[key] = cls()
    return cls


def get_algorithm(name: str) -> MuonAlgorithm:
    """The registered algorithm instance for ``name`` (case-insensitive)."""
    try:
        return _REGISTRY[name.lower()]
    except KeyError:
        raise ValueError(
            f"Unknown algorithm '{name}'. Registered Muon algorithms: "
            f"{sorted(_REGISTRY)}; 'adam' and 'adamw' select the Adam path."
        ) from None


def registered_algorithms() -> tuple[str, ...]:
    """Sorted names of every registered Muon algorithm (Adam names excluded)."""
    return tuple(sorted(_REGISTRY))
