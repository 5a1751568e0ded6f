"""``Muon``: the unified Muon-family + Adam optimizer.

Public contract of the reference's ``muonium.optim.optim.Muon``
(src/muonium/optim/optim.py:81-719): constructor signature and validation
messages, per-group ``algorithm`` routing, the group keys written into
``state_dict`` (lr as a 0-dim tensor, resolved ``foreach``, algorithm
options), lazy per-parameter state (CPU ``step`` and ``lr_ratio`` scalars plus
the algorithm's ``state_spec`` buffers shaped like the transformed gradient),
legacy-default loading in ``__setstate__``, the per-parameter and batched
drivers, ``batch_size`` chunking and the CPU-offload round trip.

Execution differs: CUDA Muon batches run the fused sm_100a kernel sequence
(:mod:`dtensor_muon_b200.ops.muon_fused`) instead of a ``torch.compile``d
region, and CUDA Adam groups run the native multi-tensor AdamW kernel.
``_muon_impls`` keeps the reference's per-algorithm callable cache so an
outer tracer (or a test) can substitute the update entry point.
"""

from __future__ import annotations

import functools
import math
from typing import cast

import torch
from torch import Tensor
from torch.optim.adam import adam as torch_adam
from torch.optim.optimizer import _device_dtype_check_for_fused, _get_scalar_dtype, _use_grad_for_differentiable

from ..ops import adamw as native_adam
from ..orthogonalize import OrthogonalizationStrategy
from ..utils import group_tensors_by_shape, move_tensors_to_device
from .algorithms import BufferSpec, MuonAlgorithm, get_algorithm
from .algorithms.base import ADAM_ALGORITHMS


def _register_dtensor_foreach_ops() -> None:
    """Give DTensor a sharding strategy for ``aten._foreach_sign_`` (pointwise:
    every input keeps its own placement). Idempotent."""
    try:
        from torch.distributed.tensor._op_schema import OpSpec, OpStrategy, RuntimeSchemaInfo, TupleStrategy
        from torch.distributed.tensor._ops.utils import register_op_strategy
    except ImportError:  # pragma: no cover - private API moved
        return
    op = torch.ops.aten._foreach_sign_.default
    if getattr(op, "_dmb_dtensor_registered", False):
        return

    @register_op_strategy(op, schema_info=RuntimeSchemaInfo(needs_pytree=True))
    def _sign_strategy(op_schema):
        children = op_schema.args_schema[0].children
        return TupleStrategy(
            [OpStrategy([OpSpec(s.output_specs, (s.output_specs,)) for s in c.strategies]) for c in children]
        )

    op._dmb_dtensor_registered = True


_register_dtensor_foreach_ops()


def _group_muon_tensors(params, grads, state_lists, lr_ratios):
    """Split a group into homogeneous (device, dtype, shape) batches, keeping order."""
    # DTensors are also split by placements and stride: a batch is stacked and
    # redistributed as one tensor, so e.g. column- and row-parallel TP weights of
    # the same shape must not share a batch.
    by_dev: dict[tuple, list[int]] = {}
    for i, p in enumerate(params):
        g = grads[i]
        layout = (tuple(g.placements), tuple(g.stride())) if hasattr(g, "placements") else None
        by_dev.setdefault((p.device, p.dtype, layout), []).append(i)
    out = []
    for (device, _, _), idxs in by_dev.items():
        shapes = group_tensors_by_shape([grads[i] for i in idxs])
        for _, (_, local) in shapes.items():
            sel = [idxs[j] for j in local]
            out.append(
                (
                    device,
                    [params[i] for i in sel],
                    [grads[i] for i in sel],
                    {k: [v[i] for i in sel] for k, v in state_lists.items()},
                    [lr_ratios[i] for i in sel],
                )
            )
    return out


class Muon(torch.optim.Optimizer):
    """Unified Muon + Adam optimizer.

    Args:
        params: parameters, or param-group dicts. A group's ``"algorithm"`` is
            ``"adamw"``/``"adam"`` for the Adam path, ``"muon"`` (default) or any
            registered Muon variant (e.g. ``"normuon"``); variant options (e.g.
            ``muon_beta2``) go in the same dict. Muon groups may also set
            ``flatten`` (collapse 3-D+ tensors to one ``(dim0, -1)`` matrix
            instead of a batch of matrices) and ``split_sizes`` (2-D only:
            orthogonalise row blocks of a fused weight separately).
        lr, wd: default learning rate and weight decay.
        use_cautious_wd: apply Muon weight decay only where ``u * p > 0``.
        maximize: ascend instead of descend.
        momentum, nesterov, ns_steps, orthogonalization_strategy: Muon settings
            (``"newton_schulz"`` or ``"polar_express"``).
        amsgrad, adam_betas, adam_eps, is_adamw, fused_adam, foreach_adam: Adam settings.
        foreach: batch Muon groups by (device, dtype, shape). ``None`` enables it
            when every param is on CUDA; ``True`` on CPU params means a CUDA round
            trip per batch (CPU offload).
        batch_size: maximum tensors per batch (``None`` = unbounded).
    """

    def __init__(
        self,
        params,
        lr: float = 1e-3,
        wd: float = 0.1,
        use_cautious_wd: bool = True,
        maximize: bool = False,
        momentum: float = 0.95,
        nesterov: bool = True,
        ns_steps: int = 5,
        orthogonalization_strategy: OrthogonalizationStrategy = "polar_express",
        amsgrad: bool = False,
        adam_betas: tuple[float, float] = (0.9, 0.95),
        adam_eps: float = 1e-8,
        is_adamw: bool = True,
        fused_adam: bool | None = None,
        foreach_adam: bool | None = None,
        foreach: bool | None = None,
        batch_size: int | None = None,
    ):
        self.lr = lr
        self.wd = wd
        self.use_cautious_wd = use_cautious_wd
        self.momentum = momentum
        self.nesterov = nesterov
        self.ns_steps = ns_steps
        self.orthogonalization_strategy = orthogonalization_strategy
        self.amsgrad = amsgrad
        self.adam_betas = adam_betas
        self.adam_eps = adam_eps
        self.is_adamw = is_adamw
        self.fused_adam = fused_adam
        self.foreach_adam = foreach_adam
        self.maximize = maximize
        self.foreach = foreach
        self.batch_size = batch_size

        if not 0.0 <= lr:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= adam_eps:
            raise ValueError(f"Invalid epsilon value: {adam_eps}")
        for i, beta in enumerate(adam_betas):
            if not 0.0 <= beta < 1.0:
                raise ValueError(f"Invalid beta parameter at index {i}: {beta}")
        if isinstance(params, dict):
            raise TypeError(
                "params must be an iterable of parameters or "
                "an iterable of param-group dicts, not a single dict."
            )
        params = list(params)
        if not params:
            raise ValueError("optimizer got an empty parameter list")
        if not isinstance(params[0], dict):
            params = [{"params": params}]

        groups: list[dict] = []
        for group in params:
            algorithm = cast(str, group.get("algorithm", "muon")).lower()
            if "params" not in group:
                raise ValueError("Param group dict must have a 'params' key")
            group["params"] = list(group["params"])
            if not group["params"]:
                continue
            if algorithm in ADAM_ALGORITHMS:
                groups.append(self._build_adam_group(group))
            else:
                groups.append(self._build_muon_group(group, get_algorithm(algorithm)))

        super().__init__(groups, {"differentiable": False})
        self._init_muon_impl()

    # ------------------------------------------------------------- impl cache
    def _init_muon_impl(self) -> None:
        """Reset the per-algorithm cache of update entry points."""
        self._muon_impls: dict[str, object] = {}

    def _raw_muon_impl(self, algorithm: MuonAlgorithm):
        return functools.partial(self.muon, algorithm)

    def _get_muon_impl(self, algorithm: MuonAlgorithm):
        impl = self._muon_impls.get(algorithm.name)
        if impl is None:
            impl = self._raw_muon_impl(algorithm)
            self._muon_impls[algorithm.name] = impl
        return impl

    # ----------------------------------------------------------- group build
    @staticmethod
    def _validate_split_sizes(group: dict) -> tuple[int, ...] | None:
        split_sizes = group.get("split_sizes")
        if split_sizes is None:
            return None
        if not isinstance(split_sizes, (tuple, list)) or len(split_sizes) < 2:
            raise ValueError(
                f"split_sizes must be a tuple or list of at least 2 block sizes, got {split_sizes!r}."
            )
        if not all(isinstance(s, int) and not isinstance(s, bool) and s > 0 for s in split_sizes):
            raise ValueError(f"split_sizes entries must be positive integers, got {split_sizes!r}.")
        for p in group["params"]:
            if p.ndim != 2:
                raise ValueError(f"split_sizes is only supported for 2D parameters, got shape {tuple(p.shape)}.")
            if sum(split_sizes) != p.shape[0]:
                raise ValueError(
                    f"split_sizes {tuple(split_sizes)} must sum to dim 0 of the parameter shape {tuple(p.shape)}."
                )
        return tuple(split_sizes)

    def _build_muon_group(self, group: dict, algorithm: MuonAlgorithm) -> dict:
        for p in group["params"]:
            algorithm.validate_param(p)
        foreach = group.get("foreach", self.foreach)
        if foreach is None:
            foreach = all(p.is_cuda for p in group["params"])
        built = {
            "params": group["params"],
            "algorithm": algorithm.name,
            "use_muon": True,
            "lr": torch.tensor(group.get("lr", self.lr)),
            "wd": group.get("wd", self.wd),
            "use_cautious_wd": group.get("use_cautious_wd", self.use_cautious_wd),
            "momentum": group.get("momentum", self.momentum),
            "nesterov": group.get("nesterov", self.nesterov),
            "ns_steps": group.get("ns_steps", self.ns_steps),
            "orthogonalization_strategy": group.get("orthogonalization_strategy", self.orthogonalization_strategy),
            "maximize": group.get("maximize", self.maximize),
            "flatten": group.get("flatten", False),
            "split_sizes": self._validate_split_sizes(group),
            "foreach": foreach,
        }
        for key, default in algorithm.options.items():
            built[key] = group.get(key, default)
        return built

    def _build_adam_group(self, group: dict) -> dict:
        algorithm = cast(str, group.get("algorithm", "adamw")).lower()
        return {
            "params": group["params"],
            "algorithm": algorithm,
            "use_muon": False,
            "lr": group.get("lr", self.lr),
            "wd": group.get("wd", self.wd),
            "amsgrad": group.get("amsgrad", self.amsgrad),
            "betas": group.get("betas", self.adam_betas),
            "eps": group.get("eps", self.adam_eps),
            "decoupled_weight_decay": group.get("decoupled_weight_decay", self.is_adamw and algorithm == "adamw"),
            "fused": group.get("fused", self.fused_adam),
            "foreach": group.get("foreach", self.foreach_adam),
            "maximize": group.get("maximize", self.maximize),
            "has_complex": any(torch.is_complex(p) for p in group["params"]),
        }

    # ------------------------------------------------------------ checkpoint
    def __setstate__(self, state):
        super().__setstate__(state)
        for group in self.param_groups:
            if group["use_muon"]:
                group.setdefault("algorithm", "muon")
                algorithm = get_algorithm(group["algorithm"])
                group.setdefault("ns_steps", 5)
                group.setdefault("nesterov", True)
                group.setdefault("flatten", False)
                group.setdefault("use_cautious_wd", True)
                group.setdefault("orthogonalization_strategy", "polar_express")
                group.setdefault("split_sizes", None)
                if "foreach" not in group:
                    group["foreach"] = all(p.is_cuda for p in group["params"])
                for key, default in algorithm.options.items():
                    group.setdefault(key, default)
                if not torch.is_tensor(group["lr"]):
                    group["lr"] = torch.tensor(float(group["lr"]))
                for p in group["params"]:
                    st = self.state.get(p, {})
                    if st and not torch.is_tensor(st["step"]):
                        st["step"] = torch.tensor(float(st["step"]))
            else:
                group.setdefault("amsgrad", False)
                group.setdefault("maximize", False)
                group.setdefault("foreach", None)
                group.setdefault("decoupled_weight_decay", False)
                if torch.is_tensor(group["wd"]):
                    group["wd"] = float(group["wd"])
                fused = group.setdefault("fused", None)
                for p in group["params"]:
                    st = self.state.get(p, {})
                    if st and not torch.is_tensor(st["step"]):
                        val = float(st["step"])
                        st["step"] = (
                            torch.tensor(val, dtype=_get_scalar_dtype(is_fused=fused), device=p.device)
                            if fused
                            else torch.tensor(val, dtype=_get_scalar_dtype())
                        )
        self._init_muon_impl()

    # ------------------------------------------------------------ state init
    def _new_state_buffer(self, p: Tensor, grad: Tensor, spec: BufferSpec) -> Tensor:
        """Allocate one ``state_spec`` buffer (fp32). Low-precision subclasses override."""
        like = grad if spec.like == "grad" else grad[..., :1]
        return torch.zeros_like(like, dtype=torch.float32, memory_format=torch.preserve_format)

    @staticmethod
    def _transform_grad(grad: Tensor, flatten: bool) -> Tensor:
        if grad.ndim > 2:
            if flatten:
                return grad.view(grad.size(0), -1)
            if grad.ndim > 3:
                return grad.flatten(end_dim=-3)
        return grad

    def _init_muon_group(self, group, algorithm, params_with_grad, grads, state_lists, lr_ratios, state_steps):
        for p in group["params"]:
            if p.grad is None:
                continue
            assert not p.grad.is_sparse, "Muon does not support sparse gradients"
            params_with_grad.append(p)
            grad = self._transform_grad(p.grad, group["flatten"])
            grads.append(grad)
            state = self.state[p]
            if len(state) == 0:
                state["step"] = torch.tensor(0.0, dtype=_get_scalar_dtype())
                for key, spec in algorithm.state_spec.items():
                    state[key] = self._new_state_buffer(p, grad, spec)
                state["lr_ratio"] = torch.tensor(math.sqrt(max(1.0, grad.shape[-2] / grad.shape[-1])))
            state["step"] += 1
            for key in algorithm.state_spec:
                state_lists[key].append(state[key])
            lr_ratios.append(state["lr_ratio"])
            state_steps.append(state["step"])

    def _init_adam_group(
        self, group, params_with_grad, grads, exp_avgs, exp_avg_sqs, max_exp_avg_sqs, state_steps, capturable
    ):
        for p in group["params"]:
            if p.grad is None:
                continue
            assert not p.grad.is_sparse, "Adam does not support sparse gradients, please consider SparseAdam instead"
            params_with_grad.append(p)
            grads.append(p.grad)
            state = self.state[p]
            if len(state) == 0:
                if group["fused"]:
                    _device_dtype_check_for_fused(p)
                state["step"] = (
                    torch.zeros((), dtype=_get_scalar_dtype(is_fused=group["fused"]), device=p.device)
                    if capturable or group["fused"]
                    else torch.tensor(0.0, dtype=_get_scalar_dtype())
                )
                state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                if group["amsgrad"]:
                    state["max_exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            elif capturable and state["step"].device != p.device:
                state["step"] = state["step"].to(p.device)
            exp_avgs.append(state["exp_avg"])
            exp_avg_sqs.append(state["exp_avg_sq"])
            if group["amsgrad"]:
                max_exp_avg_sqs.append(state["max_exp_avg_sq"])
            state_steps.append(state["step"])

    # ---------------------------------------------------------------- driver
    def muon(
        self,
        algorithm: MuonAlgorithm,
        params: list[Tensor],
        grads: list[Tensor],
        state: dict[str, list[Tensor]],
        lr_ratios: list[Tensor],
        *,
        foreach: bool = False,
        nesterov: bool,
        lr: Tensor,
        weight_decay: float,
        cautious_wd: bool,
        momentum: float,
        ns_steps: int,
        orthogonalization_strategy: OrthogonalizationStrategy,
        maximize: bool,
        split_sizes: tuple[int, ...] | None = None,
        **opts,
    ) -> None:
        """Muon-family update of a list of parameters.

        ``foreach=False``: ``algorithm.update`` per tensor. ``foreach=True``:
        homogeneous batches (chunked by ``batch_size``) through
        ``algorithm.foreach_update``, with a CUDA round trip for CPU tensors.
        """
        if not params:
            return
        kw = dict(
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
        if not foreach and self._per_param_can_batch(algorithm, params, state):
            # The built-in algorithms' per-parameter update is the fp32 math of the
            # fused kernels, so same-shape CUDA parameters are stepped as one batch
            # (identical arithmetic, better GPU occupancy).
            foreach = True
        if not foreach:
            for i, (p, g, r) in enumerate(zip(params, grads, lr_ratios, strict=True)):
                algorithm.update(p, g, {k: v[i] for k, v in state.items()}, r, **kw)
            return

        for device, dp, dg, dstate, dlr in _group_muon_tensors(params, grads, state, lr_ratios):
            idx = list(range(len(dg)))
            bs = self.batch_size
            batches = [idx[i : i + bs] for i in range(0, len(idx), bs)] if bs and len(idx) > bs else [idx]
            cuda = torch.device("cuda")
            for sel in batches:
                p_orig = [dp[i] for i in sel]
                g_orig = [dg[i] for i in sel]
                s_orig = {k: [v[i] for i in sel] for k, v in dstate.items()}
                r_orig = [dlr[i] for i in sel]
                p_b = move_tensors_to_device(p_orig, device, cuda)
                g_b = move_tensors_to_device(g_orig, device, cuda)
                s_b = {k: move_tensors_to_device(v, device, cuda) for k, v in s_orig.items()}
                r_b = move_tensors_to_device(r_orig, device, cuda)
                algorithm.foreach_update(p_b, g_b, s_b, r_b, **kw)
                pairs = [(p_orig, p_b), (g_orig, g_b), (r_orig, r_b)] + [(s_orig[k], s_b[k]) for k in s_orig]
                for originals, moved in pairs:
                    if originals is moved:
                        continue
                    for o, m in zip(originals, moved, strict=True):
                        if o is not None and m is not None:
                            o.copy_(m.to(o.device))

    @staticmethod
    def _per_param_can_batch(algorithm, params, state) -> bool:
        from .algorithms import MuonBaseline, NorMuon
        from .algorithms import base as _base

        if type(algorithm) not in (MuonBaseline, NorMuon) or not _base._seams_are_builtin():
            return False
        tensors = list(params) + [t for ts in state.values() for t in ts]
        return all(isinstance(t, Tensor) and t.is_cuda and not hasattr(t, "device_mesh") for t in tensors)

    def _step_muon_group(self, group: dict) -> None:
        algorithm = get_algorithm(group.get("algorithm", "muon"))
        params, grads, steps, lr_ratios = [], [], [], []
        state_lists: dict[str, list[Tensor]] = {k: [] for k in algorithm.state_spec}
        self._init_muon_group(group, algorithm, params, grads, state_lists, lr_ratios, steps)
        impl = self._raw_muon_impl(algorithm) if torch.compiler.is_compiling() else self._get_muon_impl(algorithm)
        from ..parallel.owner_compute import deferred

        with deferred():  # owner-compute batches of this group run phase by phase at exit
            self._call_impl(impl, group, algorithm, params, grads, state_lists, lr_ratios)

    def _call_impl(self, impl, group, algorithm, params, grads, state_lists, lr_ratios) -> None:
        impl(
            params,
            grads,
            state_lists,
            lr_ratios,
            foreach=group["foreach"],
            nesterov=group["nesterov"],
            lr=group["lr"],
            weight_decay=group["wd"],
            cautious_wd=group["use_cautious_wd"],
            momentum=group["momentum"],
            ns_steps=group["ns_steps"],
            orthogonalization_strategy=group["orthogonalization_strategy"],
            maximize=group["maximize"],
            split_sizes=group["split_sizes"],
            **{k: group[k] for k in algorithm.options},
        )

    def _step_adam_group(self, group: dict) -> None:
        params, grads, steps, m1, m2, mx = [], [], [], [], [], []
        beta1, beta2 = group["betas"]
        capturable = torch.compiler.is_compiling()
        self._init_adam_group(group, params, grads, m1, m2, mx, steps, capturable)
        if not params:
            return
        lr = group["lr"]
        wd = group["wd"]
        # Adam is elementwise: DTensors that share placements update through their local shards.
        if all(hasattr(t, "to_local") for t in params + grads + m1 + m2 + mx):
            places = {tuple(t.placements) for t in params + grads + m1 + m2 + mx}
            if len(places) == 1:
                params, grads = [t.to_local() for t in params], [t.to_local() for t in grads]
                m1, m2, mx = [t.to_local() for t in m1], [t.to_local() for t in m2], [t.to_local() for t in mx]
        grad_scale = getattr(self, "grad_scale", None)
        found_inf = getattr(self, "found_inf", None)
        use_native = (
            not capturable
            and grad_scale is None
            and found_inf is None
            and not group["has_complex"]
            and all(not s.is_cuda for s in steps)
            and native_adam.native_eligible(params, grads, m1, m2, mx, group["amsgrad"])
        )
        if use_native:
            native_adam.fused_adam(
                params,
                grads,
                m1,
                m2,
                mx,
                steps,
                amsgrad=group["amsgrad"],
                beta1=beta1,
                beta2=beta2,
                lr=float(lr),
                weight_decay=float(wd),
                eps=group["eps"],
                maximize=group["maximize"],
                decoupled_weight_decay=group["decoupled_weight_decay"],
            )
            return
        if not group["fused"] and not capturable:
            lr = float(lr) if torch.is_tensor(lr) else lr
            wd = float(wd) if torch.is_tensor(wd) else wd
        torch_adam(
            params,
            grads,
            m1,
            m2,
            mx,
            steps,
            amsgrad=group["amsgrad"],
            has_complex=group["has_complex"],
            beta1=beta1,
            beta2=beta2,
            lr=lr,
            weight_decay=wd,
            eps=group["eps"],
            maximize=group["maximize"],
            capturable=capturable,
            differentiable=False,
            fused=group["fused"],
            foreach=group["foreach"],
            grad_scale=grad_scale,
            found_inf=found_inf,
            decoupled_weight_decay=group["decoupled_weight_decay"],
        )

    @_use_grad_for_differentiable
    def step(self, closure=None):
        """One optimization step: Muon-family groups through their registered
        algorithm, the rest through Adam/AdamW."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            if group["use_muon"]:
                self._step_muon_group(group)
            else:
                self._step_adam_group(group)
        return loss
