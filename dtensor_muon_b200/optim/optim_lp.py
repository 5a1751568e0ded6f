"""``MuonLP``: Muon with block-quantised momentum state.

API of the reference's ``muonium.optim.optim_lp`` (src/muonium/optim/optim_lp.py:21-133):
``MuonLP(..., foreach=False, block_size=2048, bf16_stochastic_round=False)``
plus ``Muon8bit`` / ``Muon4bit`` / ``MuonFp8``. Only ``like="grad"`` buffers
(the momentum) are quantised, and only when the local tensor has at least 4096
elements and a multiple of ``block_size``; row-shaped buffers stay fp32. The
base ``MuonLP`` stores plain fp32 buffers.

The reference builds these buffers from torchao subclasses but cannot step
them. Here the state is a :class:`QuantizedState` (codes + one fp32 scale per
block + the code map) and a step is: dequantise, momentum update in fp32,
requantise per block. On CUDA with a built-in algorithm that is one fused
kernel per tensor (``lp_momentum_step``) feeding the orthogonalisation
workspace; every other case dequantises into an fp32 temporary, runs the
algorithm's normal update and requantises.
"""

from __future__ import annotations

import math

import torch
import torch.utils._pytree as pytree
from torch import Tensor
from torch.distributed.tensor import DTensor

from ..ops import _ext, muon_fused
from ..orthogonalize import OrthogonalizationStrategy
from ..utils import to_local
from .algorithms import BufferSpec, MuonAlgorithm
from .algorithms import base as algo_base
from .algorithms.muon import MuonBaseline, lr_effs
from .algorithms.normuon import NorMuon
from .optim import Muon

FMT_FP8, FMT_8BIT, FMT_4BIT = 0, 1, 2
_FMT_BITS = {FMT_8BIT: 8, FMT_4BIT: 4}


def _tree_mag(V: int, j: int) -> float:
    """Ascending magnitude ``j`` of a ``V``-bit dynamic-tree map, built with
    correctly rounded float32 operations in a fixed order (the CUDA kernels
    evaluate the same expression, so device and table agree bit for bit)."""
    import numpy as np

    f32 = np.float32
    lg = (j + 1).bit_length() - 1
    nk, k = 1 << lg, V - 1 - lg
    p = f32(1.0)
    for _ in range(k):
        p = f32(p * f32(0.1))
    f = f32(f32(0.1) + f32(f32(f32(0.9) * f32(j + 2 - nk)) / f32(nk)))
    return float(f32(f * p))


def dynamic_tree_map(total_bits: int, signed: bool = True) -> Tensor:
    """Sorted code map of dynamic tree quantisation (Dettmers, arXiv:1511.04561).

    After an optional sign bit, ``k`` leading zero bits select the decade
    ``10**-k`` and the bits after the first one-bit split ``(0.1, 1]`` of that
    decade into equal steps (right edges, so 1.0 itself is a code). Zero is a
    code; a signed map is padded with a second zero to ``2**total_bits`` entries.
    Values are float32 results of one fixed expression (:func:`_tree_mag`).
    """
    value_bits = total_bits - (1 if signed else 0)
    mags = [_tree_mag(value_bits, j) for j in range(2**value_bits - 1)]
    vals = [0.0] + mags + ([-m for m in mags] if signed else [])
    while len(vals) < 2**total_bits:
        vals.append(0.0)
    return torch.tensor(sorted(vals), dtype=torch.float32)


_QMAPS: dict[tuple, Tensor] = {}


def qmap_for(fmt: int, signed: bool, device: torch.device) -> Tensor:
    if fmt == FMT_FP8:
        key = (fmt, True, str(device))
        if key not in _QMAPS:
            _QMAPS[key] = torch.zeros(1, dtype=torch.float32, device=device)
        return _QMAPS[key]
    key = (fmt, signed, str(device))
    if key not in _QMAPS:
        _QMAPS[key] = dynamic_tree_map(_FMT_BITS[fmt], signed).to(device)
    return _QMAPS[key]


def _nearest_codes(x: Tensor, qmap: Tensor) -> Tensor:
    """Index of the nearest map entry (ties to the lower index), CPU path."""
    hi = torch.searchsorted(qmap, x.contiguous(), right=True).clamp(1, qmap.numel() - 1)
    lo = hi - 1
    pick_hi = (qmap[hi] - x).abs() < (x - qmap[lo]).abs()
    return torch.where(pick_hi, hi, lo).to(torch.uint8)


_aten = torch.ops.aten


class QuantizedState(torch.Tensor):
    """Block-quantised fp32 tensor: ``codes`` (uint8), ``scale`` (fp32, one per
    block), the code map ``qmap``, ``fmt`` (0 fp8 e4m3, 1 8-bit map, 2 4-bit
    map), ``block_size``, ``signed`` and the logical ``shape``.

    It is a ``torch.Tensor`` wrapper subclass with the logical shape and dtype
    float32, so it can be the local tensor of a DTensor: a quantised momentum of
    a sharded parameter keeps that parameter's mesh and placements (the
    reference does the same with torchao subclasses,
    src/muonium/optim/optim_lp.py:92-101). Semantics of tensor operations:

    * ``detach`` / ``alias`` / same-shape ``view``: a QuantizedState sharing
      the same codes and scales;
    * ``copy_`` into it: requantise the source (a QuantizedState source with
      the same format and block size is copied code for code, losslessly);
    * ``to`` / ``cpu`` / ``cuda`` (``_to_copy``): move codes and scales; the
      requested dtype is ignored because the state is logically fp32 (this
      keeps it quantised through ``Optimizer.load_state_dict``'s cast);
    * every other operation sees the dequantised fp32 values and returns
      plain tensors (so ``narrow``, arithmetic and checkpoint readers work).
    """

    codes: Tensor
    scale: Tensor
    qmap: Tensor

    @staticmethod
    def __new__(cls, codes: Tensor, scale: Tensor, qmap: Tensor, fmt: int, block_size: int, signed: bool, shape):
        return torch.Tensor._make_wrapper_subclass(
            cls, torch.Size(shape), dtype=torch.float32, device=codes.device, requires_grad=False
        )

    def __init__(self, codes: Tensor, scale: Tensor, qmap: Tensor, fmt: int, block_size: int, signed: bool, shape):
        self.codes = codes
        self.scale = scale
        self.qmap = qmap
        self.fmt = int(fmt)
        self.block_size = int(block_size)
        self.signed = bool(signed)

    # -- subclass protocol -------------------------------------------------
    def __tensor_flatten__(self):
        return ["codes", "scale", "qmap"], (self.fmt, self.block_size, self.signed, tuple(self.shape))

    @staticmethod
    def __tensor_unflatten__(inner, meta, outer_size, outer_stride):
        fmt, block_size, signed, shape = meta
        return QuantizedState(inner["codes"], inner["scale"], inner["qmap"], fmt, block_size, signed, shape)

    __torch_function__ = torch._C._disabled_torch_function_impl

    def _alias(self, shape=None) -> "QuantizedState":
        return QuantizedState(self.codes, self.scale, self.qmap, self.fmt, self.block_size, self.signed,
                              self.shape if shape is None else shape)

    def _moved(self, device) -> "QuantizedState":
        return QuantizedState(self.codes.to(device), self.scale.to(device), self.qmap.to(device), self.fmt,
                              self.block_size, self.signed, self.shape)

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func in (_aten.detach.default, _aten.alias.default):
            return args[0]._alias()
        if func in (_aten.view.default, _aten._unsafe_view.default, _aten.reshape.default):
            src, shape = args[0], args[1]
            if isinstance(src, QuantizedState) and src.numel() == math.prod(shape) and -1 not in shape:
                return src._alias(shape)
        if func is _aten.copy_.default and isinstance(args[0], QuantizedState):
            return args[0]._assign(args[1])
        if func is _aten._to_copy.default and isinstance(args[0], QuantizedState):
            dev = kwargs.get("device")
            return args[0]._moved(dev if dev is not None else args[0].device)
        if func is _aten.is_pinned.default:
            return args[0].codes.is_pinned()

        def plain(x):
            return x.dequantize() if isinstance(x, QuantizedState) else x

        return func(*pytree.tree_map(plain, args), **pytree.tree_map(plain, kwargs))

    # -- construction ------------------------------------------------------
    @classmethod
    def zeros(cls, shape, fmt: int, block_size: int, signed: bool, device) -> "QuantizedState":
        n = math.prod(int(s) for s in shape)
        nbytes = (n + 1) // 2 if fmt == FMT_4BIT else n
        qmap = qmap_for(fmt, signed, torch.device(device))
        zero_code = 0
        if fmt != FMT_FP8:
            zero_code = int(torch.nonzero(qmap.cpu() == 0)[0])
        codes = torch.full((nbytes,), zero_code | (zero_code << 4) if fmt == FMT_4BIT else zero_code,
                           dtype=torch.uint8, device=device)
        scale = torch.zeros((n + block_size - 1) // block_size, dtype=torch.float32, device=device)
        return cls(codes, scale, qmap, fmt, block_size, signed, shape)

    def dequantize(self) -> Tensor:
        """The fp32 values (a plain tensor of this state's shape)."""
        n = self.numel()
        if self.codes.is_cuda:
            out = _ext.load().lp_dequantize(self.codes, self.scale, self.qmap, self.fmt, self.block_size, n)
            return out.view(self.shape)
        scale = self.scale.repeat_interleave(self.block_size)[:n]
        if self.fmt == FMT_FP8:
            vals = self.codes.view(torch.float8_e4m3fn).float()
        elif self.fmt == FMT_8BIT:
            vals = self.qmap[self.codes.long()]
        else:
            lo = (self.codes & 15).long()
            hi = (self.codes >> 4).long()
            vals = self.qmap[torch.stack([lo, hi], dim=1).reshape(-1)[:n]]
        return (vals * scale).view(self.shape)

    def _assign(self, src) -> "QuantizedState":
        if isinstance(src, QuantizedState) and (src.fmt, src.block_size, src.signed, src.numel()) == (
            self.fmt, self.block_size, self.signed, self.numel()
        ):
            self.codes.copy_(src.codes)
            self.scale.copy_(src.scale)
            return self
        if isinstance(src, QuantizedState):
            src = src.dequantize()
        return self._requantize(src)

    def copy_(self, src, non_blocking: bool = False) -> "QuantizedState":
        """Requantise from ``src`` (fp32 values of this state's shape)."""
        return self._assign(src)

    def _requantize(self, src: Tensor) -> "QuantizedState":
        x = src.detach().to(self.codes.device, torch.float32).contiguous().view(-1)
        if self.codes.is_cuda:
            _ext.load().lp_quantize(x, self.codes, self.scale, self.qmap, self.fmt, self.block_size)
            return self
        n = x.numel()
        nb = self.scale.numel()
        padded = torch.zeros(nb * self.block_size, dtype=torch.float32)
        padded[:n] = x
        blocks = padded.view(nb, self.block_size)
        amax = blocks.abs().amax(dim=1)
        s = amax / 448.0 if self.fmt == FMT_FP8 else amax
        inv = torch.where(s > 0, 1.0 / s, torch.zeros_like(s))
        y = (blocks * inv[:, None]).view(-1)[:n]
        self.scale.copy_(s)
        if self.fmt == FMT_FP8:
            self.codes.copy_(y.to(torch.float8_e4m3fn).view(torch.uint8))
        else:
            codes = _nearest_codes(y, self.qmap)
            if self.fmt == FMT_4BIT:
                if n % 2:
                    codes = torch.cat([codes, codes.new_zeros(1)])
                pairs = codes.view(-1, 2)
                codes = pairs[:, 0] | (pairs[:, 1] << 4)
            self.codes.copy_(codes)
        return self

    def __repr__(self, *, tensor_contents=None) -> str:
        return f"QuantizedState(shape={tuple(self.shape)}, fmt={self.fmt}, block_size={self.block_size})"


def local_quantized(x) -> "QuantizedState | None":
    """The QuantizedState behind ``x`` (itself, or a DTensor's local tensor), else None."""
    if isinstance(x, QuantizedState):
        return x
    if isinstance(x, DTensor) and isinstance(x._local_tensor, QuantizedState):
        return x._local_tensor
    return None


try:  # allow torch.load(weights_only=True) of MuonLP checkpoints
    torch.serialization.add_safe_globals([QuantizedState, torch.Size])
except AttributeError:  # pragma: no cover
    pass


class MuonLP(Muon):
    """Low-precision Muon: momentum buffers stored block-quantised."""

    #: quantisation format of the subclass; None keeps fp32 buffers
    _fmt: int | None = None
    #: tensors dequantised at once on the generic path (bounds the fp32 temporaries)
    _LP_CHUNK = 8

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
        foreach_adam: bool | None = None,
        fused_adam: bool | None = None,
        foreach: bool | None = False,
        batch_size: int | None = None,
        block_size: int = 2048,
        bf16_stochastic_round: bool = False,
    ):
        super().__init__(
            params=params,
            lr=lr,
            wd=wd,
            use_cautious_wd=use_cautious_wd,
            maximize=maximize,
            momentum=momentum,
            nesterov=nesterov,
            ns_steps=ns_steps,
            orthogonalization_strategy=orthogonalization_strategy,
            amsgrad=amsgrad,
            adam_betas=adam_betas,
            adam_eps=adam_eps,
            is_adamw=is_adamw,
            fused_adam=fused_adam,
            foreach_adam=foreach_adam,
            foreach=foreach,
            batch_size=batch_size,
        )
        self.block_size = block_size
        # Kept for API compatibility; the updates write fp32/bf16 params with
        # round-to-nearest.
        self.bf16_stochastic_round = bf16_stochastic_round

    @classmethod
    def _subclass_zeros(cls, p: Tensor, signed: bool, block_size: int):
        """Quantised zeros for ``p``'s shape, or plain fp32 zeros in the base class."""
        if cls._fmt is None:
            return torch.zeros_like(p, dtype=torch.float32)
        return QuantizedState.zeros(p.shape, cls._fmt, block_size, signed, p.device)

    def _new_buffer(self, p: Tensor, signed: bool):
        local = to_local(p)
        if local.numel() >= 4096 and local.numel() % self.block_size == 0:
            return self._subclass_zeros(local, signed, self.block_size)
        return torch.zeros_like(local, dtype=torch.float32)

    def _new_state_buffer(self, p: Tensor, grad: Tensor, spec: BufferSpec):
        if spec.like == "grad":
            buf = self._new_buffer(grad, spec.signed)
            if isinstance(buf, Tensor) and isinstance(grad, DTensor):
                return DTensor.from_local(
                    buf, device_mesh=grad.device_mesh, placements=grad.placements, run_check=False,
                    shape=grad.shape, stride=grad.stride(),
                )
            return buf
        return super()._new_state_buffer(p, grad, spec)

    # ---------------------------------------------------------------- driver
    def muon(self, algorithm: MuonAlgorithm, params, grads, state, lr_ratios, **kw):
        if not params:
            return
        quant_keys = [k for k, v in state.items() if any(local_quantized(b) is not None for b in v)]
        if not quant_keys:
            return super().muon(algorithm, params, grads, state, lr_ratios, **kw)
        opts = {k: v for k, v in kw.items() if k not in ("foreach",)}
        pending: dict[tuple, list[int]] = {}
        fused: dict[tuple, list[tuple]] = {}
        for i, (p, g, r) in enumerate(zip(params, grads, lr_ratios, strict=True)):
            st = {k: v[i] for k, v in state.items()}
            item = self._fused_lp(algorithm, p, g, st, r, opts)
            if item is not None:
                pl, ge, var, _ = item
                fused.setdefault((tuple(ge.shape), pl.dtype, var is not None), []).append(item)
                continue
            pending.setdefault((tuple(g.shape), g.dtype, str(g.device)), []).append(i)
        # Quantised momentum already stepped per tensor (lp_momentum_step); the
        # orthogonalisation + apply run batched per shape.
        for items in fused.values():
            ps, gs, vs = [it[0] for it in items], [it[1] for it in items], [it[2] for it in items]
            effs = [it[3] for it in items]
            muon_fused.fused_muon_update(
                ps, gs, gs, effs,
                weight_decay=opts["weight_decay"], cautious_wd=opts["cautious_wd"], momentum=0.0, nesterov=False,
                maximize=False, ns_steps=opts["ns_steps"], strategy=opts["orthogonalization_strategy"],
                variances=vs if vs[0] is not None else None, muon_beta2=opts.get("muon_beta2", 0.95),
                momentum_done=True,
            )
        # Generic: dequantise into fp32 temporaries, run the normal (batched when
        # on CUDA) update for a bounded chunk of same-shape tensors, requantise.
        for idxs in pending.values():
            for s in range(0, len(idxs), self._LP_CHUNK):
                sel = idxs[s : s + self._LP_CHUNK]
                temps: list[tuple[QuantizedState, Tensor]] = []
                sub = {k: [] for k in state}
                for i in sel:
                    g = grads[i]
                    for k in state:
                        q = local_quantized(state[k][i])
                        if q is None:
                            q = state[k][i]
                        else:
                            t = q.dequantize()
                            if isinstance(g, DTensor):
                                t = DTensor.from_local(
                                    t, device_mesh=g.device_mesh, placements=g.placements, run_check=False,
                                    shape=g.shape, stride=g.stride(),
                                )
                            temps.append((q, t))
                            q = t
                        sub[k].append(q)
                on_cuda = all(to_local(params[i]).is_cuda for i in sel)
                super().muon(
                    algorithm, [params[i] for i in sel], [grads[i] for i in sel], sub,
                    [lr_ratios[i] for i in sel], foreach=on_cuda, **opts,
                )
                for q, t in temps:
                    q.copy_(to_local(t))

    def _fused_lp(self, algorithm, p, g, st, lr_ratio, opts):
        """Step the quantised momentum of one tensor; returns (param, g', variance, lr_eff)
        for the batched orthogonalisation, or None when the fused path does not apply."""
        q = local_quantized(st.get("momentum_buffer"))
        if q is None or not q.codes.is_cuda:
            return None
        if type(algorithm) not in (MuonBaseline, NorMuon) or not algo_base._seams_are_builtin():
            return None
        if opts.get("split_sizes") is not None:
            return None
        if isinstance(p, DTensor) or isinstance(g, DTensor):
            # Dim-0-sharded 3-D stacks (EP experts): local shards are whole matrices.
            from ..orthogonalize import is_fsdp_3d_sharded

            if not (isinstance(p, DTensor) and is_fsdp_3d_sharded([g])):
                return None
            p, g = p.to_local(), g.to_local()
        if not (p.is_contiguous() and g.is_contiguous() and _ext.available()):
            return None
        if p.dtype not in (torch.float32, torch.bfloat16) or g.dtype not in (torch.float32, torch.bfloat16):
            return None
        variances = None
        if isinstance(algorithm, NorMuon):
            v = to_local(st["variance_neuron"])
            if local_quantized(v) is not None or not (v.is_cuda and v.is_contiguous()):
                return None
            variances = [v]
        g_eff = torch.empty(g.shape, dtype=torch.bfloat16, device=g.device)
        _ext.load().lp_momentum_step(
            q.codes, q.scale, q.qmap, q.fmt, q.block_size, g, g_eff, float(opts["momentum"]),
            bool(opts["nesterov"]), bool(opts["maximize"]),
        )
        return p, g_eff, variances[0] if variances is not None else None, lr_effs(opts["lr"], [lr_ratio])[0]


class Muon8bit(MuonLP):
    """MuonLP with 8-bit dynamic-tree momentum."""

    _fmt = FMT_8BIT


class Muon4bit(MuonLP):
    """MuonLP with 4-bit dynamic-tree momentum (two codes per byte)."""

    _fmt = FMT_4BIT


class MuonFp8(MuonLP):
    """MuonLP with fp8 (e4m3) block-scaled momentum."""

    _fmt = FMT_FP8
