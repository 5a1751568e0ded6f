"""Native (sm_100a) orthogonalisation engine.

Replaces the reference's compiled loops ``ns_loop_triton`` / ``pe_loop_triton``
(src/muonium/orthogonalize/newton_schulz.py:60-107, polar_express.py:69-115)
and its Triton Gram kernel (src/muonium/kernels/gram.py). One call runs:

1. ``muon_pack``: stack, cast to bf16, transpose into the N <= M orientation
   and zero-pad to 256 multiples, with per-tile partial sums of squares;
2. ``norm_finalize``: 1 / (||X||_F * fac + eps) per matrix;
3. ``ortho_iterate``: for each step, three tcgen05 GEMMs with fused epilogues
   (A = s^2 X X^T, B = c A A + b A, X' = s (a X + B X)); the normalisation is
   folded into the first iteration's epilogues;
4. ``muon_unpack``: back to the caller's [B, R, C] bf16 layout.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor

from . import _ext

# Newton-Schulz quintic coefficients (newton_schulz.py:21-23 in the reference).
NS_COEFFS = (3.4445, -4.7750, 2.0315)

# Polar Express per-step coefficients, arXiv:2505.16932 (the published table,
# as used in polar_express.py:19-25 of the reference).
POLAR_EXPRESS_COEFFS = [
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
]

PAD = 256
# Upper bound on the bytes of one batch's workspace; larger batches are chunked.
MAX_WORKSPACE_BYTES = 6 << 30


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def coefficient_table(strategy: str, steps: int) -> Tensor:
    if strategy == "newton_schulz":
        rows = [NS_COEFFS] * steps
    elif strategy == "polar_express":
        if steps > len(POLAR_EXPRESS_COEFFS):
            raise AssertionError(
                "polar express orthogonalization only supports up to 5 optimization steps."
            )
        rows = POLAR_EXPRESS_COEFFS[:steps]
    else:
        raise ValueError(f"Unknown orthogonalization strategy: {strategy}")
    return torch.tensor(rows, dtype=torch.float64).reshape(steps, 3)


def norm_factor(strategy: str) -> float:
    # Polar Express divides by 1.02 * ||X|| (polar_express.py:56, :89).
    return 1.02 if strategy == "polar_express" else 1.0


@dataclass
class _Layout:
    R: int
    C: int
    transpose: bool
    N: int
    M: int
    Np: int
    Mp: int


def layout_for(R: int, C: int) -> _Layout:
    transpose = R > C
    N, M = (C, R) if transpose else (R, C)
    return _Layout(R, C, transpose, N, M, round_up(N, PAD), round_up(M, PAD))


class _WorkspacePool:
    """Grow-only per-device scratch for X, X', A and B (bf16)."""

    def __init__(self):
        self._bufs: dict[tuple[int, str], Tensor] = {}

    def get(self, device: torch.device, name: str, shape: tuple[int, ...]) -> Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), name)
        n = math.prod(shape)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < n:
            self._bufs.pop(key, None)
            buf = torch.empty(n, dtype=torch.bfloat16, device=device)
            self._bufs[key] = buf
        return buf[:n].view(shape)

    def clear(self):
        self._bufs.clear()


WORKSPACE = _WorkspacePool()


def ptr_tensor(ptrs: list[int], device: torch.device) -> Tensor:
    host = torch.tensor(ptrs, dtype=torch.int64)
    if device.type == "cuda":
        host = host.pin_memory()
    return host.to(device, non_blocking=True)


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return 0
    if dtype == torch.bfloat16:
        return 1
    raise TypeError(f"unsupported dtype {dtype}; native Muon paths take fp32 or bf16")


def batch_chunk(lay: _Layout, batch: int) -> int:
    per = 2 * (2 * lay.Np * lay.Mp + 2 * lay.Np * lay.Np)
    return max(1, min(batch, MAX_WORKSPACE_BYTES // max(per, 1)))


def run_iteration(x: Tensor, inv_norm: Tensor, lay: _Layout, steps: int, strategy: str, tag: str = "") -> Tensor:
    """Run ``steps`` fused iterations on the packed workspace ``x`` [B, Np, Mp]."""
    C = _ext.load()
    B = x.size(0)
    if steps == 0:
        return x
    x2 = WORKSPACE.get(x.device, "x2" + tag, (B, lay.Np, lay.Mp))
    a = WORKSPACE.get(x.device, "a" + tag, (B, lay.Np, lay.Np))
    b = WORKSPACE.get(x.device, "b" + tag, (B, lay.Np, lay.Np))
    return C.ortho_iterate(x, x2, a, b, inv_norm, coefficient_table(strategy, steps), 0)


def orthogonalize_native(
    mats: list[Tensor], steps: int, strategy: str, eps: float = 1e-7
) -> list[Tensor]:
    """Orthogonalise same-shape CUDA matrices; returns bf16 tensors of the same shape."""
    if not mats:
        return []
    C = _ext.load()
    R, Cc = mats[0].shape[-2], mats[0].shape[-1]
    device = mats[0].device
    coefficient_table(strategy, steps)  # validates strategy / steps
    lay = layout_for(R, Cc)
    outs: list[Tensor] = []
    chunk = batch_chunk(lay, len(mats))
    for i in range(0, len(mats), chunk):
        part = [m if m.is_contiguous() else m.contiguous() for m in mats[i : i + chunk]]
        if part[0].dtype not in (torch.float32, torch.bfloat16):
            part = [m.float() for m in part]
        B = len(part)
        x = WORKSPACE.get(device, "x", (B, lay.Np, lay.Mp))
        ptrs = ptr_tensor([m.data_ptr() for m in part], device)
        vec_ok = all(m.data_ptr() % 16 == 0 for m in part)
        partial = C.muon_pack_ex(
            ptrs, None, dtype_code(part[0].dtype), R, Cc, Cc, lay.transpose, x, 0.0, False, False, vec_ok
        )
        inv = C.norm_finalize(partial, norm_factor(strategy), eps)
        if steps == 0:
            out = C.muon_unpack(x, lay.transpose, R, Cc, inv)
        else:
            res = run_iteration(x, inv, lay, steps, strategy)
            out = C.muon_unpack(res, lay.transpose, R, Cc, None)
        outs.extend(out.unbind(0))
    return outs


def gram(x: Tensor) -> Tensor:
    """``x @ x.mT`` over the last two dims with the symmetric tcgen05 kernel (bf16)."""
    C = _ext.load()
    assert x.is_cuda and x.dtype == torch.bfloat16 and x.ndim >= 2
    lead = x.shape[:-2]
    M, K = x.shape[-2], x.shape[-1]
    xb = x.reshape(-1, M, K)
    B = xb.size(0)
    Mp, Kp = round_up(M, PAD), round_up(K, PAD)
    xp = torch.zeros(B, Mp, Kp, dtype=torch.bfloat16, device=x.device)
    xp[:, :M, :K] = xb
    out = torch.empty(B, Mp, Mp, dtype=torch.bfloat16, device=x.device)
    C.gram_sym(xp, out, None, None, 1.0, 0.0, 0, 0, 0)
    return out[:, :M, :M].reshape(*lead, M, M)
