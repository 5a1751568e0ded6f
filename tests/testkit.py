"""Test kit: tolerant comparison, forward/backward checks of an implementation
against a baseline, CUDA-event timing, and the distributed spawner.

Covers what the reference's tests/testkit.py offers (``assert_close`` with a
mismatch budget, ``clone_args``, ``run_example`` with a backward check,
``do_bench``), built differently:

* :func:`check_impls` runs every candidate and the baseline on private clones
  of the inputs, compares all outputs in fp32 against the FIRST baseline and,
  with ``bwd=True``, pushes one shared random cotangent through every callable
  and compares the input gradients.
* :func:`time_cuda` times with CUDA events on the current stream, flushing L2
  (a write larger than the 126 MB L2) before every timed call, and returns the
  median in ms; no Triton.
"""

from __future__ import annotations

import statistics
import sys
from typing import Callable, Sequence

import torch

from dtensor_muon_b200.testing import run_distributed  # noqa: F401  (re-export for the test files)

Fn = Callable[..., object]


def assert_close(actual, expected, *, rtol=1e-2, atol=1e-1, max_mismatch_pct=None, msg=None):
    """``torch.testing.assert_close`` in fp32, optionally allowing a small
    percentage of elements outside tolerance (for bf16 kernels)."""
    a = actual.detach().to(torch.float32).cpu()
    e = expected.detach().to(torch.float32).cpu()
    if max_mismatch_pct is None:
        torch.testing.assert_close(a, e, rtol=rtol, atol=atol, msg=msg)
        return
    if a.shape != e.shape:
        raise AssertionError(f"{msg or ''}\nshape mismatch: {tuple(a.shape)} vs {tuple(e.shape)}")
    bad = ~torch.isclose(a, e, rtol=rtol, atol=atol)
    pct = 100.0 * bad.sum().item() / max(bad.numel(), 1)
    if pct > max_mismatch_pct:
        raise AssertionError(
            f"{msg or ''}\n{pct:.4f}% of elements mismatched (allowed {max_mismatch_pct}%) at rtol={rtol}, atol={atol}"
        )


def clone_args(args):
    """Fresh tuple; tensors detached and cloned with their ``requires_grad``, other values shared."""
    return tuple(
        a.detach().clone().requires_grad_(a.requires_grad) if isinstance(a, torch.Tensor) else a for a in args
    )


def as_tensors(out) -> list[torch.Tensor]:
    """A callable's result as a list of tensors (a tensor, or a tuple/list of tensors)."""
    if isinstance(out, torch.Tensor):
        return [out]
    if isinstance(out, (list, tuple)) and all(isinstance(t, torch.Tensor) for t in out):
        return list(out)
    raise TypeError(f"expected a tensor or a sequence of tensors, got {type(out).__name__}")


def _named(fns, default: str) -> dict[str, Fn]:
    return dict(fns) if isinstance(fns, dict) else {default: fns}


def check_impls(
    impls: Fn | dict[str, Fn],
    baselines: Fn | dict[str, Fn],
    args: Sequence[object],
    *,
    rtol: float = 1e-2,
    atol: float = 1e-1,
    max_mismatch_pct: float | None = None,
    bwd: bool = False,
    bench: bool | None = None,
) -> dict[str, float]:
    """Check ``impls`` (and any extra baselines) against the first baseline.

    Every callable gets its own clones of ``args``. With ``bwd`` one random
    cotangent per output (shared by all callables) is back-propagated and the
    gradients of the inputs that require grad are compared, including which
    of them received a gradient at all. With ``bench`` (default: CUDA
    available) each callable is then timed with :func:`time_cuda`; returns
    ``{name: median ms}`` (empty when not timed).
    """
    cand = _named(impls, "impl")
    base = _named(baselines, "baseline")
    ref_name = next(iter(base))
    others = {**cand, **{k: v for k, v in base.items() if k != ref_name}}

    want = as_tensors(base[ref_name](*clone_args(args)))
    for name, fn in others.items():
        got = as_tensors(fn(*clone_args(args)))
        if len(got) != len(want):
            raise AssertionError(f"{name}: {len(got)} outputs, baseline {ref_name} has {len(want)}")
        for i, (g, w) in enumerate(zip(got, want)):
            assert_close(g, w, rtol=rtol, atol=atol, max_mismatch_pct=max_mismatch_pct,
                         msg=f"{name}: output {i} {tuple(g.shape)}")

    if bwd:
        idx = [i for i, a in enumerate(args) if isinstance(a, torch.Tensor) and a.requires_grad]
        if not idx:
            raise AssertionError("bwd=True needs at least one input with requires_grad=True")

        def grads_of(fn, cot=None):
            local = clone_args(args)
            outs = as_tensors(fn(*local))
            if cot is None:
                cot = [torch.randn_like(o) for o in outs]
            if len(cot) != len(outs):
                raise AssertionError(f"{len(outs)} outputs, baseline has {len(cot)}")
            torch.autograd.backward(outs, cot)
            return cot, [None if local[i].grad is None else local[i].grad.detach().clone() for i in idx]

        cot, want_g = grads_of(base[ref_name])
        if all(g is None for g in want_g):
            raise AssertionError(f"baseline {ref_name} produced no gradients")
        for name, fn in others.items():
            _, got_g = grads_of(fn, cot)
            for i, g, w in zip(idx, got_g, want_g):
                if (g is None) != (w is None):
                    raise AssertionError(f"{name}: gradient of input {i} present={g is not None}, "
                                         f"baseline present={w is not None}")
                if w is not None:
                    assert_close(g, w, rtol=rtol, atol=atol, max_mismatch_pct=max_mismatch_pct,
                                 msg=f"{name}: gradient of input {i} {tuple(g.shape)}")

    if bench is None:
        bench = torch.cuda.is_available()
    if not bench:
        return {}
    times = {name: time_cuda(lambda fn=fn, a=clone_args(args): fn(*a)) for name, fn in {**base, **cand}.items()}
    print_times(times, ref_name)
    return times


_FLUSH: dict[int, torch.Tensor] = {}


def time_cuda(fn: Callable[[], object], *, warmup: int = 3, reps: int = 20, flush_l2: bool = True) -> float:
    """Median device time of ``fn`` in ms: CUDA events on the current stream,
    ``warmup`` untimed calls, a synchronize on both sides, and (``flush_l2``) a
    256 MiB write before every timed call so no input is served from L2."""
    dev = torch.cuda.current_device()
    if flush_l2 and dev not in _FLUSH:
        _FLUSH[dev] = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        if flush_l2:
            _FLUSH[dev].zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.median(times)


def print_times(times: dict[str, float], ref: str, file=sys.stderr) -> None:
    """One line per callable: ms and speed-up over ``ref`` (marked ``*``)."""
    t0 = times.get(ref)
    for name, t in times.items():
        mark = "*" if name == ref else " "
        speed = f"{t0 / t:6.2f}x" if t0 and t else "   n/a"
        print(f"{mark} {name:<24} {t:10.4f} ms  {speed}", file=file)
