"""Test helpers: mismatch-budget comparison and the distributed spawner."""

from __future__ import annotations

import torch

from dtensor_muon_b200.testing import run_distributed  # noqa: F401

requires_cuda = None


def assert_close(actual, expected, *, rtol=1e-2, atol=1e-1, max_mismatch_pct=None, msg=None):
    """``torch.testing.assert_close`` in fp32, optionally allowing a small
    percentage of elements outside tolerance (for bf16 kernels)."""
    a = actual.detach().to(torch.float32).cpu()
    e = expected.detach().to(torch.float32).cpu()
    if max_mismatch_pct is None:
        torch.testing.assert_close(a, e, rtol=rtol, atol=atol, msg=msg)
        return
    bad = ~torch.isclose(a, e, rtol=rtol, atol=atol)
    pct = 100.0 * bad.sum().item() / max(bad.numel(), 1)
    if pct > max_mismatch_pct:
        raise AssertionError(
            f"{msg or ''}\n{pct:.4f}% of elements mismatched (allowed {max_mismatch_pct}%) at rtol={rtol}, atol={atol}"
        )


def clone_args(args):
    return tuple(
        a.detach().clone().requires_grad_(a.requires_grad) if isinstance(a, torch.Tensor) else a for a in args
    )
