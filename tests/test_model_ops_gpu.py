"""Fused RoPE / SwiGLU kernels against fp32 PyTorch (forward and backward)."""

import pytest
import torch
import torch.nn.functional as F

from dtensor_muon_b200.models.llama import rope_tables
from dtensor_muon_b200.ops import _ext, model_ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(2, 64, 4, 128), (1, 33, 8, 64), (1, 4096, 8, 128)])
def test_rope_fwd_bwd(shape):
    torch.manual_seed(0)
    cos, sin = rope_tables(shape[-1], shape[1], 10000.0, "cuda")
    x = torch.randn(shape, device="cuda").bfloat16().requires_grad_()
    xr = x.detach().float().requires_grad_()
    n0 = _ext.launch_count
    y = model_ops.rope(x, cos, sin)
    yr = model_ops.rope_reference(xr, cos, sin)
    torch.testing.assert_close(y.float(), yr, rtol=1e-2, atol=1e-2)
    g = torch.randn(shape, device="cuda")
    y.backward(g.bfloat16())
    yr.backward(g)
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=1e-2, atol=2e-2)
    assert _ext.launch_count - n0 == 2


def test_swiglu_fwd_bwd():
    torch.manual_seed(1)
    a = torch.randn(257, 384, device="cuda").bfloat16().requires_grad_()
    b = torch.randn(257, 384, device="cuda").bfloat16().requires_grad_()
    ar, br = a.detach().float().requires_grad_(), b.detach().float().requires_grad_()
    h = model_ops.swiglu(a, b)
    hr = F.silu(ar) * br
    torch.testing.assert_close(h.float(), hr, rtol=1e-2, atol=1e-2)
    g = torch.randn_like(hr)
    h.backward(g.bfloat16())
    hr.backward(g)
    torch.testing.assert_close(a.grad.float(), ar.grad, rtol=2e-2, atol=3e-2)
    torch.testing.assert_close(b.grad.float(), br.grad, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("T,V", [(64, 1024), (33, 32000), (8, 128256)])
def test_cross_entropy_fwd_bwd(T, V):
    torch.manual_seed(2)
    logits = (torch.randn(T, V, device="cuda") * 3).bfloat16().requires_grad_()
    targets = torch.randint(0, V, (T,), device="cuda")
    ref_in = logits.detach().float().requires_grad_()
    loss = model_ops.cross_entropy(logits, targets)
    ref = F.cross_entropy(ref_in, targets)
    torch.testing.assert_close(loss, ref, rtol=1e-4, atol=1e-4)
    loss.backward()
    ref.backward()
    torch.testing.assert_close(logits.grad.float(), ref_in.grad, rtol=2e-2, atol=1e-4)


def test_swiglu_and_rope_through_the_test_kit():
    """Fused kernels vs fp32 PyTorch via check_impls (forward, shared-cotangent
    backward, CUDA-event timing with L2 flush)."""
    from testkit import check_impls

    torch.manual_seed(2)
    a = torch.randn(1024, 2048, device="cuda").bfloat16().requires_grad_()
    b = torch.randn(1024, 2048, device="cuda").bfloat16().requires_grad_()
    times = check_impls(
        {"dmb.swiglu": model_ops.swiglu},
        {"torch_fp32": lambda x, y: (F.silu(x.float()) * y.float()), "torch_bf16": lambda x, y: F.silu(x) * y},
        (a, b), rtol=2e-2, atol=2e-2, bwd=True,
    )
    assert set(times) == {"dmb.swiglu", "torch_fp32", "torch_bf16"} and all(t > 0 for t in times.values())
    cos, sin = rope_tables(128, 512, 10000.0, "cuda")
    x = torch.randn(2, 512, 8, 128, device="cuda").bfloat16().requires_grad_()
    check_impls(lambda t: model_ops.rope(t, cos, sin), lambda t: model_ops.rope_reference(t.float(), cos, sin),
                (x,), rtol=2e-2, atol=3e-2, bwd=True, bench=False)
