"""torch.library registrations (``torch.ops.dmb``): schemas, fake kernels,
autograd formulas and the CPU kernels against fp32 PyTorch references."""

import pytest
import torch
import torch.nn.functional as F

from dtensor_muon_b200.ops import library
from dtensor_muon_b200.orthogonalize import zeropower as zp


def _rope_inputs(device="cpu", dtype=torch.float32):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 6, 3, 8, generator=g).to(device, dtype)
    ang = torch.randn(6, 4, generator=g)
    return x, ang.cos().to(device), ang.sin().to(device)


def _opcheck(op, args):
    torch.library.opcheck(op, args, test_utils=("test_schema", "test_autograd_registration", "test_faketensor"))


def test_ops_are_registered():
    for name in ("rope", "swiglu", "swiglu_backward", "cross_entropy", "cross_entropy_backward", "gram", "zeropower"):
        assert hasattr(torch.ops.dmb, name)


def test_rope_cpu_matches_rotation_and_inverts():
    x, cos, sin = _rope_inputs()
    y = torch.ops.dmb.rope(x, cos, sin, 1.0)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    c, s = cos[None, :, None], sin[None, :, None]
    ref = torch.stack((x0 * c - x1 * s, x0 * s + x1 * c), -1).flatten(-2)
    torch.testing.assert_close(y, ref)
    torch.testing.assert_close(torch.ops.dmb.rope(y, cos, sin, -1.0), x, atol=1e-5, rtol=1e-5)
    _opcheck(torch.ops.dmb.rope.default, (x.requires_grad_(), cos, sin, 1.0))


def test_rope_backward_is_inverse_rotation():
    x, cos, sin = _rope_inputs()
    x.requires_grad_()
    g = torch.randn_like(x)
    torch.ops.dmb.rope(x, cos, sin, 1.0).backward(g)
    torch.testing.assert_close(x.grad, torch.ops.dmb.rope(g, cos, sin, -1.0))


def test_swiglu_cpu_forward_backward():
    a = torch.randn(4, 16, requires_grad=True)
    b = torch.randn(4, 16, requires_grad=True)
    g = torch.randn(4, 16)
    library.swiglu(a, b).backward(g)
    a2, b2 = a.detach().clone().requires_grad_(), b.detach().clone().requires_grad_()
    (F.silu(a2) * b2).backward(g)
    torch.testing.assert_close(a.grad, a2.grad, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(b.grad, b2.grad, atol=1e-5, rtol=1e-5)
    _opcheck(torch.ops.dmb.swiglu.default, (a, b))
    _opcheck(torch.ops.dmb.swiglu_backward.default, (a.detach(), b.detach(), g))


def test_cross_entropy_cpu_forward_backward():
    logits = torch.randn(10, 32, requires_grad=True)
    t = torch.randint(0, 32, (10,))
    loss, lse = library.cross_entropy(logits, t)
    (2.0 * loss).backward()
    l2 = logits.detach().clone().requires_grad_()
    ref = F.cross_entropy(l2, t)
    (2.0 * ref).backward()
    torch.testing.assert_close(loss, ref)
    torch.testing.assert_close(lse, torch.logsumexp(logits.detach(), -1))
    torch.testing.assert_close(logits.grad, l2.grad, atol=1e-6, rtol=1e-5)
    _opcheck(torch.ops.dmb.cross_entropy.default, (logits, t))


def test_gram_and_zeropower_cpu():
    x = torch.randn(3, 8, 24)
    torch.testing.assert_close(torch.ops.dmb.gram(x).float(), x @ x.mT, atol=0.1, rtol=1e-2)
    u = torch.ops.dmb.zeropower(x, 5, "polar_express", 1e-7)
    assert u.dtype == torch.bfloat16 and u.shape == x.shape
    torch.testing.assert_close(u, zp(x, steps=5, strategy="polar_express", use_native=False))
    _opcheck(torch.ops.dmb.gram.default, (x,))
    _opcheck(torch.ops.dmb.zeropower.default, (x, 5, "newton_schulz", 1e-7))


def test_ops_trace_under_fake_mode():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty(2, 6, 3, 8)
        cos = torch.empty(6, 4)
        assert torch.ops.dmb.rope(x, cos, cos, 1.0).shape == x.shape
        assert torch.ops.dmb.gram(torch.empty(5, 7, 9)).shape == (5, 7, 7)
        loss, lse = torch.ops.dmb.cross_entropy(torch.empty(4, 11), torch.zeros(4, dtype=torch.long))
        assert loss.shape == () and lse.shape == (4,)


@pytest.mark.gpu
def test_cuda_ops_match_cpu_kernels_and_compile():
    dev = "cuda"
    x, cos, sin = _rope_inputs(dev, torch.bfloat16)
    torch.testing.assert_close(torch.ops.dmb.rope(x, cos, sin, 1.0).float(),
                               torch.ops.dmb.rope(x.float().cpu(), cos.cpu(), sin.cpu(), 1.0).to(dev),
                               atol=2e-2, rtol=2e-2)
    a = torch.randn(64, 256, device=dev, dtype=torch.bfloat16)
    b = torch.randn(64, 256, device=dev, dtype=torch.bfloat16)
    torch.testing.assert_close(torch.ops.dmb.swiglu(a, b).float(), (F.silu(a.float()) * b.float()), atol=3e-2, rtol=2e-2)
    xg = torch.randn(2, 256, 512, device=dev, dtype=torch.bfloat16)
    torch.testing.assert_close(torch.ops.dmb.gram(xg).float(), xg.float() @ xg.float().mT, atol=0.5, rtol=2e-2)
    for op, args in (
        (torch.ops.dmb.rope.default, (x.detach().requires_grad_(), cos, sin, 1.0)),
        (torch.ops.dmb.swiglu.default, (a.requires_grad_(), b)),
    ):
        _opcheck(op, args)

    def block(h, w, t):
        h = torch.ops.dmb.rope(h, cos, sin, 1.0)
        z = h.flatten(1) @ w
        u, v = z.chunk(2, dim=-1)
        y = torch.ops.dmb.swiglu(u.contiguous(), v.contiguous())
        return torch.ops.dmb.cross_entropy(y.contiguous(), t)[0]

    h = torch.randn(12, 6, 3, 8, device=dev, dtype=torch.bfloat16)
    w = (0.1 * torch.randn(144, 128, device=dev)).bfloat16().requires_grad_()
    t = torch.randint(0, 64, (12,), device=dev)
    loss_e = block(h, w, t)
    (gw_e,) = torch.autograd.grad(loss_e, w)
    compiled = torch.compile(block, fullgraph=True)
    loss_c = compiled(h, w, t)
    (gw_c,) = torch.autograd.grad(loss_c, w)
    torch.testing.assert_close(loss_c, loss_e, atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(gw_c.float(), gw_e.float(), atol=1e-2, rtol=1e-2)
