"""MuonLP and the block-quantised momentum state on CPU (mirrors the reference's
tests/optim/test_optim_lp.py; unlike the reference, quantised states step)."""

import pytest
import torch
import torch.nn as nn

from dtensor_muon_b200 import Muon, Muon4bit, Muon8bit, MuonFp8, MuonLP, QuantizedState
from dtensor_muon_b200.optim.optim_lp import FMT_4BIT, FMT_8BIT, FMT_FP8, dynamic_tree_map


def test_dynamic_tree_map_shape_and_range():
    for bits in (8, 4):
        m = dynamic_tree_map(bits, signed=True)
        assert m.numel() == 2**bits
        assert torch.all(m[1:] >= m[:-1])
        assert m.max() == 1.0 and m.min() == -1.0 and (m == 0).any()
    u = dynamic_tree_map(8, signed=False)
    assert u.min() == 0 and u.max() == 1.0


@pytest.mark.parametrize("fmt,tol", [(FMT_FP8, 0.07), (FMT_8BIT, 0.06), (FMT_4BIT, 0.35)])
def test_quantize_round_trip(fmt, tol):
    torch.manual_seed(0)
    x = torch.randn(4096 * 2)
    q = QuantizedState.zeros(x.shape, fmt, 2048, True, "cpu")
    assert q.dequantize().abs().max() == 0
    q.copy_(x)
    y = q.dequantize()
    rel = (y - x).norm() / x.norm()
    assert rel < tol, rel
    # block absmax is exact
    blocks = x.view(-1, 2048)
    assert torch.allclose(y.view(-1, 2048).abs().amax(1), blocks.abs().amax(1), rtol=1e-6)


def test_lp_defaults_and_buffer_selection():
    big = nn.Parameter(torch.randn(64, 64))  # 4096 elements, divisible by 2048
    small = nn.Parameter(torch.randn(8, 8))
    odd = nn.Parameter(torch.randn(65, 64))
    opt = Muon8bit([big, small, odd])
    assert opt.param_groups[0]["foreach"] is False and opt.block_size == 2048
    assert opt.bf16_stochastic_round is False
    for p in (big, small, odd):
        p.grad = torch.randn_like(p)
    opt.step()
    assert isinstance(opt.state[big]["momentum_buffer"], QuantizedState)
    assert isinstance(opt.state[small]["momentum_buffer"], torch.Tensor)
    assert isinstance(opt.state[odd]["momentum_buffer"], torch.Tensor)
    base = MuonLP([nn.Parameter(torch.randn(64, 64))])
    p = base.param_groups[0]["params"][0]
    p.grad = torch.randn_like(p)
    base.step()
    assert base.state[p]["momentum_buffer"].dtype == torch.float32


@pytest.mark.parametrize("cls", [Muon8bit, Muon4bit, MuonFp8])
def test_quantized_states_step_and_track_fp32(cls):
    """A quantised momentum tracks the fp32 optimizer closely over a few steps."""
    torch.manual_seed(0)
    a = nn.Parameter(torch.randn(64, 128))
    b = nn.Parameter(a.detach().clone())
    oa = cls([a], lr=0.02, block_size=256)
    ob = Muon([b], lr=0.02)
    for i in range(3):
        g = torch.randn(64, 128, generator=torch.Generator().manual_seed(i))
        a.grad, b.grad = g.clone(), g.clone()
        oa.step()
        ob.step()
    m = oa.state[a]["momentum_buffer"]
    assert isinstance(m, QuantizedState)
    ref = ob.state[b]["momentum_buffer"]
    rel = (m.dequantize() - ref).norm() / ref.norm()
    assert rel < (0.3 if cls is Muon4bit else 0.08), rel
    assert torch.isfinite(a).all()
    assert ((a - b).norm() / (b.norm())) < 0.05


def test_lp_state_dict_round_trip(tmp_path):
    torch.manual_seed(0)
    a = nn.Parameter(torch.randn(64, 64))
    opt = MuonFp8([a], lr=0.01)
    a.grad = torch.randn_like(a)
    opt.step()
    path = tmp_path / "lp.pt"
    torch.save(opt.state_dict(), path)
    sd = torch.load(path, weights_only=True)
    b = nn.Parameter(a.detach().clone())
    opt2 = MuonFp8([b], lr=0.01)
    opt2.load_state_dict(sd)
    q = opt2.state[b]["momentum_buffer"]
    assert isinstance(q, QuantizedState)
    torch.testing.assert_close(q.dequantize(), opt.state[a]["momentum_buffer"].dequantize())
    g = torch.randn_like(a)
    a.grad, b.grad = g.clone(), g.clone()
    opt.step()
    opt2.step()
    torch.testing.assert_close(a, b)
