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


def _closed_form_codes(x, qmap):
    """float32 restatement of the CUDA kernel's closed-form nearest code
    (``nearest_code`` in ops/csrc/lp_quant.cu), vectorised with numpy."""
    import numpy as np

    q = qmap.numpy().astype(np.float32)
    n = q.size
    bits = 8 if n == 256 else 4
    sgn = q[0] < 0
    V = bits - 1 if sgn else bits
    P = (1 << V) - 1
    neg0 = P if sgn else 0
    x = x.numpy().astype(np.float32)

    f32 = np.float32
    lim = [f32(1.0)]
    for _ in range(8):
        lim.append(f32(lim[-1] * f32(0.1)))
    lim = np.array(lim[1:], dtype=np.float32)  # lim[k] = 10^-(k+1)
    up = [f32(1.0)]
    for _ in range(8):
        up.append(f32(up[-1] * f32(10.0)))
    up = np.array(up, dtype=np.float32)
    cnt = np.array([f32(f32(1 << (V - k - 1)) / f32(0.9)) if k < V else 0 for k in range(8)], dtype=np.float32)

    def count_le(t):
        k = np.zeros(t.shape, dtype=np.int64)
        for j in range(7):
            if j < V - 1:
                k += (t <= lim[j]).astype(np.int64)
        nk = (1 << (V - k - 1)).astype(np.float32)
        fm = (t.astype(np.float64) * up[k].astype(np.float64) - np.float64(f32(0.1))).astype(np.float32)
        f = np.floor((fm * cnt[k]).astype(np.float32))
        return (nk - 1 + np.clip(f, 0, nk)).astype(np.int64)

    P_ = P
    zoff = n - P_
    le = np.where(x >= 0, zoff + count_le(np.abs(x)), P - count_le(np.abs(x)))
    lo = np.clip(le - 1, 0, n - 2)
    hi = lo + 1
    return torch.from_numpy(np.where(np.abs(q[hi] - x) < np.abs(x - q[lo]), hi, lo).astype(np.uint8))


def test_closed_form_values_equal_the_table():
    from dtensor_muon_b200.optim.optim_lp import _tree_mag

    for bits, signed in ((8, True), (4, True), (8, False), (4, False)):
        q = dynamic_tree_map(bits, signed)
        V = bits - 1 if signed else bits
        mags = torch.tensor([_tree_mag(V, j) for j in range(2**V - 1)], dtype=torch.float32)
        assert torch.equal(q[-(2**V - 1):], mags)


@pytest.mark.parametrize("bits,signed", [(8, True), (4, True), (8, False), (4, False)])
def test_closed_form_code_index_matches_search(bits, signed):
    """The kernel's arithmetic code index equals the sorted-map search on every
    code value, every midpoint between codes, their float neighbours and random
    values in [-1, 1]."""
    from dtensor_muon_b200.optim.optim_lp import _nearest_codes

    qmap = dynamic_tree_map(bits, signed)
    mids = (qmap[1:] + qmap[:-1]) / 2
    base = torch.cat([qmap, mids, torch.rand(200000) * 2 - 1 if signed else torch.rand(200000)])
    xs = torch.cat([base, torch.nextafter(base, torch.tensor(2.0)), torch.nextafter(base, torch.tensor(-2.0))])
    if not signed:
        xs = xs.clamp(min=0.0)
    want = _nearest_codes(xs, qmap)
    got = _closed_form_codes(xs, qmap)
    bad = (want != got).nonzero().flatten()
    assert bad.numel() == 0, [(xs[i].item(), want[i].item(), got[i].item()) for i in bad[:5]]


def _lp_dcp_worker(rank, world, ckpt_dir, cls_name):
    import torch
    import torch.distributed.checkpoint as dcp
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import DTensor, Shard, distribute_tensor

    import dtensor_muon_b200 as dmb
    from dtensor_muon_b200.optim.optim_lp import QuantizedState

    cls = getattr(dmb, cls_name)
    mesh = init_device_mesh("cpu", (world,))
    torch.manual_seed(0)
    full = torch.randn(128, 64)
    grads = [torch.randn(128, 64) for _ in range(3)]

    def make():
        p = torch.nn.Parameter(distribute_tensor(full.clone(), mesh, [Shard(0)]))
        return p, (cls([p], lr=0.02) if cls_name == "Muon" else cls([p], lr=0.02, block_size=1024))

    p, opt = make()
    for g in grads[:2]:
        p.grad = distribute_tensor(g, mesh, [Shard(0)])
        opt.step()
    m = opt.state[p]["momentum_buffer"]
    # the quantised momentum keeps the parameter's mesh and placements
    assert isinstance(m, DTensor) and list(m.placements) == [Shard(0)] and m.shape == p.shape
    quantised = cls_name != "Muon"
    assert isinstance(m.to_local(), QuantizedState) == quantised
    dcp.save({"optim": opt.state_dict()}, checkpoint_id=ckpt_dir)

    p2, opt2 = make()
    p2.grad = distribute_tensor(torch.zeros(128, 64), mesh, [Shard(0)])
    opt2.step()  # materialise state with the same structure, then load into it in place
    with torch.no_grad():
        p2.copy_(p)
    sd = {"optim": opt2.state_dict()}
    dcp.load(sd, checkpoint_id=ckpt_dir)
    opt2.load_state_dict(sd["optim"])
    m2 = opt2.state[p2]["momentum_buffer"]
    assert isinstance(m2, DTensor) and isinstance(m2.to_local(), QuantizedState) == quantised
    if quantised:
        torch.testing.assert_close(m2.to_local().dequantize(), m.to_local().dequantize())
    else:
        torch.testing.assert_close(m2.full_tensor(), m.full_tensor())
    for o, q in ((opt, p), (opt2, p2)):
        q.grad = distribute_tensor(grads[2], mesh, [Shard(0)])
        o.step()
    torch.testing.assert_close(p2.full_tensor(), p.full_tensor())


@pytest.mark.parametrize("cls_name", ["Muon8bit", "Muon4bit", "MuonFp8", "Muon"])
def test_quantized_dtensor_state_dcp_round_trip_gloo(tmp_path, cls_name):
    """DTensor optimizer state (quantised or fp32) saved and reloaded through
    torch.distributed.checkpoint; training resumes identically."""
    from dtensor_muon_b200.testing.distributed import run_distributed

    run_distributed(_lp_dcp_worker, 2, args=(str(tmp_path / "ckpt"), cls_name))


def _lut_codes(x, qmap):
    """numpy restatement of the persistent kernel's table-driven nearest code
    (``lut_fill`` / ``nearest_code_lut`` in ops/csrc/lp_quant.cu)."""
    import numpy as np

    q = qmap.numpy().astype(np.float32)
    n = q.size
    bits = 8 if n == 256 else 4
    V = bits - 1 if q[0] < 0 else bits
    P = (1 << V) - 1
    zoff = n - P
    mag = q[zoff:]
    MB, EMIN = 8, 127 - 24
    N = 25 << MB
    idx = np.arange(N, dtype=np.uint64)
    edges = ((idx + (EMIN << MB)) << (23 - MB)).astype(np.uint32).view(np.float32)
    edges[0] = 0.0
    lut = np.searchsorted(mag, edges, side="right")  # magnitudes <= edge
    x = x.numpy().astype(np.float32)
    t = np.abs(x)
    key = np.clip((t.view(np.uint32) >> (23 - MB)).astype(np.int64) - (EMIN << MB), 0, N - 1)
    c = lut[key]
    cnt = c + ((c < P) & (mag[np.minimum(c, P - 1)] <= t))
    le = np.where(x >= 0, zoff + cnt, P - cnt)
    lo = np.clip(le - 1, 0, n - 2)
    hi = lo + 1
    return torch.from_numpy(np.where(np.abs(q[hi] - x) < np.abs(x - q[lo]), hi, lo).astype(np.uint8))


@pytest.mark.parametrize("bits,signed", [(8, True), (4, True), (8, False), (4, False)])
def test_table_code_index_matches_search(bits, signed):
    from dtensor_muon_b200.optim.optim_lp import _nearest_codes

    qmap = dynamic_tree_map(bits, signed)
    mids = (qmap[1:] + qmap[:-1]) / 2
    base = torch.cat([qmap, mids, torch.rand(200000) * 2 - 1 if signed else torch.rand(200000),
                      torch.tensor([1e-30, 3e-8, 1e-7, 1.0, 1.0000001])])
    xs = torch.cat([base, torch.nextafter(base, torch.tensor(2.0)), torch.nextafter(base, torch.tensor(-2.0))])
    if not signed:
        xs = xs.clamp(min=0.0)
    want = _nearest_codes(xs, qmap)
    got = _lut_codes(xs, qmap)
    bad = (want != got).nonzero().flatten()
    assert bad.numel() == 0, [(xs[i].item(), want[i].item(), got[i].item()) for i in bad[:5]]
