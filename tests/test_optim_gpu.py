"""Native CUDA optimizer paths against the PyTorch formulations
(mirrors the reference's CUDA-gated tests in tests/optim/)."""

import pytest
import torch
import torch.nn as nn

import dtensor_muon_b200.optim.algorithms.base as algo_base
from dtensor_muon_b200 import Muon, Muon4bit, Muon8bit, MuonFp8
from dtensor_muon_b200.ops import _ext
from testkit import assert_close

pytestmark = pytest.mark.gpu

RTOL, ATOL, PCT = 1e-2, 3e-2, 5.0
SHAPES = [(64, 96), (96, 64), (128, 128), (3, 32, 48), (256, 1024), (1024, 256), (17, 33)]


def _params(seed, device="cuda", dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return [nn.Parameter(torch.randn(s, generator=g).to(device=device, dtype=dtype)) for s in SHAPES]


def _run(opt, params, steps=3, seed=123, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    for _ in range(steps):
        for p in params:
            p.grad = torch.randn(p.shape, generator=g).to(device=p.device, dtype=dtype)
        opt.step()
    torch.cuda.synchronize()


@pytest.mark.parametrize("strategy", ["newton_schulz", "polar_express"])
@pytest.mark.parametrize("cautious", [True, False])
@pytest.mark.parametrize("nesterov", [True, False])
@pytest.mark.parametrize("wd", [0.0, 0.3])
def test_foreach_matches_per_param(monkeypatch, strategy, cautious, nesterov, wd):
    """Fused foreach kernels vs the per-parameter PyTorch formulation with the
    PyTorch orthogonalisation loop (no native kernel on that side)."""
    from dtensor_muon_b200.orthogonalize import orthogonalize as om

    kw = dict(lr=0.2, wd=wd, nesterov=nesterov, use_cautious_wd=cautious, orthogonalization_strategy=strategy)
    a, b = _params(0), _params(0)
    monkeypatch.setattr(algo_base, "zeropower", lambda g, **k: om.zeropower(g, use_native=False, **k))
    monkeypatch.setattr(algo_base, "foreach_zeropower",
                        lambda gs, **k: om.foreach_zeropower(gs, use_native=False, **k))
    oa = Muon(a, foreach=False, **kw)
    n0 = _ext.launch_count
    _run(oa, a)
    assert _ext.launch_count == n0, "the per-parameter torch side must not launch native kernels"
    monkeypatch.undo()
    ob = Muon(b, foreach=True, **kw)
    _run(ob, b)
    assert _ext.launch_count > n0
    for x, y in zip(a, b):
        assert_close(y, x, rtol=RTOL, atol=ATOL, max_mismatch_pct=PCT)
    _ext.check_device_errors("cuda")


@pytest.mark.parametrize("algorithm", ["muon", "normuon"])
@pytest.mark.parametrize("maximize", [False, True])
def test_native_matches_torch_formulation(monkeypatch, algorithm, maximize):
    """Fused kernels vs the PyTorch formulation (forced by wrapping the seam)."""
    from dtensor_muon_b200.orthogonalize import orthogonalize as om

    a, b = _params(1), _params(1)
    kw = dict(lr=0.1, wd=0.2, maximize=maximize)
    oa = Muon([{"params": a, "algorithm": algorithm}], **kw)
    _run(oa, a)
    # a wrapper around the same function disables the fused path
    monkeypatch.setattr(algo_base, "foreach_zeropower", lambda gs, **k: om.foreach_zeropower(gs, **k))
    ob = Muon([{"params": b, "algorithm": algorithm}], **kw)
    _run(ob, b)
    for x, y in zip(a, b):
        assert_close(x, y, rtol=RTOL, atol=ATOL, max_mismatch_pct=PCT)
    if algorithm == "normuon":
        for x, y in zip(a, b):
            assert_close(oa.state[x]["variance_neuron"], ob.state[y]["variance_neuron"], rtol=5e-2, atol=1e-6)


def test_bf16_params_fp32_momentum():
    a = _params(2, dtype=torch.bfloat16)
    opt = Muon(a, lr=0.05)
    _run(opt, a, dtype=torch.bfloat16)
    for p in a:
        assert p.dtype == torch.bfloat16 and opt.state[p]["momentum_buffer"].dtype == torch.float32
        assert torch.isfinite(p).all()


@pytest.mark.parametrize("amsgrad", [False, True])
@pytest.mark.parametrize("algorithm", ["adamw", "adam"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_native_adam_matches_torch(amsgrad, algorithm, dtype):
    g = torch.Generator().manual_seed(0)
    shapes = [(7,), (33, 5), (1000,)]
    a = [nn.Parameter(torch.randn(s, generator=g).cuda().to(dtype)) for s in shapes]
    # fp32 reference: the native kernel does fp32 math with one rounding per
    # state write, while torch's bf16 path rounds after every sub-step.
    b = [nn.Parameter(t.detach().clone().float()) for t in a]
    opt = Muon([{"params": a, "algorithm": algorithm, "lr": 0.01, "wd": 0.1, "amsgrad": amsgrad}])
    cls = torch.optim.AdamW if algorithm == "adamw" else torch.optim.Adam
    ref = cls(b, lr=0.01, weight_decay=0.1, betas=(0.9, 0.95), amsgrad=amsgrad, foreach=False)
    n0 = _ext.launch_count
    for _ in range(3):
        for x, y in zip(a, b):
            gr = torch.randn(x.shape, generator=g).cuda().to(dtype)
            x.grad, y.grad = gr.clone(), gr.clone().float()
        opt.step()
        ref.step()
    assert _ext.launch_count - n0 == 3, "native AdamW kernel must run once per step"
    tol = dict(rtol=1e-5, atol=1e-6) if dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)
    for x, y in zip(a, b):
        torch.testing.assert_close(x.float(), y.detach(), **tol)


@pytest.mark.parametrize("algorithm,maximize", [("adamw", False), ("adam", True)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_vector_adam_matches_torch(algorithm, maximize, dtype):
    """Aligned sizes (multiples of 8) take the 16-byte vector path; the group mixes
    tiny and large tensors so several CTAs look up their tensor in one launch."""
    g = torch.Generator().manual_seed(3)
    shapes = [(3 * 2048 + 16,), (64, 72), (8,), (2048,), (40, 1000)]
    a = [nn.Parameter(torch.randn(s, generator=g).cuda().to(dtype)) for s in shapes]
    b = [nn.Parameter(x.detach().float().clone()) for x in a]
    opt = Muon([{"params": a, "algorithm": algorithm, "lr": 0.01, "wd": 0.1, "maximize": maximize}])
    cls = torch.optim.AdamW if algorithm == "adamw" else torch.optim.Adam
    ref = cls(b, lr=0.01, betas=(0.9, 0.95), weight_decay=0.1, maximize=maximize)
    n0 = _ext.launch_count
    for _ in range(4):
        for x, y in zip(a, b):
            gr = torch.randn(x.shape, generator=g).cuda()
            x.grad = gr.to(dtype)
            y.grad = x.grad.float().clone()
        opt.step()
        ref.step()
    assert _ext.launch_count - n0 == 4, "one native AdamW launch per step"
    tol = dict(rtol=1e-5, atol=1e-6) if dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)
    for x, y in zip(a, b):
        torch.testing.assert_close(x.detach().float(), y.detach(), **tol)
    _ext.check_device_errors("cuda")


@pytest.mark.parametrize("cls", [Muon8bit, Muon4bit, MuonFp8])
def test_lp_fused_cuda_matches_cpu_semantics(cls):
    """Fused quantised-momentum kernels on CUDA track the CPU implementation."""
    torch.manual_seed(0)
    cpu = nn.Parameter(torch.randn(64, 128))
    gpu = nn.Parameter(cpu.detach().clone().cuda())
    oc, og = cls([cpu], lr=0.02, block_size=512), cls([gpu], lr=0.02, block_size=512)
    n0 = _ext.launch_count
    for i in range(3):
        gr = torch.randn(64, 128, generator=torch.Generator().manual_seed(i))
        cpu.grad, gpu.grad = gr.clone(), gr.cuda()
        oc.step()
        og.step()
    assert _ext.launch_count > n0
    assert_close(gpu.cpu(), cpu, rtol=RTOL, atol=ATOL, max_mismatch_pct=PCT)
    mc = oc.state[cpu]["momentum_buffer"].dequantize()
    mg = og.state[gpu]["momentum_buffer"].dequantize().cpu()
    assert ((mc - mg).norm() / mc.norm()) < 0.05


def test_lp_quantize_kernel_matches_cpu():
    from dtensor_muon_b200.optim.optim_lp import FMT_4BIT, FMT_8BIT, FMT_FP8, QuantizedState

    torch.manual_seed(0)
    x = torch.randn(8192)
    for fmt in (FMT_FP8, FMT_8BIT, FMT_4BIT):
        qc = QuantizedState.zeros(x.shape, fmt, 1024, True, "cpu").copy_(x)
        qg = QuantizedState.zeros(x.shape, fmt, 1024, True, "cuda").copy_(x.cuda())
        torch.testing.assert_close(qg.scale.cpu(), qc.scale)
        same = (qg.codes.cpu() == qc.codes).float().mean().item()
        assert same > 0.999, (fmt, same)
        torch.testing.assert_close(qg.dequantize().cpu(), qc.dequantize(), rtol=0, atol=1e-6)


@pytest.mark.parametrize("n,block", [(8192, 2048), (16384, 4096), (4 * 1030, 1030), (8190, 1024)])
def test_lp_kernels_vector_and_generic_paths_match_cpu(n, block):
    """Vector path (block and n multiples of 8) and generic path (any block size)
    of the quantise / momentum-step kernels against the CPU formulation: the
    dynamic-tree codes (closed-form index on the GPU, search on the CPU) agree exactly."""
    from dtensor_muon_b200.optim.optim_lp import FMT_4BIT, FMT_8BIT, FMT_FP8, QuantizedState

    torch.manual_seed(1)
    x = torch.randn(n)
    g = torch.randn(n)
    for fmt in (FMT_FP8, FMT_8BIT, FMT_4BIT):
        qc = QuantizedState.zeros(x.shape, fmt, block, True, "cpu").copy_(x)
        qg = QuantizedState.zeros(x.shape, fmt, block, True, "cuda").copy_(x.cuda())
        torch.testing.assert_close(qg.scale.cpu(), qc.scale)
        if fmt != FMT_FP8:
            assert torch.equal(qg.codes.cpu(), qc.codes), fmt
        gout = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        _ext.load().lp_momentum_step(qg.codes, qg.scale, qg.qmap, qg.fmt, block, g.cuda(), gout, 0.9, True, False)
        m = qc.dequantize() * 0.9 + g
        torch.testing.assert_close(gout.float().cpu(), (m * 0.9 + g).bfloat16().float(), rtol=1e-2, atol=1e-6)
        qc.copy_(m)
        torch.testing.assert_close(qg.scale.cpu(), qc.scale)
        if fmt != FMT_FP8:
            agree = (qg.codes.cpu() == qc.codes).float().mean().item()
            assert agree > 0.999, (fmt, agree)


def test_cpu_offload_round_trip_matches_cuda():
    a = [nn.Parameter(t.detach().cpu()) for t in _params(3)]
    b = _params(3)
    oa = Muon(a, foreach=True, lr=0.1)
    ob = Muon(b, foreach=True, lr=0.1)
    g = torch.Generator().manual_seed(5)
    for _ in range(2):
        for x, y in zip(a, b):
            gr = torch.randn(x.shape, generator=g)
            x.grad, y.grad = gr.clone(), gr.cuda()
        oa.step()
        ob.step()
    for x, y in zip(a, b):
        assert x.device.type == "cpu"
        assert_close(x, y.cpu(), rtol=RTOL, atol=ATOL, max_mismatch_pct=PCT)


def test_muon_step_uses_native_kernels():
    a = _params(4)
    opt = Muon(a)
    n0 = _ext.launch_count
    _run(opt, a, steps=1)
    assert _ext.launch_count - n0 >= len(set(SHAPES)) * 15


def test_fused_adam_group_keeps_step_on_device_and_matches_torch():
    g = torch.Generator().manual_seed(0)
    a = [nn.Parameter(torch.randn(64, generator=g).cuda())]
    b = [nn.Parameter(a[0].detach().clone())]
    opt = Muon([{"params": a, "algorithm": "adamw", "fused": True, "lr": 0.01}])
    ref = torch.optim.AdamW(b, lr=0.01, weight_decay=0.1, betas=(0.9, 0.95), fused=True)
    for _ in range(2):
        gr = torch.randn(64, generator=g).cuda()
        a[0].grad, b[0].grad = gr.clone(), gr.clone()
        opt.step()
        ref.step()
    assert opt.state[a[0]]["step"].device == a[0].device
    torch.testing.assert_close(a[0], b[0])


@pytest.mark.parametrize("n", [4096, 4099])
def test_native_adamw_edge_values_match_torch(n):
    """Zero gradients, tiny gradients (subnormal second moment) and one huge
    gradient element (second moment overflows to +inf) on the vector (n % 8 == 0)
    and scalar paths: same results as torch.optim.AdamW, no NaN introduced."""
    g = torch.zeros(n)
    g[: n // 4] = 1e-20  # g^2 ~ 1e-40: subnormal fp32
    g[n // 4 : n // 2] = torch.randn(n // 2 - n // 4, generator=torch.Generator().manual_seed(4))
    g[7] = 1e20  # g^2 overflows to inf
    a = nn.Parameter(torch.randn(n, generator=torch.Generator().manual_seed(5)).cuda())
    b = nn.Parameter(a.detach().clone())
    opt = Muon([{"params": [a], "algorithm": "adamw", "lr": 0.01, "wd": 0.1}])
    ref = torch.optim.AdamW([b], lr=0.01, weight_decay=0.1, betas=(0.9, 0.95), foreach=False)
    for _ in range(2):
        a.grad, b.grad = g.cuda(), g.cuda()
        opt.step()
        ref.step()
    assert torch.isfinite(a).all()
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
    # subnormal second moments carry few significant bits: compare them absolutely
    torch.testing.assert_close(opt.state[a]["exp_avg_sq"], ref.state[b]["exp_avg_sq"], rtol=1e-5, atol=1e-38)
