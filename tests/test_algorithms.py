"""Registry, custom algorithms, NorMuon math and split_sizes on CPU
(mirrors the reference's tests/optim/test_algorithms.py)."""

import math

import pytest
import torch
import torch.nn as nn

import dtensor_muon_b200.optim.algorithms.base as algo_base
from dtensor_muon_b200 import (
    BufferSpec,
    Muon,
    MuonAlgorithm,
    get_algorithm,
    register_muon_algorithm,
    registered_algorithms,
)
from dtensor_muon_b200.optim.algorithms import split_lr_scales


def _identity(monkeypatch):
    monkeypatch.setattr(algo_base, "zeropower", lambda g, **_: g)
    monkeypatch.setattr(algo_base, "foreach_zeropower", lambda gs, **_: list(gs))


@register_muon_algorithm
class _SignStep(MuonAlgorithm):
    """Third-party style algorithm: sign of the raw gradient, no orthogonalisation."""

    name = "test-sign-step"
    options = {"scale": 1.0}

    def update(self, param, grad, state, lr_ratio, *, lr, scale, **kwargs):
        state["momentum_buffer"].copy_(grad)
        param.copy_(param - lr * scale * grad.sign())


def test_builtins_registered():
    names = registered_algorithms()
    assert "muon" in names and "normuon" in names and names == tuple(sorted(names))


def test_unknown_algorithm_message_lists_names():
    with pytest.raises(ValueError, match="Unknown algorithm 'nope'.*muon"):
        get_algorithm("nope")


def test_register_rejects_reserved_duplicates_and_shadowing():
    class AdamNamed(MuonAlgorithm):
        name = "AdamW"

        def update(self, *a, **k):
            pass

    with pytest.raises(ValueError, match="reserved for the Adam path"):
        register_muon_algorithm(AdamNamed)

    class Dup(MuonAlgorithm):
        name = "muon"

        def update(self, *a, **k):
            pass

    with pytest.raises(ValueError, match="already registered"):
        register_muon_algorithm(Dup)

    class Shadow(MuonAlgorithm):
        name = "test-shadow"
        options = {"lr": 1.0}

        def update(self, *a, **k):
            pass

    with pytest.raises(ValueError, match="reserved group keys"):
        register_muon_algorithm(Shadow)

    class Nameless(MuonAlgorithm):
        name = ""

        def update(self, *a, **k):
            pass

    with pytest.raises(ValueError, match="non-empty string"):
        register_muon_algorithm(Nameless)


def test_reregistering_same_class_is_allowed():
    register_muon_algorithm(_SignStep)
    assert isinstance(get_algorithm("TEST-SIGN-STEP"), _SignStep)


def test_custom_algorithm_steps_and_option_default():
    p = nn.Parameter(torch.zeros(3, 3))
    opt = Muon([{"params": [p], "algorithm": "test-sign-step", "scale": 2.0}], lr=0.5)
    assert opt.param_groups[0]["scale"] == 2.0
    p.grad = torch.tensor([[1.0, -1.0, 0.0]] * 3)
    opt.step()
    torch.testing.assert_close(p.detach(), torch.tensor([[-1.0, 1.0, 0.0]] * 3))
    q = nn.Parameter(torch.zeros(2, 2))
    opt2 = Muon([{"params": [q], "algorithm": "test-sign-step"}])
    assert opt2.param_groups[0]["scale"] == 1.0
    assert opt2.state_dict()["param_groups"][0]["algorithm"] == "test-sign-step"


def _normuon_ref(p, g, buf, v, *, lr, wd, momentum, beta2):
    buf.mul_(momentum).add_(g)
    u = g + momentum * buf
    fro = u.norm(dim=(-2, -1), keepdim=True)
    v.lerp_((u * u).mean(dim=-1, keepdim=True), 1 - beta2)
    u = u / (v.sqrt() + 1e-8)
    u = u * (fro / u.norm(dim=(-2, -1), keepdim=True).clamp(min=1e-8))
    u = u + wd * p * (u * p > 0)
    p.sub_(math.sqrt(max(1.0, p.shape[-2] / p.shape[-1])) * lr * u)


@pytest.mark.parametrize("shape", [(4, 3), (3, 4), (2, 3, 4)])
def test_normuon_matches_transcription(monkeypatch, shape):
    _identity(monkeypatch)
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(shape))
    rp, rb, rv = p.detach().clone(), torch.zeros(shape), torch.zeros(*shape[:-1], 1)
    opt = Muon([{"params": [p], "algorithm": "normuon", "muon_beta2": 0.9}], lr=0.1, wd=0.1, momentum=0.5)
    for step in range(3):
        g = torch.randn(shape, generator=torch.Generator().manual_seed(100 + step))
        p.grad = g.clone()
        opt.step()
        _normuon_ref(rp, g.clone(), rb, rv, lr=0.1, wd=0.1, momentum=0.5, beta2=0.9)
    torch.testing.assert_close(p.detach(), rp, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(opt.state[p]["variance_neuron"], rv, rtol=1e-5, atol=1e-7)


def test_normuon_state_spec_and_buffers():
    assert get_algorithm("normuon").state_spec["variance_neuron"] == BufferSpec(like="grad_rows", signed=False)
    p = nn.Parameter(torch.randn(6, 4))
    opt = Muon([{"params": [p], "algorithm": "normuon"}])
    p.grad = torch.randn_like(p)
    opt.step()
    assert opt.state[p]["variance_neuron"].shape == (6, 1)
    assert opt.param_groups[0]["muon_beta2"] == 0.95


def test_normuon_foreach_path_matches_per_param(monkeypatch):
    """The torch foreach formulation (CPU tensors forced through it) equals the per-param one."""
    _identity(monkeypatch)
    torch.manual_seed(0)
    shapes = [(4, 6), (4, 6), (5, 3)]
    a = [nn.Parameter(torch.randn(s)) for s in shapes]
    b = [nn.Parameter(t.detach().clone()) for t in a]
    oa = Muon([{"params": a, "algorithm": "normuon"}], foreach=False, lr=0.1)
    ob = Muon([{"params": b, "algorithm": "normuon"}], foreach=False, lr=0.1)
    alg = get_algorithm("normuon")
    for _ in range(2):
        grads = [torch.randn(s) for s in shapes]
        for p, g in zip(a, grads):
            p.grad = g.clone()
        oa.step()
        for p, g in zip(b, grads):
            p.grad = g.clone()
        # drive the batched formulation directly, per same-shape batch
        params, grads_, state = [], [], {"momentum_buffer": [], "variance_neuron": []}
        ratios = []
        for p in b:
            st = ob.state[p]
            if not st:
                st["step"] = torch.tensor(0.0)
                st["momentum_buffer"] = torch.zeros_like(p)
                st["variance_neuron"] = torch.zeros(p.shape[0], 1)
                st["lr_ratio"] = torch.tensor(math.sqrt(max(1.0, p.shape[0] / p.shape[1])))
            params.append(p)
            grads_.append(p.grad)
            state["momentum_buffer"].append(st["momentum_buffer"])
            state["variance_neuron"].append(st["variance_neuron"])
            ratios.append(st["lr_ratio"])
        for idx in ([0, 1], [2]):
            with torch.no_grad():
                alg.foreach_update(
                    [params[i] for i in idx], [grads_[i] for i in idx],
                    {k: [v[i] for i in idx] for k, v in state.items()}, [ratios[i] for i in idx],
                    lr=torch.tensor(0.1), weight_decay=0.1, cautious_wd=True, momentum=0.95, nesterov=True,
                    maximize=False, ns_steps=5, orthogonalization_strategy="polar_express", split_sizes=None,
                    muon_beta2=0.95,
                )
    for p, q in zip(a, b):
        torch.testing.assert_close(p.detach(), q.detach(), rtol=1e-5, atol=1e-6)


def test_split_sizes_validation():
    p = nn.Parameter(torch.randn(6, 4))
    for bad, match in [
        ((6,), "at least 2 block sizes"),
        ((3, 0, 3), "positive integers"),
        ((3, True, 2), "positive integers"),
        ((3, 2), "must sum to dim 0"),
    ]:
        with pytest.raises(ValueError, match=match):
            Muon([{"params": [p], "split_sizes": bad}])
    with pytest.raises(ValueError, match="only supported for 2D"):
        Muon([{"params": [nn.Parameter(torch.randn(2, 3, 4))], "split_sizes": (1, 1)}])
    opt = Muon([{"params": [p], "split_sizes": [2, 4]}])
    assert opt.param_groups[0]["split_sizes"] == (2, 4)


def test_split_lr_scales_rule():
    scales = split_lr_scales((12, 2), (8, 2, 2))
    full = math.sqrt(6.0)
    assert scales == pytest.approx((2.0 / full, 1.0 / full, 1.0 / full))


def test_split_sizes_orthogonalizes_blocks_independently(monkeypatch):
    seen = []

    def rec(gs, **_):
        seen.append([tuple(g.shape) for g in gs])
        return [torch.full_like(g, float(g.shape[0])) for g in gs]

    monkeypatch.setattr(algo_base, "foreach_zeropower", rec)
    p = nn.Parameter(torch.zeros(8, 4))
    opt = Muon([{"params": [p], "split_sizes": (4, 2, 2)}], lr=1.0, wd=0.0, momentum=0.0, nesterov=False)
    p.grad = torch.ones_like(p)
    opt.step()
    assert sorted(map(sorted, seen)) == [[(2, 4), (2, 4)], [(4, 4)]]
    full = math.sqrt(2.0)
    expected = torch.cat([torch.full((4, 4), -4.0 * 1.0), torch.full((4, 4), -2.0 * 1.0)]) / full * full
    torch.testing.assert_close(p.detach(), expected)


def test_normuon_split_sizes_normalizes_per_block(monkeypatch):
    _identity(monkeypatch)
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(6, 4))
    opt = Muon([{"params": [p], "algorithm": "normuon", "split_sizes": (4, 2)}], lr=0.1, wd=0.0)
    p.grad = torch.randn_like(p)
    opt.step()
    v = opt.state[p]["variance_neuron"]
    assert v.shape == (6, 1) and torch.all(v > 0)


def test_legacy_checkpoint_without_algorithm_loads_as_muon():
    p = nn.Parameter(torch.randn(4, 4))
    opt = Muon([p])
    p.grad = torch.randn_like(p)
    opt.step()
    sd = opt.state_dict()
    del sd["param_groups"][0]["algorithm"]
    opt2 = Muon([nn.Parameter(p.detach().clone())])
    opt2.load_state_dict(sd)
    assert opt2.param_groups[0]["algorithm"] == "muon"


def test_checkpoint_with_unregistered_algorithm_raises():
    p = nn.Parameter(torch.randn(4, 4))
    opt = Muon([p])
    sd = opt.state_dict()
    sd["param_groups"][0]["algorithm"] = "not-registered"
    with pytest.raises(ValueError, match="Unknown algorithm"):
        Muon([nn.Parameter(p.detach().clone())]).load_state_dict(sd)


def test_normuon_round_trip_continues_training():
    torch.manual_seed(0)
    a = nn.Parameter(torch.randn(6, 4))
    b = nn.Parameter(a.detach().clone())
    kw = dict(lr=0.05)
    oa = Muon([{"params": [a], "algorithm": "normuon"}], **kw)
    ob = Muon([{"params": [b], "algorithm": "normuon"}], **kw)
    grads = [torch.randn(6, 4, generator=torch.Generator().manual_seed(i)) for i in range(4)]
    for g in grads[:2]:
        a.grad, b.grad = g.clone(), g.clone()
        oa.step()
        ob.step()
    c = nn.Parameter(b.detach().clone())
    oc = Muon([{"params": [c], "algorithm": "normuon"}], **kw)
    oc.load_state_dict(ob.state_dict())
    for g in grads[2:]:
        a.grad, c.grad = g.clone(), g.clone()
        oa.step()
        oc.step()
    torch.testing.assert_close(a, c)


def test_split_sizes_batch_groups_blocks_across_matrices(monkeypatch):
    """Three fused weights with blocks (4, 2, 2): one engine call per block height
    for the whole batch (3 blocks of height 4, 6 of height 2), not one per matrix."""
    calls = []

    def rec(gs, **_):
        calls.append(len(gs))
        return [torch.full_like(g, float(g.shape[0])).bfloat16() for g in gs]

    monkeypatch.setattr(algo_base, "foreach_zeropower", rec)
    gs = [torch.randn(8, 4) for _ in range(3)]
    outs = algo_base.orthogonalize_batch(gs, ns_steps=5, strategy="polar_express", split_sizes=(4, 2, 2))
    assert sorted(calls) == [3, 6]
    scales = split_lr_scales((8, 4), (4, 2, 2))
    for u in outs:
        assert u.dtype == torch.bfloat16 and u.shape == (8, 4)
        torch.testing.assert_close(u[:4].float(), torch.full((4, 4), 4.0 * scales[0]).bfloat16().float())
        torch.testing.assert_close(u[4:].float(), torch.full((4, 4), 2.0 * scales[1]).bfloat16().float())


def _split_dtensor_worker(rank, world):
    import torch
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import DTensor, Shard, distribute_tensor

    from dtensor_muon_b200.optim.algorithms import base

    mesh = init_device_mesh("cpu", (world,))
    torch.manual_seed(11)
    fulls = [torch.randn(12, 8) for _ in range(3)]
    ds = [distribute_tensor(f, mesh, [Shard(0)]) for f in fulls]
    split = (8, 2, 2)
    got = base.orthogonalize_batch(ds, ns_steps=5, strategy="newton_schulz", split_sizes=split)
    want = base.orthogonalize_batch(fulls, ns_steps=5, strategy="newton_schulz", split_sizes=split)
    for g, w in zip(got, want):
        assert isinstance(g, DTensor) and list(g.placements) == [Shard(0)]
        torch.testing.assert_close(g.full_tensor().float(), w.float())
    one = base.orthogonalize_single(ds[0], ns_steps=5, strategy="newton_schulz", split_sizes=split)
    torch.testing.assert_close(one.full_tensor().float(), want[0].float())


def test_split_sizes_dtensor_batch_gloo():
    from dtensor_muon_b200.testing.distributed import run_distributed

    run_distributed(_split_dtensor_worker, 2)
