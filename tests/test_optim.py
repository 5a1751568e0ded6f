"""Optimizer-shell behaviour on CPU (mirrors the reference's tests/optim/test_optim.py)."""

import math

import pytest
import torch

import dtensor_muon_b200.optim.algorithms.base as algo_base
from dtensor_muon_b200 import Muon
from dtensor_muon_b200.optim.algorithms import get_algorithm


def _identity_ortho(monkeypatch):
    monkeypatch.setattr(algo_base, "zeropower", lambda g, **_: g)
    monkeypatch.setattr(algo_base, "foreach_zeropower", lambda gs, **_: list(gs))


def test_step_goes_through_cached_impl():
    p = torch.nn.Parameter(torch.randn(2, 2))
    p.grad = torch.randn_like(p)
    opt = Muon([p])
    calls = []
    opt._muon_impls["muon"] = lambda *a, **k: calls.append((a, k))
    opt.step()
    assert len(calls) == 1 and calls[0][0][0] == [p]


@pytest.mark.parametrize(
    "kwargs,match",
    [
        ({"lr": -1.0}, "Invalid learning rate"),
        ({"adam_eps": -1.0}, "Invalid epsilon value"),
        ({"adam_betas": (1.0, 0.9)}, "Invalid beta parameter at index 0"),
        ({"adam_betas": (0.9, -0.1)}, "Invalid beta parameter at index 1"),
    ],
)
def test_constructor_validates_scalars(kwargs, match):
    with pytest.raises(ValueError, match=match):
        Muon([torch.nn.Parameter(torch.randn(2, 2))], **kwargs)


def test_constructor_rejects_bad_param_containers():
    p = torch.nn.Parameter(torch.randn(2, 2))
    with pytest.raises(TypeError, match="not a single dict"):
        Muon({"params": [p]})
    with pytest.raises(ValueError, match="empty parameter list"):
        Muon([])
    with pytest.raises(ValueError, match="'params' key"):
        Muon([{"lr": 0.1}])


def test_constructor_skips_empty_groups():
    p = torch.nn.Parameter(torch.randn(2, 2))
    opt = Muon([{"params": []}, {"params": [p]}])
    assert len(opt.param_groups) == 1


def test_constructor_rejects_unknown_algorithm_and_bad_params():
    p = torch.nn.Parameter(torch.randn(2, 2))
    with pytest.raises(ValueError, match="Unknown algorithm"):
        Muon([{"params": [p], "algorithm": "sgd"}])
    with pytest.raises(ValueError, match="2D\\+"):
        Muon([torch.nn.Parameter(torch.randn(3))])
    with pytest.raises(NotImplementedError, match="Complex parameters"):
        Muon([torch.nn.Parameter(torch.randn(2, 2, dtype=torch.complex64))])


def test_group_normalization_keys_and_types():
    w = torch.nn.Parameter(torch.randn(4, 4))
    b = torch.nn.Parameter(torch.randn(4))
    opt = Muon([{"params": [w], "lr": 0.5}, {"params": [b], "algorithm": "AdamW", "lr": 0.01}], wd=0.2)
    g0, g1 = opt.param_groups
    assert g0["algorithm"] == "muon" and g0["use_muon"] is True
    assert torch.is_tensor(g0["lr"]) and g0["lr"].ndim == 0 and float(g0["lr"]) == 0.5
    assert g0["foreach"] is False  # CPU params resolve foreach=None -> False
    assert g0["orthogonalization_strategy"] == "polar_express"
    assert g1["algorithm"] == "adamw" and g1["use_muon"] is False
    assert g1["decoupled_weight_decay"] is True and g1["wd"] == 0.2
    assert g1["has_complex"] is False
    adam = Muon([{"params": [b], "algorithm": "adam"}])
    assert adam.param_groups[0]["decoupled_weight_decay"] is False


def test_3d_muon_and_complex_adam_allowed():
    w = torch.nn.Parameter(torch.randn(2, 3, 4))
    c = torch.nn.Parameter(torch.randn(3, dtype=torch.complex64))
    opt = Muon([{"params": [w]}, {"params": [c], "algorithm": "adamw"}])
    assert opt.param_groups[1]["has_complex"] is True


def _steps(opt, params, refs, ref_opt, n=3, seed=0):
    gen = torch.Generator().manual_seed(seed)
    for _ in range(n):
        for p, r in zip(params, refs):
            g = torch.randn(p.shape, generator=gen, dtype=p.dtype)
            p.grad = g.clone()
            r.grad = g.clone()
        opt.step()
        ref_opt.step()


@pytest.mark.parametrize("amsgrad", [False, True])
def test_adamw_group_matches_torch(amsgrad):
    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(5, 3)), torch.nn.Parameter(torch.randn(7))]
    refs = [torch.nn.Parameter(p.detach().clone()) for p in params]
    opt = Muon([{"params": params, "algorithm": "adamw", "lr": 0.01, "wd": 0.1, "amsgrad": amsgrad}])
    ref = torch.optim.AdamW(refs, lr=0.01, weight_decay=0.1, betas=(0.9, 0.95), amsgrad=amsgrad)
    _steps(opt, params, refs, ref)
    for p, r in zip(params, refs):
        torch.testing.assert_close(p, r)


def test_adam_coupled_weight_decay_matches_torch():
    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(4, 4))]
    refs = [torch.nn.Parameter(params[0].detach().clone())]
    opt = Muon([{"params": params, "algorithm": "adam", "lr": 0.01, "wd": 0.1}])
    ref = torch.optim.Adam(refs, lr=0.01, weight_decay=0.1, betas=(0.9, 0.95))
    _steps(opt, params, refs, ref)
    torch.testing.assert_close(params[0], refs[0])


def test_complex_adam_steps():
    p = torch.nn.Parameter(torch.randn(3, dtype=torch.complex64))
    before = p.detach().clone()
    opt = Muon([{"params": [p], "algorithm": "adamw"}])
    p.grad = torch.randn_like(p)
    opt.step()
    assert not torch.equal(p.detach(), before)


def test_step_returns_closure_loss():
    p = torch.nn.Parameter(torch.randn(2, 2))
    opt = Muon([p])

    def closure():
        loss = (p**2).sum()
        loss.backward()
        return loss

    loss = opt.step(closure)
    assert torch.is_tensor(loss)


def test_state_init_and_shape_lr_ratio(monkeypatch):
    _identity_ortho(monkeypatch)
    p = torch.nn.Parameter(torch.zeros(8, 2))
    opt = Muon([p], lr=0.1, wd=0.0, momentum=0.0, nesterov=False)
    p.grad = torch.ones_like(p)
    opt.step()
    st = opt.state[p]
    assert float(st["step"]) == 1.0 and st["step"].device.type == "cpu"
    assert math.isclose(float(st["lr_ratio"]), 2.0)
    assert st["momentum_buffer"].dtype == torch.float32
    torch.testing.assert_close(p.detach(), torch.full_like(p, -0.2))


def test_nesterov_uses_updated_buffer(monkeypatch):
    _identity_ortho(monkeypatch)
    p = torch.nn.Parameter(torch.zeros(2, 2))
    opt = Muon([p], lr=1.0, wd=0.0, momentum=0.5, nesterov=True)
    for _ in range(2):
        p.grad = torch.ones_like(p)
        opt.step()
    # step 1: buf=1, g'=1.5 ; step 2: buf=1.5, g'=1.75 -> p = -(1.5 + 1.75)
    torch.testing.assert_close(p.detach(), torch.full_like(p, -3.25))


def test_cautious_weight_decay_masks_by_sign(monkeypatch):
    _identity_ortho(monkeypatch)
    p = torch.nn.Parameter(torch.tensor([[1.0, -1.0], [2.0, -2.0]]))
    opt = Muon([p], lr=1.0, wd=0.5, momentum=0.0, nesterov=False, use_cautious_wd=True)
    p.grad = torch.tensor([[1.0, 1.0], [-1.0, -1.0]])
    opt.step()
    # u*p > 0 at (0,0) and (1,1): u += 0.5 p there
    expected = torch.tensor([[1.0 - 1.5, -1.0 - 1.0], [2.0 + 1.0, -2.0 + 2.0]])
    torch.testing.assert_close(p.detach(), expected)


def test_plain_weight_decay_everywhere(monkeypatch):
    _identity_ortho(monkeypatch)
    p = torch.nn.Parameter(torch.tensor([[1.0, -1.0], [2.0, -2.0]]))
    opt = Muon([p], lr=1.0, wd=0.5, momentum=0.0, nesterov=False, use_cautious_wd=False)
    p.grad = torch.tensor([[1.0, 1.0], [-1.0, -1.0]])
    opt.step()
    expected = torch.tensor([[1.0 - 1.5, -1.0 - 0.5], [2.0 + 1.0 - 1.0, -2.0 + 1.0 + 1.0]])
    torch.testing.assert_close(p.detach(), expected)


def test_maximize_ascends(monkeypatch):
    _identity_ortho(monkeypatch)
    p = torch.nn.Parameter(torch.zeros(2, 2))
    opt = Muon([p], lr=1.0, wd=0.0, momentum=0.0, nesterov=False, maximize=True)
    g = torch.ones_like(p)
    p.grad = g
    opt.step()
    torch.testing.assert_close(p.detach(), torch.ones_like(p))
    torch.testing.assert_close(g, torch.ones_like(p))  # grad itself untouched
    opt.step()  # reusing the same grad keeps ascending
    torch.testing.assert_close(p.detach(), torch.full_like(p, 2.0))


def test_fp32_momentum_for_bf16_params(monkeypatch):
    _identity_ortho(monkeypatch)
    p = torch.nn.Parameter(torch.zeros(4, 4, dtype=torch.bfloat16))
    opt = Muon([p])
    p.grad = torch.ones_like(p)
    opt.step()
    assert opt.state[p]["momentum_buffer"].dtype == torch.float32
    assert p.dtype == torch.bfloat16


def test_params_without_grad_are_skipped(monkeypatch):
    _identity_ortho(monkeypatch)
    a = torch.nn.Parameter(torch.zeros(2, 2))
    b = torch.nn.Parameter(torch.zeros(2, 2))
    opt = Muon([a, b], wd=0.0)
    a.grad = torch.ones_like(a)
    opt.step()
    assert len(opt.state[a]) > 0 and len(opt.state[b]) == 0
    assert torch.equal(b.detach(), torch.zeros(2, 2))


def test_flatten_true_collapses_to_matrix(monkeypatch):
    seen = []

    def rec(g, **_):
        seen.append(tuple(g.shape))
        return g

    monkeypatch.setattr(algo_base, "zeropower", rec)
    p = torch.nn.Parameter(torch.zeros(4, 3, 2, 2))
    opt = Muon([{"params": [p], "flatten": True}], wd=0.0)
    p.grad = torch.ones_like(p)
    opt.step()
    assert seen == [(4, 12)]
    assert opt.state[p]["momentum_buffer"].shape == (4, 12)
    assert math.isclose(float(opt.state[p]["lr_ratio"]), 1.0)


def test_flatten_false_batches_leading_dims(monkeypatch):
    seen = []

    def rec(g, **_):
        seen.append(tuple(g.shape))
        return g

    monkeypatch.setattr(algo_base, "zeropower", rec)
    p4 = torch.nn.Parameter(torch.zeros(2, 3, 8, 2))
    p3 = torch.nn.Parameter(torch.zeros(5, 8, 2))
    opt = Muon([p4, p3], wd=0.0)
    p4.grad = torch.ones_like(p4)
    p3.grad = torch.ones_like(p3)
    opt.step()
    assert seen == [(6, 8, 2), (5, 8, 2)]
    assert opt.state[p4]["momentum_buffer"].shape == (6, 8, 2)
    assert math.isclose(float(opt.state[p3]["lr_ratio"]), 2.0)


def test_load_state_dict_applies_legacy_defaults():
    p = torch.nn.Parameter(torch.randn(4, 4))
    opt = Muon([p])
    p.grad = torch.randn_like(p)
    opt.step()
    sd = opt.state_dict()
    g = sd["param_groups"][0]
    for k in ("algorithm", "ns_steps", "nesterov", "flatten", "use_cautious_wd", "orthogonalization_strategy",
              "split_sizes", "foreach"):
        g.pop(k)
    g["lr"] = 0.02
    sd["state"][0]["step"] = 3.0
    opt2 = Muon([torch.nn.Parameter(p.detach().clone())])
    opt2.load_state_dict(sd)
    g2 = opt2.param_groups[0]
    assert g2["algorithm"] == "muon" and g2["ns_steps"] == 5 and g2["nesterov"] is True
    assert g2["flatten"] is False and g2["use_cautious_wd"] is True
    assert g2["orthogonalization_strategy"] == "polar_express" and g2["split_sizes"] is None
    assert g2["foreach"] is False
    assert torch.is_tensor(g2["lr"]) and math.isclose(float(g2["lr"]), 0.02, rel_tol=1e-6)
    st = opt2.state[opt2.param_groups[0]["params"][0]]
    assert torch.is_tensor(st["step"]) and float(st["step"]) == 3.0


def test_load_state_dict_adam_legacy_defaults():
    p = torch.nn.Parameter(torch.randn(4))
    opt = Muon([{"params": [p], "algorithm": "adamw"}])
    p.grad = torch.randn_like(p)
    opt.step()
    sd = opt.state_dict()
    g = sd["param_groups"][0]
    for k in ("amsgrad", "maximize", "foreach", "decoupled_weight_decay", "fused"):
        g.pop(k)
    g["wd"] = torch.tensor(0.3)
    sd["state"][0]["step"] = 2.0
    opt2 = Muon([{"params": [torch.nn.Parameter(p.detach().clone())], "algorithm": "adamw"}])
    opt2.load_state_dict(sd)
    g2 = opt2.param_groups[0]
    assert g2["amsgrad"] is False and g2["decoupled_weight_decay"] is False and g2["fused"] is None
    assert isinstance(g2["wd"], float)
    st = opt2.state[opt2.param_groups[0]["params"][0]]
    assert torch.is_tensor(st["step"]) and float(st["step"]) == 2.0


def test_setstate_resets_impl_cache():
    p = torch.nn.Parameter(torch.randn(2, 2))
    opt = Muon([p])
    opt._muon_impls["muon"] = object()
    opt.load_state_dict(opt.state_dict())
    assert opt._muon_impls == {}


def test_state_dict_round_trip_continues_training():
    torch.manual_seed(0)
    a = torch.nn.Parameter(torch.randn(6, 4))
    b = torch.nn.Parameter(a.detach().clone())
    oa = Muon([a], lr=0.05)
    ob = Muon([b], lr=0.05)
    gen = torch.Generator().manual_seed(1)
    grads = [torch.randn(6, 4, generator=gen) for _ in range(4)]
    for g in grads[:2]:
        a.grad = g.clone()
        oa.step()
        b.grad = g.clone()
        ob.step()
    sd = ob.state_dict()
    c = torch.nn.Parameter(b.detach().clone())
    oc = Muon([c], lr=0.05)
    oc.load_state_dict(sd)
    for g in grads[2:]:
        a.grad = g.clone()
        oa.step()
        c.grad = g.clone()
        oc.step()
    torch.testing.assert_close(a, c)


def test_mixed_muon_and_adam_groups(monkeypatch):
    _identity_ortho(monkeypatch)
    w = torch.nn.Parameter(torch.randn(4, 4))
    b = torch.nn.Parameter(torch.randn(4))
    opt = Muon([{"params": [w]}, {"params": [b], "algorithm": "adamw"}])
    w0, b0 = w.detach().clone(), b.detach().clone()
    w.grad = torch.randn_like(w)
    b.grad = torch.randn_like(b)
    opt.step()
    assert not torch.equal(w0, w.detach()) and not torch.equal(b0, b.detach())
    assert set(opt.state[b]) == {"step", "exp_avg", "exp_avg_sq"}


def test_get_algorithm_is_case_insensitive():
    assert get_algorithm("MUON").name == "muon"


def test_outer_torch_compile_of_step_matches_eager(monkeypatch):
    """An outer torch.compile around step() runs the same update (graph breaks allowed)."""
    _identity_ortho(monkeypatch)
    p = torch.nn.Parameter(torch.ones(4, 2))
    ref = torch.nn.Parameter(p.detach().clone())
    opt = Muon([p], lr=0.1, wd=0.0, momentum=0.0, nesterov=False)
    ref_opt = Muon([ref], lr=0.1, wd=0.0, momentum=0.0, nesterov=False)
    compiled = torch.compile(opt.step, backend="eager")
    for value in (0.5, 0.25):
        p.grad = torch.full_like(p, value)
        ref.grad = torch.full_like(ref, value)
        compiled()
        ref_opt.step()
    torch.testing.assert_close(p, ref)
    torch.testing.assert_close(opt.state[p]["momentum_buffer"], ref_opt.state[ref]["momentum_buffer"])
