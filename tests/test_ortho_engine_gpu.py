"""Numerics of the tcgen05 orthogonalisation engine against fp32 PyTorch."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from dtensor_muon_b200.ops import _ext, ortho
from dtensor_muon_b200.orthogonalize.newton_schulz import ns_loop
from dtensor_muon_b200.orthogonalize.polar_express import pe_loop


def _close_frac(a, b, rtol, atol):
    return (~torch.isclose(a.float(), b.float(), rtol=rtol, atol=atol)).float().mean().item()


@pytest.mark.parametrize("shape", [(1, 256, 256), (2, 300, 520), (3, 512, 1024), (1, 1024, 4096), (2, 96, 40)])
def test_gram_matches_fp32(shape):
    torch.manual_seed(0)
    x = torch.randn(*shape, device="cuda").bfloat16()
    y = ortho.gram(x)
    ref = x.float() @ x.float().mT
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2 * shape[-1] ** 0.5)
    assert torch.equal(y, y.mT), "gram output must be exactly symmetric"
    _ext.check_device_errors("cuda")


@pytest.mark.parametrize("B,N,M", [(1, 256, 256), (2, 256, 768), (3, 512, 1024)])
def test_gemm_ax_matches_fp32(B, N, M):
    torch.manual_seed(1)
    C = _ext.load()
    a = torch.randn(B, N, N, device="cuda").bfloat16()
    x = torch.randn(B, N, M, device="cuda").bfloat16()
    res = torch.randn(B, N, M, device="cuda").bfloat16()
    out = torch.empty_like(x)
    C.gemm_ax(a, x, out, res, None, 0.5, -1.5, 0, 0, 0)
    ref = 0.5 * (a.float() @ x.float()) - 1.5 * res.float()
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=3e-2 * N**0.5)
    _ext.check_device_errors("cuda")


def test_gram_poly_epilogue():
    torch.manual_seed(2)
    C = _ext.load()
    x = torch.randn(2, 512, 512, device="cuda")
    a = (x @ x.mT / 512).bfloat16()  # symmetric
    out = torch.empty_like(a)
    C.gram_sym(a, out, a, None, 2.0, -3.0, 0, 0, 0)
    ref = 2.0 * (a.float() @ a.float()) - 3.0 * a.float()
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=5e-2)


@pytest.mark.parametrize("strategy", ["newton_schulz", "polar_express"])
@pytest.mark.parametrize("shape", [(4, 256, 256), (2, 384, 200), (2, 200, 384), (1, 1024, 3072), (3, 17, 33)])
def test_orthogonalize_matches_torch(strategy, shape):
    torch.manual_seed(3)
    g = torch.randn(*shape, device="cuda")
    got = torch.stack(ortho.orthogonalize_native(list(g.unbind(0)), 5, strategy, 1e-7))
    loop = ns_loop if strategy == "newton_schulz" else pe_loop
    ref = loop(g.double(), 5, eps=1e-7).float()
    assert got.dtype == torch.bfloat16 and got.shape == g.shape
    # bf16 iteration vs fp64: the reference's own triton-vs-eager budget.
    frac = _close_frac(got, ref, rtol=1e-2, atol=5e-2)
    assert frac < 0.02, frac
    _ext.check_device_errors("cuda")


def test_orthogonalize_steps0_is_normalized_input():
    g = torch.randn(2, 64, 128, device="cuda")
    got = torch.stack(ortho.orthogonalize_native(list(g.unbind(0)), 0, "newton_schulz", 1e-7))
    ref = g / (g.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    torch.testing.assert_close(got.float(), ref, rtol=1e-2, atol=1e-3)


# ---- 2-SM (cta_group::2) kernels ------------------------------------------
@pytest.mark.parametrize("shape", [(1, 256, 256), (2, 512, 768), (3, 1024, 2048)])
def test_gram2_matches_fp32(shape):
    torch.manual_seed(5)
    C = _ext.load()
    x = torch.randn(*shape, device="cuda").bfloat16()
    out = torch.empty(shape[0], shape[1], shape[1], device="cuda", dtype=torch.bfloat16)
    C.gram_sym2(x, out, None, None, 1.0, 0.0, 0, 0)
    ref = x.float() @ x.float().mT
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2 * shape[-1] ** 0.5)
    assert torch.equal(out, out.mT)
    _ext.check_device_errors("cuda")


@pytest.mark.parametrize("B,N,M", [(1, 256, 256), (2, 512, 768), (2, 1024, 2048)])
def test_gemm_ax2_matches_fp32(B, N, M):
    torch.manual_seed(6)
    C = _ext.load()
    a = torch.randn(B, N, N, device="cuda").bfloat16()
    x = torch.randn(B, N, M, device="cuda").bfloat16()
    out = torch.empty_like(x)
    C.gemm_ax2(a, x, out, x, None, 0.5, -1.5, 0, 0)
    ref = 0.5 * (a.float() @ x.float()) - 1.5 * x.float()
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=3e-2 * N**0.5)
    _ext.check_device_errors("cuda")


@pytest.mark.parametrize("strategy", ["newton_schulz", "polar_express"])
def test_orthogonalize_2sm_matches_1sm(strategy):
    C = _ext.load()
    torch.manual_seed(7)
    g = torch.randn(3, 384, 1000, device="cuda")
    prev = C.get_gemm_variant()
    try:
        C.set_gemm_variant(0)
        one = torch.stack(ortho.orthogonalize_native(list(g.unbind(0)), 5, strategy, 1e-7))
        C.set_gemm_variant(1)
        two = torch.stack(ortho.orthogonalize_native(list(g.unbind(0)), 5, strategy, 1e-7))
    finally:
        C.set_gemm_variant(prev)
    assert _close_frac(two, one, rtol=1e-2, atol=3e-2) < 0.01
    _ext.check_device_errors("cuda")


# ---- contracts, determinism, degenerate inputs (mirrors tests/kernels/test_gram.py) ----
def test_orthogonalize_is_deterministic():
    torch.manual_seed(8)
    g = list(torch.randn(3, 300, 700, device="cuda").unbind(0))
    a = torch.stack(ortho.orthogonalize_native(g, 5, "polar_express"))
    b = torch.stack(ortho.orthogonalize_native(g, 5, "polar_express"))
    assert torch.equal(a, b)
    x = torch.randn(2, 512, 1024, device="cuda").bfloat16()
    assert torch.equal(ortho.gram(x), ortho.gram(x))


def test_non_contiguous_and_transposed_inputs():
    from dtensor_muon_b200.orthogonalize import foreach_zeropower, zeropower

    torch.manual_seed(9)
    base = torch.randn(2, 512, 384, device="cuda")
    views = [base[i].mT for i in range(2)]  # non-contiguous [384, 512]
    got = foreach_zeropower(views, steps=5, strategy="newton_schulz")
    ref = foreach_zeropower([v.contiguous() for v in views], steps=5, strategy="newton_schulz")
    for a, b in zip(got, ref):
        assert a.shape == (384, 512) and torch.equal(a, b)
    one = zeropower(base[0][:, ::2], steps=5)  # strided columns
    assert one.shape == (512, 192) and torch.isfinite(one.float()).all()


def test_zero_and_rank_one_inputs_stay_finite():
    z = torch.zeros(2, 256, 512, device="cuda")
    out = torch.stack(ortho.orthogonalize_native(list(z.unbind(0)), 5, "polar_express"))
    assert torch.isfinite(out.float()).all() and out.abs().max() == 0
    r = torch.randn(256, 1, device="cuda") @ torch.randn(1, 512, device="cuda")
    out = ortho.orthogonalize_native([r], 5, "newton_schulz")[0]
    assert torch.isfinite(out.float()).all()
    assert ortho.orthogonalize_native([], 5, "newton_schulz") == []


def test_engine_contracts_raise():
    C = _ext.load()
    x = torch.randn(1, 256, 256, device="cuda")  # fp32: not accepted by the GEMM
    out = torch.empty(1, 256, 256, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        C.gram_sym(x, out, None, None, 1.0, 0.0, 0, 0, 0)
    xb = torch.randn(1, 200, 256, device="cuda").bfloat16()  # rows not a multiple of 256
    with pytest.raises(RuntimeError, match="multiples of 256"):
        C.gram_sym2(xb, out, None, None, 1.0, 0.0, 0, 0)
    with pytest.raises(AssertionError, match="only supports up to 5"):
        ortho.orthogonalize_native([torch.randn(8, 8, device="cuda")], 6, "polar_express")


@pytest.mark.parametrize("strategy", ["newton_schulz", "polar_express"])
def test_orthogonalize_llama_size_batch_matches_fp64(strategy):
    """A Llama-3-8B gate/up batch (2 x 4096 x 14336, the transposed long-K path
    of the 2-SM engine) against the fp64 PyTorch loop."""
    torch.manual_seed(7)
    g = torch.randn(2, 4096, 14336, device="cuda")
    got = torch.stack(ortho.orthogonalize_native(list(g.unbind(0)), 5, strategy, 1e-7))
    loop = ns_loop if strategy == "newton_schulz" else pe_loop
    ref = loop(g.double(), 5, eps=1e-7).float()
    del g
    frac = _close_frac(got, ref, rtol=1e-2, atol=5e-2)
    assert frac < 0.02, frac
    # orthogonality: the singular values of the bf16 result sit near 1 (NS-5 and PE-5 leave a spread)
    sv = torch.linalg.svdvals(got[0].float())
    assert 0.3 < float(sv.min()) and float(sv.max()) < 1.3
    _ext.check_device_errors("cuda")
