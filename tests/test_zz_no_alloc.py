"""The allocation-free C entry point ``dmb_pack_normalize_noalloc``.

It serves callers that cannot allocate device memory when they call in (for
example code running inside an allocator or memory-pool callback, or a host
that owns all GPU memory up front). The test calls it through its exported C
symbol, twice in a row on different inputs (the shared scratch keeps the
previous call's contents), and compares it with the PyTorch-facing pair
``muon_pack`` + ``norm_finalize`` that it mirrors. This file is collected last
on purpose.
"""

import ctypes
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


def _symbol():
    mod = importlib.import_module("dtensor_muon_b200._C")
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.dmb_pack_normalize_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [
        ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_float, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
    ]
    return fn


def _reference(src, Np, Mp, fac, eps):
    from dtensor_muon_b200.ops import _ext
    from dtensor_muon_b200.ops.ortho import ptr_tensor

    C = _ext.load()
    B, R, Cc = src.shape
    x = torch.empty(B, Np, Mp, dtype=torch.bfloat16, device=src.device)
    ptrs = ptr_tensor([src[b].data_ptr() for b in range(B)], src.device)
    partial = C.muon_pack(ptrs, None, 0 if src.dtype == torch.float32 else 1, R, Cc, Cc, R > Cc, x, 0.0, False, False)
    return x, C.norm_finalize(partial, fac, eps)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_binding_two_calls(dtype):
    fn = _symbol()
    torch.manual_seed(0)
    stream = torch.cuda.current_stream()
    cases = [(3, 200, 384, 256, 384, 1.0), (2, 384, 100, 128, 384, 1.02)]  # second one transposes
    for B, R, Cc, Np, Mp, fac in cases:
        src = (torch.randn(B, R, Cc, device="cuda") * 3).to(dtype)
        out = torch.full((B, Np, Mp), 7.0, dtype=torch.bfloat16, device="cuda")
        inv = torch.full((B,), -1.0, device="cuda")
        rc = fn(src.data_ptr(), 0 if dtype == torch.float32 else 1, B, R, Cc, Np, Mp, fac, 1e-7,
                out.data_ptr(), inv.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, rc
        x_ref, inv_ref = _reference(src, Np, Mp, fac, 1e-7)
        torch.cuda.synchronize()
        assert torch.equal(out, x_ref)
        torch.testing.assert_close(inv, inv_ref, rtol=1e-6, atol=0.0)
        ref_norm = src.float().norm(dim=(-2, -1))
        torch.testing.assert_close(inv, 1.0 / (ref_norm * fac + 1e-7), rtol=1e-2, atol=0.0)


def test_noalloc_rejects_oversized_problem():
    fn = _symbol()
    src = torch.zeros(1, 8, 8, device="cuda")
    out = torch.zeros(1, 64, 64, dtype=torch.bfloat16, device="cuda")
    inv = torch.zeros(1, device="cuda")
    rc = fn(src.data_ptr(), 0, 2048, 8, 8, 64, 64, 1.0, 1e-7, out.data_ptr(), inv.data_ptr(), None)
    assert rc == -1
