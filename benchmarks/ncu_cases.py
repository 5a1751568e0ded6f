"""Small single-kernel cases for ncu captures (one GPU, a few launches, inputs
larger than L2 but a few GB at most).

    python benchmarks/ncu_cases.py --case pack|apply|adamw|lp|rope|swiglu|gemm2_gram|gemm2_bx|pe_64x1024
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    from dtensor_muon_b200.ops import _ext, model_ops
    from dtensor_muon_b200.ops.ortho import layout_for, ptr_tensor

    C = _ext.load()
    dev = torch.device("cuda")
    torch.manual_seed(0)
    case = args.case
    # 8 matrices of 4096 x 4096 (and transposed 14336 x 4096 for pack/apply): > L2.
    if case in ("pack", "apply"):
        B, R, Cc = 4, 14336, 4096  # transposed (R > C) path: the gate/up shape
        lay = layout_for(R, Cc)
        g = torch.randn(B, R, Cc, device=dev).bfloat16()
        buf = torch.zeros(B, R, Cc, device=dev)
        p = torch.randn(B, R, Cc, device=dev).bfloat16()
        x = torch.empty(B, lay.Np, lay.Mp, device=dev, dtype=torch.bfloat16)
        gp = ptr_tensor([g[b].data_ptr() for b in range(B)], dev)
        bp = ptr_tensor([buf[b].data_ptr() for b in range(B)], dev)
        pp = ptr_tensor([p[b].data_ptr() for b in range(B)], dev)
        for _ in range(args.reps):
            if case == "pack":
                C.muon_pack(gp, bp, 1, R, Cc, Cc, True, x, 0.95, True, False)
            else:
                C.muon_apply(x, True, R, Cc, Cc, pp, 1, None, None, 1e-3, 0.1, True)
    elif case == "adamw":
        n = 256 << 20  # 256 M bf16 params, bf16 states
        ts = [torch.randn(n, device=dev).bfloat16() for _ in range(4)]
        steps = [torch.tensor(0.0)]
        from dtensor_muon_b200.ops.adamw import fused_adam

        for _ in range(args.reps):
            fused_adam([ts[0]], [ts[1]], [ts[2]], [ts[3]], [], steps, amsgrad=False, beta1=0.9, beta2=0.95,
                       lr=1e-3, weight_decay=0.1, eps=1e-8, maximize=False, decoupled_weight_decay=True)
    elif case == "lp":
        from dtensor_muon_b200.optim.optim_lp import FMT_8BIT, QuantizedState

        n = 128 << 20
        q = QuantizedState.zeros((n,), FMT_8BIT, 2048, True, dev)
        g = torch.randn(n, device=dev).bfloat16()
        out = torch.empty(n, device=dev, dtype=torch.bfloat16)
        for _ in range(args.reps):
            C.lp_momentum_step(q.codes, q.scale, q.qmap, q.fmt, q.block_size, g, out, 0.95, True, False)
    elif case == "rope":
        from dtensor_muon_b200.models.llama import rope_tables

        x = torch.randn(1, 4096, 32, 128, device=dev).bfloat16()
        cos, sin = rope_tables(128, 4096, 5e5, dev)
        for _ in range(args.reps * 4):
            C.rope(x, cos, sin, 1.0)
    elif case == "swiglu":
        a = torch.randn(4096, 14336, device=dev).bfloat16()
        b = torch.randn(4096, 14336, device=dev).bfloat16()
        for _ in range(args.reps):
            h = model_ops.swiglu(a, b)
            C.swiglu_bwd(a, b, h)
    elif case in ("gemm2_gram", "gemm2_bx"):
        x = torch.randn(4, 2048, 8192, device=dev).bfloat16()
        a = torch.empty(4, 2048, 2048, device=dev, dtype=torch.bfloat16)
        out = torch.empty_like(x)
        for _ in range(args.reps):
            if case == "gemm2_gram":
                C.gram_sym2(x, a, None, None, 1.0, 0.0, 0, 0)
            else:
                C.gemm_ax2(a, x, out, x, None, 1.0, 0.5, 0, 0)
    elif case == "pe_64x1024":
        # short-K case: PE-5 on 64 x 1024 x 1024 through the public engine entry (18 launches per call)
        from dtensor_muon_b200.ops import ortho

        mats = list(torch.randn(64, 1024, 1024, device=dev).bfloat16().unbind(0))
        for _ in range(8):
            ortho.orthogonalize_native(mats, 5, "polar_express")
    else:
        raise SystemExit(f"unknown case {case}")
    torch.cuda.synchronize()
    _ext.check_device_errors(dev)


if __name__ == "__main__":
    main()
