"""Kernel benchmarks: the tcgen05 Gram and the full NS / PE orthogonalisation
against cuBLAS-based PyTorch (and, with --with-reference, the reference's Triton
Gram and compiled loops from baseline/_ref).

Config-2 shapes (the headline orthogonalisation microbench): 4096x4096, 4096x14336, 14336x4096 and 64 x 1024x1024,
bf16 inputs N(0,1), 5 steps. Reports ms and the fraction of the measured bf16
peak for the dense FLOP count (the symmetric kernels do less actual work, so a
fraction above the cuBLAS denominator is expected).

``--ncu-case gram|bx`` runs a small single case a few times for an ncu capture.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from benchmarks.harness import bench, clocks, markdown_table, ortho_flops, peaks  # noqa: E402

CONFIG2 = [(1, 4096, 4096), (1, 4096, 14336), (1, 14336, 4096), (64, 1024, 1024)]
QUICK = [(1, 4096, 4096), (8, 1024, 1024)]
GRAM = [(32, 2048, 1024), (32, 1024, 1024), (1, 2048, 2048), (32, 2048, 4096)]


def torch_loop(strategy):
    from dtensor_muon_b200.orthogonalize import ns_loop, pe_loop

    loop = ns_loop if strategy == "newton_schulz" else pe_loop
    return lambda x: loop(x.bfloat16(), 5, eps=1e-7)


def reference_loop(strategy):
    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    sys.path.insert(0, root)
    from muonium.orthogonalize.newton_schulz import ns_loop_triton
    from muonium.orthogonalize.polar_express import pe_loop_triton

    loop = ns_loop_triton if strategy == "newton_schulz" else pe_loop_triton
    return lambda x: loop(x.bfloat16(), 5, eps=1e-7)


def run(shapes, with_reference: bool) -> str:
    from dtensor_muon_b200.ops import ortho

    pk = peaks()
    rows = []
    for strategy in ("newton_schulz", "polar_express"):
        for B, R, C in shapes:
            torch.manual_seed(0)
            x = torch.randn(B, R, C, device="cuda").bfloat16()
            x = x / x.float().norm(dim=(-2, -1), keepdim=True).bfloat16()  # Frobenius-normalised (config 2)
            mats = list(x.unbind(0))
            with clocks() as ck:
                ours = bench(lambda: ortho.orthogonalize_native(mats, 5, strategy), reps=20)
            tl = bench(lambda: torch_loop(strategy)(x))
            ref = None
            if with_reference:
                try:
                    ref = bench(lambda: reference_loop(strategy)(x))
                except Exception as exc:  # compile / import failure is reported, not fatal
                    ref = f"unavailable: {type(exc).__name__}"
            fl = ortho_flops(B, R, C)
            frac = fl / (ours * 1e-3) / (pk["bf16_tflops"] * 1e12)
            ck = ck.result or {}
            rows.append([strategy, f"{B}x{R}x{C}", ours, tl, ref if ref is not None else "-", frac,
                         ck.get("sm_mhz"), ",".join(ck.get("reasons", [])) or "none"])
    t1 = markdown_table(
        ["strategy", "shape", "ours ms", "torch bf16 loop ms", "reference triton ms",
         f"dense frac of {pk['source']} burst peak ({pk['bf16_tflops']} TF)", "median SM MHz (ours)", "throttle"],
        rows,
    )
    grows = []
    for B, M, K in GRAM:
        x = torch.randn(B, M, K, device="cuda").bfloat16()
        xp = x.contiguous()
        out = torch.empty(B, M, M, device="cuda", dtype=torch.bfloat16)
        from dtensor_muon_b200.ops import _ext

        C_ = _ext.load()
        ok = M % 256 == 0 and K % 256 == 0
        ours = bench(lambda: C_.gram_sym(xp, out, None, None, 1.0, 0.0, 0, 0, 0)) if ok else float("nan")
        grows.append([f"{B}x{M}x{K}", ours, bench(lambda: x @ x.mT)])
    t2 = markdown_table(["gram shape", "ours ms", "torch x@x.mT ms"], grows)
    return t1 + "\n\n" + t2


def ncu_case(which: str) -> None:
    """Small case for ncu: 1 x 2048 x 8192 (32 MiB input > L2 working sets of a tile)."""
    from dtensor_muon_b200.ops import _ext

    C_ = _ext.load()
    x = torch.randn(4, 2048, 8192, device="cuda").bfloat16()
    a = torch.empty(4, 2048, 2048, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(x)
    for _ in range(3):
        if which == "gram":
            C_.gram_sym(x, a, None, None, 1.0, 0.0, 0, 0, 0)
        else:
            C_.gemm_ax(a, x, out, x, None, 1.0, 0.5, 0, 0, 0)
    torch.cuda.synchronize()
    _ext.check_device_errors("cuda")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--with-reference", action="store_true")
    ap.add_argument("--ncu-case", choices=["gram", "bx"])
    args = ap.parse_args()
    if args.ncu_case:
        ncu_case(args.ncu_case)
        return
    print(run(QUICK if args.quick else CONFIG2, args.with_reference))


if __name__ == "__main__":
    main()
