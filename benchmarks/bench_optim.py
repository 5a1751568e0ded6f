"""optimizer.step() benchmark on one GPU: naive eager Muon vs Muon per-param vs
Muon foreach (NS and PE) vs the quantised-state MuonLP variants.

Workload (as in the reference's benchmark/bench_optim.py): 12 layers of a
d_model=2048 transformer, qkv 2048x6144, out 2048x2048, mlp_in 2048x8192,
mlp_out 8192x2048 (``--quick``: 4 layers at d_model=512). Cautious WD off to
match the naive baseline.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from benchmarks.harness import bench, markdown_table  # noqa: E402
from benchmarks.naive_muon import NaiveMuon  # noqa: E402

FULL = [(12, (2048, 6144)), (12, (2048, 2048)), (12, (2048, 8192)), (12, (8192, 2048))]
QUICK = [(4, (512, 1536)), (4, (512, 512)), (4, (512, 2048)), (4, (2048, 512))]


def shapes(profile):
    return [s for n, s in profile for _ in range(n)]


def reference_variants():
    """The unmodified reference optimizer from baseline/_ref (compiled update, Triton Gram)."""
    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.isdir(os.path.join(root, "muonium")):
        return {}
    sys.path.insert(0, root)
    from muonium import Muon as RefMuon

    return {
        "reference Muon per-param (pe)": lambda ps: RefMuon(ps, foreach=False, use_cautious_wd=False),
        "reference Muon foreach (pe)": lambda ps: RefMuon(ps, foreach=True, use_cautious_wd=False),
    }


def run(profile, with_reference: bool = False) -> str:
    from dtensor_muon_b200 import Muon, Muon4bit, Muon8bit, MuonFp8

    sh = shapes(profile)
    gen = torch.Generator(device="cuda").manual_seed(0)
    grads = [torch.randn(s, device="cuda", generator=gen) for s in sh]
    variants = {
        "naive (ns)": lambda ps: NaiveMuon(ps, lr=1e-3, wd=0.1),
        "Muon per-param (ns)": lambda ps: Muon(ps, foreach=False, use_cautious_wd=False,
                                               orthogonalization_strategy="newton_schulz"),
        "Muon per-param (pe)": lambda ps: Muon(ps, foreach=False, use_cautious_wd=False),
        "Muon foreach (ns)": lambda ps: Muon(ps, foreach=True, use_cautious_wd=False,
                                             orthogonalization_strategy="newton_schulz"),
        "Muon foreach (pe)": lambda ps: Muon(ps, foreach=True, use_cautious_wd=False),
        "Muon8bit (pe)": lambda ps: Muon8bit(ps, use_cautious_wd=False),
        "Muon4bit (pe)": lambda ps: Muon4bit(ps, use_cautious_wd=False),
        "MuonFp8 (pe)": lambda ps: MuonFp8(ps, use_cautious_wd=False),
    }
    if with_reference:
        variants.update(reference_variants())
    rows = []
    base = None
    for name, make in variants.items():
        params = [torch.nn.Parameter(torch.randn(s, device="cuda", generator=gen)) for s in sh]
        opt = make(params)

        def step():
            for p, g in zip(params, grads):
                p.grad = g
            opt.step()

        ms = bench(step, warmup=3, reps=10, flush_l2=False)
        base = base or ms
        rows.append([name, ms, base / ms])
    return markdown_table(["optimizer", "step ms", "speedup vs naive"], rows)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--with-reference", action="store_true")
    args = ap.parse_args()
    print(run(QUICK if args.quick else FULL, args.with_reference))


if __name__ == "__main__":
    main()
