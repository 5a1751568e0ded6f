"""Config 1: CPU fp32 parity run of the 2-layer Llama (d 256, 4 heads, SwiGLU 1024,
vocab 1024) for 20 steps, batch 8 x seq 128, Muon (polar_express, 5 steps, momentum
0.95 Nesterov, lr 1e-3, wd 0.1 cautious) on 2-D weights and AdamW (0.9, 0.95) on
embeddings / norms / head.

``python -m dtensor_muon_b200.testing.parity --impl ours|reference`` prints one JSON
line with the per-step losses and a checksum of the final parameters. The
reference arm imports ``muonium`` from ``baseline/_ref`` and drives it through its
own CPU seam (``zeropower`` with ``use_triton=False``; run with
``TORCH_COMPILE_DISABLE=1``), on the same model, data and init.
"""

from __future__ import annotations

import argparse
import functools
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def run(impl: str, steps: int = 20, load: str | None = None, save: str | None = None, start: int = 0) -> dict:
    """Train ``steps`` steps (data steps ``start`` .. ``start + steps``); optionally
    resume model + optimizer from ``load`` and write them to ``save`` (torch.save)."""
    sys.path.insert(0, ROOT)
    from dtensor_muon_b200.models.llama import Llama, lm_loss, muon_and_adam_params, preset

    torch.manual_seed(0)
    cfg = preset("tiny")
    model = Llama(cfg)
    model.init_weights(seed=0)
    muon, adam = muon_and_adam_params(model)
    kw = dict(lr=1e-3, wd=0.1, orthogonalization_strategy="polar_express", ns_steps=5, momentum=0.95,
              nesterov=True, use_cautious_wd=True, adam_betas=(0.9, 0.95))
    groups = [{"params": muon}, {"params": adam, "algorithm": "adamw"}]
    if impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        from install_reference import ensure_reference

        sys.path.insert(0, ensure_reference())
        import muonium.optim.algorithms.base as ref_base
        from muonium import Muon as RefMuon
        from muonium.orthogonalize import foreach_zeropower, zeropower

        ref_base.zeropower = functools.partial(zeropower, use_triton=False)
        ref_base.foreach_zeropower = functools.partial(foreach_zeropower, use_triton=False)
        opt = RefMuon(groups, **kw)
    else:
        from dtensor_muon_b200 import Muon

        opt = Muon(groups, **kw)
    if load:
        ckpt = torch.load(load, weights_only=False)
        model.load_state_dict(ckpt["model"])
        opt.load_state_dict(ckpt["optim"])
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (start + steps, 8, 129), generator=gen)
    losses = []
    for s in range(start, start + steps):
        loss = lm_loss(model(ids[s, :, :-1]), ids[s, :, 1:])
        loss.backward()
        opt.step()
        opt.zero_grad()
        losses.append(loss.item())
    checksum = float(sum(p.detach().double().abs().sum() for p in model.parameters()))
    if save:
        torch.save({"model": model.state_dict(), "optim": opt.state_dict()}, save)
    return {"impl": impl, "losses": losses, "param_abs_sum": checksum}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--start", type=int, default=0)
    ap.add_argument("--load")
    ap.add_argument("--save")
    args = ap.parse_args()
    print(json.dumps(run(args.impl, args.steps, args.load, args.save, args.start)))


if __name__ == "__main__":
    main()
