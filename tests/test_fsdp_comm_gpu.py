"""FSDP2 with the P2P all-gather / reduce-scatter kernels (and with the Muon momentum
fused into the reduce-scatter) against FSDP2 on NCCL (2 GPUs)."""

import pytest
import torch

from testkit import run_distributed

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world, ag_mode="ce", rs_mode="auto"):
    import torch
    from torch.distributed.device_mesh import init_device_mesh

    from dtensor_muon_b200.models.llama import lm_loss, preset
    from dtensor_muon_b200.ops import _ext
    from dtensor_muon_b200.parallel import fsdp_comm
    from dtensor_muon_b200.train import build_llama, build_optimizer

    fsdp_comm.AG_MODE = ag_mode
    fsdp_comm.RS_MODE = rs_mode

    mesh = init_device_mesh("cuda", (world,))
    cfg = preset("tiny", vocab_size=1024, dim=256, n_layers=2)
    dev = torch.device("cuda", rank)
    results = {}
    for comm in ("nccl", "p2p", "p2p+fused"):
        model = build_llama(cfg, dev, mesh=mesh, seed=0, fsdp_comm=comm.split("+")[0])
        opt = build_optimizer(model, lr=1e-2, fuse_momentum=comm.endswith("fused"))
        gen = torch.Generator().manual_seed(7 + rank)
        losses = []
        for _ in range(3):
            ids = torch.randint(0, cfg.vocab_size, (2, 65), generator=gen).to(dev)
            loss = lm_loss(model(ids[:, :-1]), ids[:, 1:])
            loss.backward()
            opt.step()
            opt.zero_grad(set_to_none=True)
            losses.append(loss.item())
        results[comm] = (losses, [p.full_tensor().float() for p in model.parameters()])
    torch.cuda.synchronize()
    _ext.check_device_errors(dev)
    from dtensor_muon_b200.parallel.fsdp_comm import FUSED_GRADS

    assert not FUSED_GRADS, "every fused gradient must be consumed by an optimizer step"
    for other in ("p2p", "p2p+fused"):
        for a, b in zip(results["nccl"][0], results[other][0]):
            assert abs(a - b) < 2e-2 * max(1.0, abs(a)), (other, a, b)
        for x, y in zip(results["nccl"][1], results[other][1]):
            bad = (~torch.isclose(x, y, rtol=2e-2, atol=2e-2)).float().mean().item()
            assert bad < 0.02, (other, bad)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("ag_mode,rs_mode", [("ce", "auto"), ("ce", "ce"), ("pull", "push"), ("push", "nvls")])
def test_fsdp_p2p_collectives_match_nccl(ag_mode, rs_mode):
    """Every all-gather / reduce-scatter scheme (copy engines, P2P kernels, NVLS
    multimem reduce where the fabric has multicast) against FSDP2 on NCCL."""
    run_distributed(_worker, 2, args=(ag_mode, rs_mode), backend="nccl", device_type="cuda")
