"""build_llama(fused_gather=True) on a CPU gloo mesh: the q/k/v and gate/up weights
leave FSDP2 as Shard(0) DTensors of the right global shape and local rows, every
other parameter stays FSDP-managed, and the optimizer sees all of them."""

from testkit import run_distributed


def _worker(rank, world):
    import torch
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import DTensor, Shard

    from dtensor_muon_b200.models import preset
    from dtensor_muon_b200.models.llama import muon_and_adam_params
    from dtensor_muon_b200.train import build_llama

    mesh = init_device_mesh("cpu", (world,))
    cfg = preset("tiny", dim=512, n_heads=4, n_kv_heads=2, ffn_dim=1024, n_layers=2)
    model = build_llama(cfg, torch.device("cpu"), mesh=mesh, seed=0, fsdp_comm="nccl", fused_gather=True)
    for layer in model.layers:
        att, ffn = layer.attention, layer.feed_forward
        assert att.gather is not None and ffn.gather is not None
        for lin, rows in ((att.wq, 512), (att.wk, 256), (att.wv, 256), (ffn.w1, 1024), (ffn.w3, 1024)):
            w = lin.weight
            assert isinstance(w, DTensor) and w.placements == (Shard(0),)
            assert tuple(w.shape) == (rows, 512)
            assert tuple(w.to_local().shape) == (rows // world, 512)
            assert w.to_local().device.type == "cpu" and torch.isfinite(w.to_local()).all()
        for p in att.gather.params + ffn.gather.params:
            assert p.requires_grad
    model2 = build_llama(cfg, torch.device("cpu"), mesh=mesh, seed=0, fsdp_comm="nccl", fused_gather="all")
    for layer in model2.layers:
        assert layer.attention.gather_out is not None and layer.feed_forward.gather_out is not None
        assert isinstance(layer.attention.wo.weight, DTensor) and tuple(layer.feed_forward.w2.weight.shape) == (512, 1024)
    muon, adam = muon_and_adam_params(model)
    assert len(muon) == 2 * 7 and all(isinstance(p, DTensor) for p in muon + adam)


def test_fused_gather_model_layout():
    run_distributed(_worker, 2, backend="gloo", device_type="cpu", timeout_s=120)


def test_eligibility_rules():
    import torch

    from dtensor_muon_b200.parallel.ag_gemm import GatherLinear

    def lins(*shapes):
        return [torch.nn.Linear(k, n, bias=False, device="meta") for n, k in shapes]

    assert GatherLinear.eligible(lins((4096, 4096), (1024, 4096), (1024, 4096)), 8)
    assert not GatherLinear.eligible(lins((4096, 4096), (1024, 4096), (1024, 4096)), 16)  # 64 k rows per rank
    assert not GatherLinear.eligible(lins((512, 256), (512, 128)), 2)  # different K
    assert not GatherLinear.eligible(lins((384, 256)), 1)  # rows not a multiple of 256
    assert not GatherLinear.eligible(lins(*[(256, 256)] * 5), 1)  # more than four weights
