"""utils (group_tensors_by_shape, move_tensors_to_device, to_local) and the
distributed spawner (mirrors tests/utils/test_foreach.py and test_testing.py)."""

import os

import pytest
import torch
import torch.multiprocessing as mp

from dtensor_muon_b200.utils import group_tensors_by_shape, move_tensors_to_device, to_local
from testkit import assert_close, clone_args, run_distributed


def test_group_by_shape_keeps_order_and_ignores_dtype():
    ts = [torch.zeros(2, 3), torch.zeros(4), torch.zeros(2, 3, dtype=torch.float64), torch.zeros(())]
    g = group_tensors_by_shape(ts)
    assert list(g) == [(2, 3), (4,), ()]
    assert g[(2, 3)][1] == [0, 2] and g[()][1] == [3]


def test_move_same_type_is_noop():
    ts = [torch.zeros(2), None]
    out = move_tensors_to_device(ts, torch.device("cpu"), torch.device("cpu"))
    assert out is ts


def test_to_local_plain_tensor_passthrough():
    t = torch.zeros(3)
    assert to_local(t) is t and to_local(t, full_tensor=True) is t


def test_assert_close_mismatch_budget():
    a = torch.zeros(100)
    b = torch.zeros(100)
    b[:3] = 1.0
    assert_close(a, b, atol=0.1, rtol=0, max_mismatch_pct=5.0)
    with pytest.raises(AssertionError, match="mismatched"):
        assert_close(a, b, atol=0.1, rtol=0, max_mismatch_pct=1.0)


def test_clone_args_detaches_and_keeps_requires_grad():
    x = torch.randn(3, requires_grad=True)
    (y, k) = clone_args((x, 5))
    assert y is not x and y.requires_grad and k == 5
    y.data.add_(1)
    assert not torch.equal(x, y)


def _env_worker(rank, world):
    import torch.distributed as dist

    assert os.environ["RANK"] == str(rank) and os.environ["WORLD_SIZE"] == str(world)
    assert os.environ["MASTER_ADDR"] == "127.0.0.1"
    assert dist.get_rank() == rank and dist.get_world_size() == world
    t = torch.tensor([rank + 1.0])
    dist.all_reduce(t)
    assert t.item() == world * (world + 1) / 2


def test_spawner_sets_env_and_collectives_work():
    run_distributed(_env_worker, 3)


def _failing_worker(rank, world):
    import time

    if rank == 1:
        raise RuntimeError("rank one failed on purpose")
    time.sleep(10)  # the healthy rank outlives the failure, so the failure is what surfaces


def test_spawner_propagates_worker_failure():
    with pytest.raises(mp.ProcessRaisedException, match="rank one failed on purpose"):
        run_distributed(_failing_worker, 2, timeout_s=20)
