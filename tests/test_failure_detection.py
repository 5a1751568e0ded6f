"""Failure detection without faulting a GPU.

Device side: the device barrier of the fused collectives waits on a flag that
no peer will ever set; the bounded wait must give up (about 2 s), record an
error code and return, and the context must stay usable. Host side: a rank
that dies makes the survivors' next collective fail within the process-group
timeout instead of hanging.
"""

import time

import pytest
import torch
import torch.multiprocessing as mp

from testkit import run_distributed


@pytest.mark.gpu
def test_device_barrier_times_out_and_reports():
    from dtensor_muon_b200.ops import _ext

    C = _ext.load()
    _ext.check_device_errors("cuda")  # start clean
    flags = torch.zeros(64, dtype=torch.int32, device="cuda")
    # A 2-rank barrier on one GPU whose "peer" is this same buffer: flags[1] is never written.
    ptrs = torch.tensor([flags.data_ptr(), flags.data_ptr()], dtype=torch.int64, device="cuda")
    t0 = time.time()
    C.dist_barrier(ptrs, 0, 2, 1)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert 1.0 < elapsed < 30.0, elapsed
    with pytest.raises(RuntimeError, match="error code 2"):
        _ext.check_device_errors("cuda")
    # the context is still usable
    x = torch.randn(1000, device="cuda")
    assert torch.isfinite((x * 2).sum())
    _ext.check_device_errors("cuda")


def _dead_rank_worker(rank, world):
    import torch.distributed as dist

    if rank == 1:
        import os

        os._exit(0)  # leaves between steps, with nothing in flight
    t = torch.ones(1)
    try:
        dist.all_reduce(t)
    except Exception as exc:  # gloo reports the lost peer / timeout
        raise RuntimeError(f"peer loss detected: {type(exc).__name__}") from None
    raise AssertionError("collective with a dead peer must not succeed")


def test_dead_rank_is_detected_on_host():
    t0 = time.time()
    with pytest.raises((mp.ProcessRaisedException, mp.ProcessExitedException)):
        run_distributed(_dead_rank_worker, 2, timeout_s=10)
    assert time.time() - t0 < 120
