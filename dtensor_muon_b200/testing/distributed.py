"""Spawn a small ``torch.distributed`` world for tests and benchmarks.

Same contract as the reference's ``test_support.distributed.run_distributed``
(test_support/distributed.py:61-85): ``worker(rank, world_size, *args,
**kwargs)`` runs in ``world_size`` spawned processes that share a process
group (gloo on CPU by default, NCCL on CUDA); worker exceptions propagate to
the caller; every rank meets at a teardown barrier before the group is
destroyed.
"""

from __future__ import annotations

import os
import socket
from typing import Any, Callable


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world_size, backend, port, device_type, fn, args, kwargs, timeout_s):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(
        MASTER_ADDR="127.0.0.1",
        MASTER_PORT=str(port),
        RANK=str(rank),
        WORLD_SIZE=str(world_size),
        LOCAL_RANK=str(rank),
    )
    device_id = None
    if device_type == "cuda":
        torch.cuda.set_device(rank)
        device_id = torch.device("cuda", rank)
    dist.init_process_group(
        backend=backend,
        rank=rank,
        world_size=world_size,
        device_id=device_id,
        timeout=datetime.timedelta(seconds=timeout_s),
    )
    try:
        fn(rank, world_size, *args, **kwargs)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def run_distributed(
    worker: Callable[..., None],
    world_size: int = 2,
    *,
    args: tuple = (),
    kwargs: dict[str, Any] | None = None,
    backend: str = "gloo",
    device_type: str = "cpu",
    timeout_s: float = 120.0,
) -> None:
    """Run ``worker`` on ``world_size`` spawned ranks; re-raises a rank's failure."""
    import torch.multiprocessing as mp

    mp.spawn(
        _entry,
        args=(world_size, backend, free_port(), device_type, worker, args, kwargs or {}, timeout_s),
        nprocs=world_size,
        join=True,
    )
