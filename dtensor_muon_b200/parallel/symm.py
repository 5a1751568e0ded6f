"""Symmetric (peer-addressable) device memory for the fused collective kernels.

Every rank allocates a buffer of the same size; after a rendezvous each rank
knows every peer's base address and the kernels in ``ops/csrc/dist_ops.cu``
read and write peers' buffers directly with P2P loads / stores over NVLink /
NVSwitch. ``torch.distributed._symmetric_memory`` is used only as the
allocator + address-exchange bootstrap; the data movement and the barrier are
our own kernels. Barriers are bounded on the device (2 s) and report through
the per-device error word, which :meth:`SymmetricWorkspace.check` raises on.

The reference moves the same data with DTensor redistributes (NCCL all-to-alls
in ``foreach_zeropower``, ``src/muonium/orthogonalize/orthogonalize.py:142-150``).
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops import _ext


def nvls_enabled() -> bool:
    """Use NVSwitch multicast (``multimem``) where the symmetric allocation has a
    multicast address; ``DMB_NVLS=0`` turns it off (the failure-detection tests
    do, because a rank that dies while bound to a multicast object has raised
    NVLink faults on its peers on this hardware)."""
    return os.environ.get("DMB_NVLS", "1") != "0"


def available() -> bool:
    if os.environ.get("DMB_DISABLE_SYMM", "0") == "1":
        return False
    if not (dist.is_available() and dist.is_initialized()):
        return False
    try:
        import torch.distributed._symmetric_memory  # noqa: F401
    except ImportError:
        return False
    return _ext.available()


class SymmetricWorkspace:
    """A grow-only symmetric byte buffer plus a persistent barrier flag array."""

    def __init__(self, group: dist.ProcessGroup, device: torch.device):
        import torch.distributed._symmetric_memory as symm_mem

        self._symm = symm_mem
        self.group = group
        self.device = device
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        name = group.group_name
        enable = getattr(symm_mem, "enable_symm_mem_for_group", None)
        if enable is not None:  # subgroups (HSDP shard groups, TP/EP groups) need their own store
            enable(name)
        self._flags = symm_mem.empty(max(64, self.world), dtype=torch.int32, device=device)
        self._flags.zero_()
        hdl = symm_mem.rendezvous(self._flags, name)
        self.flag_ptrs = torch.tensor(list(hdl.buffer_ptrs), dtype=torch.int64).to(device)
        torch.cuda.synchronize(device)
        dist.barrier(group)
        self.epoch = 0
        self._buf: torch.Tensor | None = None
        self.peer_base: torch.Tensor | None = None
        # NVSwitch multicast address of the current buffer (0: none / disabled)
        self.mc_base = 0
        self._keep = [hdl]

    def barrier(self) -> None:
        """Device-side barrier over the group (bounded wait in the kernel)."""
        self.epoch = (self.epoch + 1) & 0x7FFFFFFF
        _ext.load().dist_barrier(self.flag_ptrs, self.rank, self.world, self.epoch)

    # -- split barrier: per-slot signals (pipelined owner compute) ----------------
    SIGNAL_SLOTS = 256

    def _signal_ptrs(self) -> torch.Tensor:
        if getattr(self, "_sig_ptrs", None) is None:
            flags = self._symm.empty(self.SIGNAL_SLOTS * self.world, dtype=torch.int32, device=self.device)
            flags.zero_()
            hdl = self._symm.rendezvous(flags, self.group.group_name)
            self._sig_ptrs = torch.tensor(list(hdl.buffer_ptrs), dtype=torch.int64).to(self.device)
            self._keep += [flags, hdl]
            torch.cuda.synchronize(self.device)
            dist.barrier(self.group)
            self.sig_epoch = 0
        return self._sig_ptrs

    def next_signal_epoch(self) -> int:
        """A fresh epoch for one round of signals (every rank calls this in step)."""
        self._signal_ptrs()
        self.sig_epoch = (self.sig_epoch + 1) & 0x7FFFFFFF
        return self.sig_epoch

    def signal(self, slot: int, epoch: int) -> None:
        """After this stream's work so far: tell every rank that this rank reached ``slot``."""
        _ext.load().flag_signal(self._signal_ptrs(), slot % self.SIGNAL_SLOTS, self.rank, self.world, epoch)

    def wait(self, slot: int, epoch: int) -> None:
        """Stream-ordered bounded wait until every rank has signalled ``slot`` in ``epoch``."""
        _ext.load().flag_wait(self._signal_ptrs(), slot % self.SIGNAL_SLOTS, self.rank, self.world, epoch)

    def buffer(self, nbytes: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Local view of at least ``nbytes`` symmetric bytes and the [world] tensor of peer base addresses.

        Growing is collective: every rank must request the same sizes in the same order.
        """
        if self._buf is None or self._buf.numel() < nbytes:
            if self._buf is not None:
                self.barrier()  # peers are done with the old buffer
            size = max(nbytes, int((self._buf.numel() if self._buf is not None else 0) * 1.25))
            size = (size + (1 << 20) - 1) // (1 << 20) * (1 << 20)
            buf = self._symm.empty(size, dtype=torch.uint8, device=self.device)
            hdl = self._symm.rendezvous(buf, self.group.group_name)
            self.peer_base = torch.tensor(list(hdl.buffer_ptrs), dtype=torch.int64).to(self.device)
            self.mc_base = int(getattr(hdl, "multicast_ptr", 0) or 0) if nvls_enabled() else 0
            self._hdl = hdl
            self._buf = buf
            self._keep.append(hdl)
        return self._buf, self.peer_base

    def peer_bytes(self, k: int, off: int, nbytes: int) -> torch.Tensor:
        """uint8 view of rank ``k``'s symmetric buffer at ``off`` (a tensor on this
        device whose memory is the peer's; copies from or to it go over NVLink,
        by the copy engines when issued as a plain device copy)."""
        return self._hdl.get_buffer(k, (nbytes,), torch.uint8, off)

    def check(self) -> None:
        _ext.check_device_errors(self.device)


_WORKSPACES: dict[tuple[str, int, str], SymmetricWorkspace] = {}


def workspace_for(group: dist.ProcessGroup, device: torch.device, purpose: str = "optim") -> SymmetricWorkspace:
    """One workspace per (group, device, purpose): users that issue barriers on
    different streams (optimizer, EP exchange, FSDP all-gather, FSDP
    reduce-scatter) must not share a barrier epoch sequence."""
    key = (group.group_name, device.index if device.index is not None else torch.cuda.current_device(), purpose)
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = SymmetricWorkspace(group, device)
        _WORKSPACES[key] = ws
    return ws
