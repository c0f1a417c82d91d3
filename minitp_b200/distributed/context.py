"""ParallelContext: process-group topology plus this rank's NVLink communicator.

Same fields, properties and ``init_context`` behaviour as the reference
(minitp/distributed/context.py:18-78): single node, one TP group equal to
WORLD, NCCL when CUDA is available, Gloo when ``MINITP_BACKEND=gloo`` or
without CUDA. torch.distributed is plumbing here: it creates the group and
exchanges the CUDA IPC handles of the peer-memory communicator once. Every
hot-path collective (RowParallel AllReduce, embedding reduce, argmax gather)
then runs in minitp_b200's own kernels over NVLink.
"""

from __future__ import annotations

import datetime as dt
import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

# Bytes of one (channel, parity, source-rank) receive slot of the
# communicator: the largest single collective message it carries.
DEFAULT_SLOT_BYTES = 8 << 20


@dataclass
class ParallelContext:
    global_rank: int
    local_rank: int
    world_size: int
    tp_rank: int
    tp_size: int
    device: torch.device
    process_group: dist.ProcessGroup | None  # None => TP=1, no collectives
    _comm: object | None = field(default=None, repr=False, compare=False)

    @property
    def is_rank_zero(self) -> bool:
        return self.global_rank == 0

    @property
    def has_tp(self) -> bool:
        return self.tp_size > 1

    def barrier(self) -> None:
        if self.process_group is not None:
            dist.barrier(self.process_group)

    def destroy(self) -> None:
        if self._comm is not None:
            self._comm.close()
            self._comm = None
        if dist.is_initialized():
            dist.destroy_process_group()

    def comm(self, slot_bytes: int = DEFAULT_SLOT_BYTES):
        """This rank's NVLink communicator (created collectively on first use).

        Every rank of the TP group must reach the first call together: it
        exchanges CUDA IPC handles with ``all_gather_object``.
        """
        if self._comm is None:
            from minitp_b200.comm import NvlinkComm
            from minitp_b200.distributed.collectives import register_comm

            self._comm = NvlinkComm.create(self, slot_bytes)
            if self.process_group is not None:
                register_comm(self.process_group, self._comm)
        return self._comm


def init_context(backend: str | None = None, timeout_s: float = 600.0) -> ParallelContext:
    """Initialise from the torchrun environment (RANK / LOCAL_RANK / WORLD_SIZE).

    Standalone (WORLD_SIZE unset or 1): TP=1 on ``cuda`` if available, else CPU,
    with no process group.
    """
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    force_cpu = os.environ.get("MINITP_BACKEND", "").lower() == "gloo"
    if world == 1:
        if force_cpu or not torch.cuda.is_available():
            device = torch.device("cpu")
        else:
            torch.cuda.set_device(local_rank)
            device = torch.device("cuda", local_rank)
        return ParallelContext(rank, local_rank, 1, 0, 1, device, None)
    if backend is None:
        backend = "gloo" if force_cpu or not torch.cuda.is_available() else "nccl"
    if backend == "gloo":
        os.environ.setdefault("USE_LIBUV", "0")
    if backend == "nccl":
        torch.cuda.set_device(local_rank)
    dist.init_process_group(
        backend=backend, rank=rank, world_size=world, timeout=dt.timedelta(seconds=timeout_s)
    )
    device = torch.device("cuda", local_rank) if backend == "nccl" else torch.device("cpu")
    return ParallelContext(rank, local_rank, world, rank, world, device, dist.group.WORLD)


def context_for(tp_size: int = 1, device: str = "cpu") -> ParallelContext:
    """Single-process TP=1 context (minitp/config.py:100-112)."""
    return ParallelContext(0, 0, 1, 0, 1, torch.device(device), None)
