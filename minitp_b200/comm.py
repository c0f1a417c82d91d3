"""Host side of the NVLink peer-memory communicator.

One ``cudaMalloc``'d buffer per rank holds control words, per-CTA flags and
double-buffered receive slots; every rank maps all peers' buffers through
CUDA IPC. The handles are exchanged once, here, with
``torch.distributed.all_gather_object``. After that, every collective on the
decode path is a store over NVLink followed by a flag: no NCCL call and no
host involvement.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from minitp_b200 import _lib


def exchange_handles(process_group, mine: bytes, world: int) -> bytes:
    """All ranks' 64-byte IPC handles concatenated in rank order (one collective)."""
    if len(mine) != 64:
        raise ValueError("an IPC handle is 64 bytes")
    handles: list = [None] * world
    dist.all_gather_object(handles, bytes(mine), group=process_group)
    if any(h is None or len(h) != 64 for h in handles):
        raise RuntimeError("IPC handle exchange returned a malformed handle")
    return b"".join(handles)


class NvlinkComm:
    """Owns a ``mtpb_comm`` handle (see include/minitp_b200.h)."""

    def __init__(self, handle: int, rank: int, world: int, device: torch.device):
        self.handle = handle
        self.rank = rank
        self.world = world
        self.device = device

    @classmethod
    def create(cls, ctx, slot_bytes: int) -> NvlinkComm:
        _lib.require_cuda(torch.empty(0, device=ctx.device))
        with torch.cuda.device(ctx.device):
            h = ctypes.c_void_p()
            _lib.call("mtpb_comm_create", ctx.tp_rank, ctx.tp_size, slot_bytes, ctypes.byref(h))
            comm = cls(h.value, ctx.tp_rank, ctx.tp_size, ctx.device)
            if ctx.tp_size > 1:
                if ctx.process_group is None:
                    raise ValueError("tp_size > 1 needs a process group to exchange IPC handles")
                mine = ctypes.create_string_buffer(64)
                _lib.call("mtpb_comm_ipc_handle", comm.handle, mine)
                all_h = exchange_handles(ctx.process_group, mine.raw, ctx.tp_size)
                blob = ctypes.create_string_buffer(all_h, 64 * ctx.tp_size)
                _lib.call("mtpb_comm_open", comm.handle, blob)
                # every rank mapped every peer before anyone sends
                dist.barrier(group=ctx.process_group)
        return comm

    # ------------------------------------------------------------------
    def set_timeout(self, seconds: float) -> None:
        _lib.call("mtpb_comm_set_timeout", self.handle, int(seconds * 1e9))

    def status(self) -> int:
        """Synchronise and return the device status word (0 = healthy)."""
        out = ctypes.c_uint32()
        with torch.cuda.device(self.device):
            _lib.call("mtpb_comm_status", self.handle, ctypes.byref(out))
        return out.value

    def clear_status(self) -> None:
        with torch.cuda.device(self.device):
            _lib.call("mtpb_comm_clear_status", self.handle)

    def raise_on_error(self) -> None:
        s = self.status()
        if s:
            msg = _lib.status_error(s)
            if s & _lib.STATUS_TIMEOUT:
                raise _lib.PeerTimeoutError(f"rank {self.rank}: {msg}")
            raise _lib.MinitpB200Error(f"rank {self.rank}: {msg}")

    def pos_ptr(self) -> int:
        return _lib.load().mtpb_comm_pos_ptr(self.handle)

    def slot_bytes(self) -> int:
        return _lib.load().mtpb_comm_slot_bytes(self.handle)

    def close(self) -> None:
        if self.handle:
            with torch.cuda.device(self.device):
                torch.cuda.synchronize()
                _lib.load().mtpb_comm_destroy(self.handle)
            self.handle = 0
