"""Collective wrappers with the reference's identity-return contract.

Mirrors minitp/distributed/collectives.py:147-245:

- ``all_reduce(t)``   -> ``t``   (in-place SUM)
- ``broadcast(t)``    -> ``t``
- ``reduce_scatter(out, t)`` -> ``out``
- ``all_gather(out, t)``     -> ``out`` (concatenated along the last dim)
- ``all_gather_dim0(out, t)`` -> ``out`` ([world, *t.shape])

CUDA ``all_reduce`` of fp32/bf16 tensors runs on minitp_b200's one-shot
NVLink kernel (``mtpb_allreduce``: rank-ordered, bit-identical on every rank).
The other collectives sit off the decode path (gather_logits debugging,
benchmark aggregation); they use torch.distributed.

Profiling (``set_profiling``) records the same fields as the reference:
op, bytes, dtype, shape, world_size, host_launch_ms, collective_gpu_ms
(CUDA events around the collective only) and postprocess_host_ms.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import torch
import torch.distributed as dist

_PROFILING = False
_RECORDS: list[dict] = []
_PENDING: list[tuple] = []
_COMMS: dict = {}


@dataclass
class CommStats:
    calls: int
    total_bytes: int
    host_launch_ms: float
    collective_gpu_ms: float | None
    postprocess_host_ms: float


def set_profiling(enabled: bool) -> None:
    global _PROFILING
    _PROFILING = enabled


def reset_comm_stats() -> None:
    _RECORDS.clear()
    _PENDING.clear()


def drain_comm_stats() -> None:
    if not _PENDING:
        return
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    for s, e, meta in _PENDING:
        meta["collective_gpu_ms"] = s.elapsed_time(e)
    _PENDING.clear()


def get_comm_stats() -> list[dict]:
    drain_comm_stats()
    return list(_RECORDS)


def comm_summary(window: list[dict] | None = None) -> CommStats:
    stats = get_comm_stats() if window is None else window
    gpu = [s["collective_gpu_ms"] for s in stats if s["collective_gpu_ms"] is not None]
    return CommStats(
        calls=len(stats),
        total_bytes=sum(s["bytes"] for s in stats),
        host_launch_ms=sum(s["host_launch_ms"] for s in stats),
        collective_gpu_ms=sum(gpu) if gpu else None,
        postprocess_host_ms=sum(s["postprocess_host_ms"] for s in stats),
    )


def _group(pg):
    return pg if pg is not None else dist.group.WORLD if dist.is_initialized() else None


def _record(op: str, t: torch.Tensor, group, fn, post=None):
    if not _PROFILING:
        fn()
        if post is not None:
            post()
        return
    meta = {
        "op": op,
        "bytes": t.numel() * t.element_size(),
        "dtype": str(t.dtype),
        "shape": list(t.shape),
        "world_size": dist.get_world_size(group) if group is not None else 1,
        "host_launch_ms": 0.0,
        "collective_gpu_ms": None,
        "postprocess_host_ms": 0.0,
    }
    t0 = time.perf_counter()
    if t.is_cuda:
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        fn()
        e.record()
        _PENDING.append((s, e, meta))
    else:
        fn()
    if post is not None:
        tp = time.perf_counter()
        post()
        meta["postprocess_host_ms"] = (time.perf_counter() - tp) * 1e3
    meta["host_launch_ms"] = (time.perf_counter() - t0) * 1e3
    _RECORDS.append(meta)


def register_comm(group, comm) -> None:
    """Route CUDA all_reduce on ``group`` through an NVLink communicator."""
    _COMMS[id(group)] = comm


def _nvlink_comm(group):
    return _COMMS.get(id(group))


def all_reduce(t: torch.Tensor, pg=None, op=dist.ReduceOp.SUM) -> torch.Tensor:
    """In-place sum across the TP group. Always returns ``t``."""
    group = _group(pg)
    if group is None:
        return t
    comm = _nvlink_comm(group)
    if (
        comm is not None
        and t.is_cuda
        and op == dist.ReduceOp.SUM
        and t.dtype in (torch.float32, torch.bfloat16)
        and t.is_contiguous()
        and t.numel() * t.element_size() <= comm.slot_bytes()
        and t.numel() > 0
    ):
        from minitp_b200 import _lib

        h = t.shape[-1] if t.dim() else 1
        rows = t.numel() // h

        def run():
            _lib.call("mtpb_allreduce", comm.handle, t.data_ptr(), rows, h,
                      _lib.dtype_code(t.dtype), _lib.stream_ptr(t.device))

        _record("all_reduce", t, group, run)
        return t
    _record("all_reduce", t, group, lambda: dist.all_reduce(t, op=op, group=group))
    return t


def all_gather(out: torch.Tensor, t: torch.Tensor, pg=None) -> torch.Tensor:
    group = _group(pg)
    if group is None:
        out.copy_(t)
        return out
    t = t.contiguous()
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    _record("all_gather", out, group, lambda: dist.all_gather(parts, t, group=group),
            lambda: out.copy_(torch.cat(parts, dim=-1)))
    return out


def all_gather_dim0(out: torch.Tensor, t: torch.Tensor, pg=None) -> torch.Tensor:
    group = _group(pg)
    if group is None:
        out.copy_(t.unsqueeze(0))
        return out
    t = t.contiguous()
    world = dist.get_world_size(group)
    if dist.get_backend(group) == "nccl":
        fn = lambda: dist.all_gather_into_tensor(out.reshape(world * t.numel()), t.reshape(-1), group=group)  # noqa: E731
    else:
        fn = lambda: dist.all_gather([out[i] for i in range(world)], t, group=group)  # noqa: E731
    _record("all_gather_dim0", out, group, fn)
    return out


def reduce_scatter(out: torch.Tensor, t: torch.Tensor, pg=None) -> torch.Tensor:
    group = _group(pg)
    if group is None:
        out.copy_(t)
        return out
    _record("reduce_scatter", t, group,
            lambda: dist.reduce_scatter_tensor(out, t.contiguous(), op=dist.ReduceOp.SUM, group=group))
    return out


def broadcast(t: torch.Tensor, src: int, pg=None) -> torch.Tensor:
    group = _group(pg)
    if group is None:
        return t
    _record("broadcast", t, group, lambda: dist.broadcast(t, src=src, group=group))
    return t
