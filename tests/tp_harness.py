"""Spawn N CPU/Gloo ranks and collect one picklable result per rank.

Generalises the reference's two-rank harness (tests/distributed/harness.py:41-62,
world size fixed at 2) to any world size. Worker functions must be
module-level. Each rank's return value comes back through a ``torch.save``
file, so tensors and numpy arrays are fine.
"""

from __future__ import annotations

import os
import socket
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def free_port() -> int:
    """A rendezvous port below Linux's ephemeral range (see tests/mp_worker.py)."""
    from tests.mp_worker import free_port as _free_port

    return _free_port()


def _worker(rank: int, world: int, fn, port: int, out_path: str, args: tuple, env: dict, init_pg: bool,
            timeout_s: float) -> None:
    os.environ.update(env)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    os.environ["LOCAL_RANK"] = str(rank)
    os.environ["MINITP_BACKEND"] = "gloo"
    os.environ.setdefault("USE_LIBUV", "0")
    torch.set_num_threads(max(1, (os.cpu_count() or 1) // world))
    import datetime as dt

    if init_pg:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=dt.timedelta(seconds=timeout_s))
    try:
        result = fn(rank, world, *args)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
    torch.save(result, f"{out_path}.{rank}")


def run_tp(world: int, fn, *args, env: dict | None = None, init_pg: bool = True,
           timeout_s: float = 600.0) -> dict[int, object]:
    """Run ``fn(rank, world, *args)`` on ``world`` Gloo ranks; returns {rank: result}.

    With ``init_pg=False`` the worker creates the process group itself (from
    the RANK / WORLD_SIZE / MASTER_* environment the harness sets).
    """
    port = free_port()
    out_path = os.path.join(tempfile.gettempdir(), f"mtpb_tp{world}_{os.getpid()}_{port}")
    try:
        mp.start_processes(
            _worker,
            args=(world, fn, port, out_path, args, dict(env or {}), init_pg, timeout_s),
            nprocs=world,
            join=True,
            start_method="spawn",
        )
        return {r: torch.load(f"{out_path}.{r}", weights_only=False) for r in range(world)}
    finally:
        for r in range(world):
            p = f"{out_path}.{r}"
            if os.path.exists(p):
                os.remove(p)
