"""Host-side multi-rank logic on CPU Gloo ranks (world size 2): no GPU needed.

Covers ``init_context`` from torchrun-style environment variables, the
collective wrappers' identity-return contract (reference
minitp/distributed/collectives.py:3-10), the IPC-handle exchange of the
NVLink communicator, and host-side failure detection: a rank that dies
before a collective makes the other rank fail with an error instead of
waiting forever.
"""

import time

import pytest
import torch

from tests.tp_harness import run_tp

pytestmark = pytest.mark.distributed


def _w_collectives(rank, world):
    from minitp_b200.distributed import all_gather, all_gather_dim0, all_reduce, broadcast
    from minitp_b200.distributed.context import init_context

    ctx = init_context()  # MINITP_BACKEND=gloo: CPU group from the environment
    assert ctx.tp_size == world and ctx.tp_rank == rank and ctx.device.type == "cpu"
    pg = ctx.process_group
    t = torch.full((2, 3), float(rank + 1))
    same = all_reduce(t, pg) is t
    g = torch.empty(2, 3 * world)
    same_g = all_gather(g, torch.full((2, 3), float(rank)), pg) is g
    d0 = torch.empty(world, 4)
    all_gather_dim0(d0, torch.full((4,), float(rank)), pg)
    b = broadcast(torch.full((3,), float(rank)), 0, pg)
    return {"same": same and same_g, "sum": t.tolist(), "gather": g.tolist(), "d0": d0.tolist(),
            "bcast": b.tolist()}


def test_init_context_and_collective_contract():
    res = run_tp(2, _w_collectives, init_pg=False)
    for r in range(2):
        assert res[r]["same"] is True
        assert res[r]["sum"] == [[3.0] * 3] * 2
        assert res[r]["gather"] == [[0.0] * 3 + [1.0] * 3] * 2
        assert res[r]["d0"] == [[0.0] * 4, [1.0] * 4]
        assert res[r]["bcast"] == [0.0] * 3


def _w_exchange(rank, world):
    import torch.distributed as dist

    from minitp_b200.comm import exchange_handles

    return list(exchange_handles(dist.group.WORLD, bytes([rank + 1]) * 64, world))


def test_ipc_handle_exchange_rank_order():
    res = run_tp(2, _w_exchange)
    want = [1] * 64 + [2] * 64
    assert res[0] == want and res[1] == want


def _w_dead_peer(rank, world):
    import torch.distributed as dist

    from minitp_b200.comm import exchange_handles

    if rank == 1:
        raise RuntimeError("rank 1 exits before the handle exchange")
    exchange_handles(dist.group.WORLD, bytes(64), world)  # the peer never joins
    return "unreachable"


def test_dead_peer_fails_the_exchange_instead_of_hanging():
    t0 = time.time()
    with pytest.raises(Exception):
        run_tp(2, _w_dead_peer, timeout_s=5.0)
    assert time.time() - t0 < 120


def test_exchange_rejects_bad_handle():
    from minitp_b200.comm import exchange_handles

    with pytest.raises(ValueError, match="64 bytes"):
        exchange_handles(None, b"x", 1)
