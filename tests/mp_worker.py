"""Multi-process workers for the multi-GPU tests (one process per GPU).

Each worker initialises a torch.distributed group (NCCL for plumbing, the
IPC handle exchange), runs minitp_b200's NVLink kernels and returns numpy
results to the parent through a file.
"""

from __future__ import annotations

import datetime as dt
import os
import socket
import sys
import tempfile

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port() -> int:
    """A port for the rendezvous store, below Linux's ephemeral range (32768+).

    An ephemeral port found free here can be taken by another socket (NCCL's
    bootstrap uses ephemeral ports) before rank 0 binds it; ports outside that
    range are only taken by an explicit bind.
    """
    import random

    rng = random.Random(os.getpid() ^ int.from_bytes(os.urandom(4), "little"))
    for _ in range(200):
        port = rng.randrange(20000, 32000)
        with socket.socket() as s:
            try:
                s.bind(("127.0.0.1", port))
            except OSError:
                continue
        return port
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, fn, port, out, args):
    sys.path.insert(0, REPO)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=dt.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        res = fn(rank, world, *args)
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()
    np.savez(f"{out}.{rank}.npz", **res)


def run(world: int, fn, *args) -> list[dict]:
    for attempt in range(3):
        port = free_port()
        out = os.path.join(tempfile.gettempdir(), f"mtpb_mp_{os.getpid()}_{port}")
        try:
            mp.start_processes(_entry, args=(world, fn, port, out, args), nprocs=world, join=True,
                               start_method="spawn")
            break
        except mp.ProcessRaisedException as e:
            # the store's port was taken between the choice and the bind: choose again
            if "EADDRINUSE" not in str(e) or attempt == 2:
                raise
    res = []
    for r in range(world):
        with np.load(f"{out}.{r}.npz") as f:
            res.append({k: f[k] for k in f.files})
        os.remove(f"{out}.{r}.npz")
    return res


def ctx_for(rank, world):
    from minitp_b200.distributed.context import ParallelContext

    return ParallelContext(rank, rank, world, rank, world, torch.device("cuda", rank), dist.group.WORLD)


# ---------------------------------------------------------------------- #
# workers (module level: picklable under spawn)
# ---------------------------------------------------------------------- #
def w_generate(rank, world, name, dtype, n_layers_override=0, two_shot=False):
    from minitp_b200 import _lib
    from minitp_b200 import config as mcfg
    from minitp_b200.generation import generate_greedy
    from minitp_b200.synthetic import make_prompt
    from minitp_b200.weight_loader import load_synthetic_tp

    cfgs = {"tiny": (mcfg.baseline_tiny, 1, 8, 16), "q05b": (mcfg.qwen25_05b, 1, 128, 128),
            "q05b_b4": (mcfg.qwen25_05b, 4, 32, 16), "q7b_l2": (lambda: mcfg.qwen25_7b(2), 1, 16, 8)}
    fac, b, p, n = cfgs[name]
    cfg = fac()
    dt_ = torch.float32 if dtype == "fp32" else torch.bfloat16
    ctx = ctx_for(rank, world)
    if two_shot:  # every AllReduce site that is not fused into a projection takes the two-shot form
        _lib.call("mtpb_set_allreduce_two_shot", 0, 2)
    model = load_synthetic_tp(cfg, ctx, dtype=dt_, device=ctx.device)
    ids = make_prompt(cfg.vocab_size, b, p).cuda()
    logits = model(ids, positions=torch.arange(p, device="cuda"), gather_logits=True).float().cpu().numpy()
    out = generate_greedy(model, ids, n, early_stop=False)
    torch.cuda.synchronize()
    ctx.comm().raise_on_error()
    return {"tokens": out.cpu().numpy(), "prefill_last_logits": logits[:, -1],
            "decode_launches": np.array(decode_launches(model, b, p + n)),
            "heads_padded": np.array(bool(model.cfg.is_padded))}


def decode_launches(model, batch: int, cap: int) -> int:
    """Kernel launches of one decode step as the library plans it (1 = the megakernel)."""
    import ctypes

    from minitp_b200 import _lib

    nk = ctypes.c_int(0)
    _lib.call("mtpb_model_decode_kernels", model.native(), batch, cap, ctypes.byref(nk))
    return nk.value


def w_teacher(rank, world, name, fixture):
    """bf16 free-running ids plus teacher-forced decode top-2 (see tests/teacher.py)."""
    from minitp_b200 import config as mcfg
    from minitp_b200.generation import generate_greedy
    from minitp_b200.weight_loader import load_synthetic_tp
    from tests.teacher import teacher_forced_tops

    cfgs = {"q05b": mcfg.qwen25_05b}
    cfg = cfgs[name]()
    g = np.load(os.path.join(REPO, "tests", "golden", fixture))
    ctx = ctx_for(rank, world)
    model = load_synthetic_tp(cfg, ctx, dtype=torch.bfloat16, device=ctx.device)
    ids = torch.from_numpy(g["prompt"]).cuda()
    ref = torch.from_numpy(g["tokens"]).cuda()
    n = g["top2_values"].shape[0]
    out = generate_greedy(model, ids, n, early_stop=False)
    vals, tids, _ = teacher_forced_tops(model, ids, ref, n)
    torch.cuda.synchronize()
    ctx.comm().raise_on_error()
    return {"tokens": out.cpu().numpy(), "top_vals": vals, "top_ids": tids,
            "decode_launches": np.array(decode_launches(model, ids.shape[0], ids.shape[1] + n))}


def w_collectives(rank, world):
    """Fused AR, embedding and argmax against the reference fixtures at this world size."""
    from minitp_b200 import ops
    from minitp_b200.parallel.linear import shard_range
    from minitp_b200.synthetic_cases import argmax_logits, embedding_case, fused_ar_case
    from tests.golden.make_golden import big_vocab_cases

    ctx = ctx_for(rank, world)
    comm = ctx.comm()
    res = {}
    for rows in (1, 8, 64, 128, 512, 2048):
        partials, residual, gain = fused_ar_case(rows, 896, world, seed=1000 + rows)
        x, y = ops.allreduce_residual_rmsnorm(partials[rank].cuda(), residual.cuda(), gain.cuda(), 1e-6, comm)
        res[f"res_r{rows}"] = x.view(torch.int16).cpu().numpy()
        res[f"norm_r{rows}"] = y.view(torch.int16).cpu().numpy()
    for vocab in (151936, 151937):
        for batch in (1, 8, 64):
            table, ids = embedding_case(vocab, 896, batch, seed=vocab * 7 + batch)
            s, e = shard_range(vocab, rank, world)
            out = ops.embedding(ids.cuda(), table[s:e].contiguous().cuda(), s, e, vocab, comm)
            res[f"emb_v{vocab}_b{batch}"] = out.view(torch.int16).cpu().numpy()
            x = argmax_logits(vocab, batch, seed=vocab + batch)
            ids_out = ops.argmax(x[:, s:e].contiguous().cuda(), s, comm)
            res[f"argmax_v{vocab}_b{batch}"] = ids_out.squeeze(-1).cpu().numpy()
    vocab = 21_000_000
    s, e = shard_range(vocab, rank, world)
    res["argmax_big"] = np.array([int(ops.argmax(c[:, s:e].contiguous().cuda(), s, comm)) for c in big_vocab_cases()])
    torch.cuda.synchronize()
    comm.raise_on_error()
    return res


def w_two_shot(rank, world, name):
    """Prefill logits and greedy tokens of a model with its non-fused AllReduce sites one-shot, then
    two-shot (reduce-scatter + all-gather): both forms sum in rank order with the same rounding."""
    from minitp_b200 import _lib
    from minitp_b200 import config as mcfg
    from minitp_b200.generation import generate_greedy
    from minitp_b200.synthetic import make_prompt
    from minitp_b200.weight_loader import load_synthetic_tp

    cfgs = {"q05b": (mcfg.qwen25_05b, 1, 128, 16), "q7b_l2": (lambda: mcfg.qwen25_7b(2), 2, 64, 8)}
    fac, b, p, n = cfgs[name]
    cfg = fac()
    ctx = ctx_for(rank, world)
    model = load_synthetic_tp(cfg, ctx, dtype=torch.bfloat16, device=ctx.device)
    ids = make_prompt(cfg.vocab_size, b, p).cuda()
    res = {}
    for form, (min_bytes, min_world) in (("one", (-1, 2)), ("two", (0, 2))):
        _lib.call("mtpb_set_allreduce_two_shot", min_bytes, min_world)
        logits = model(ids, positions=torch.arange(p, device="cuda"), gather_logits=True)
        res[f"{form}_logits"] = logits.view(torch.int16).cpu().numpy()
        res[f"{form}_tokens"] = generate_greedy(model, ids, n, early_stop=False).cpu().numpy()
    _lib.call("mtpb_set_allreduce_two_shot", -1, 4)
    torch.cuda.synchronize()
    ctx.comm().raise_on_error()
    return res


def w_peer_timeout(rank, world):
    """Rank 1 skips one collective: rank 0's bounded wait must expire and report it.

    Both ranks stay between steps (no kernel of rank 1 is in flight while rank
    0 waits); the wait budget is 0.3 s.
    """
    from minitp_b200 import _lib, ops

    ctx = ctx_for(rank, world)
    comm = ctx.comm()
    comm.set_timeout(0.3)
    t = torch.ones(1, 896, device="cuda")
    ops.allreduce_(t, comm)  # both ranks: healthy
    torch.cuda.synchronize()
    ok_before = comm.status() == 0
    dist.barrier()
    raised = False
    if rank == 0:
        ops.allreduce_(torch.ones(1, 896, device="cuda"), comm)  # rank 1 never joins this one
        try:
            comm.raise_on_error()
        except _lib.PeerTimeoutError:
            raised = True
    dist.barrier()
    return {"ok_before": np.array(ok_before), "raised": np.array(raised), "first_sum": t.cpu().numpy()}
