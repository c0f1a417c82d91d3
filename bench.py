"""Decode throughput of the B200 TP path: ``python bench.py --gpus N --steps K --warmup W``.

One step = one fixed-length greedy generation over a batch of synthetic
prompts at TP = N (one process per GPU under torchrun): the Qwen2.5-0.5B
shape (B=1, prompt 128, 128 new tokens) at N <= 2, the Qwen2.5-7B shape
(prompt 1024, 256 new tokens, B = 1, 8 and 32) at N >= 4; bf16, seeded
random weights. The prefill runs eagerly; the decode steps are replays of
the CUDA graph of the device-resident decode step, captured once per shape
during warm-up (the decode session ``generate_greedy`` keeps).

Reported (rank 0, one JSON line):
* value: decode tokens/s = B * decode steps / decode time, where the decode
  time is measured with CUDA events per step and the max over ranks is taken
  (the first batch of the run; the others under ``batches``).
* e2e: the same metric through ``generate_greedy``, starting from pinned host
  prompt ids and ending with the output ids copied back to the host.
* parity: before any timing, fp32 greedy generations of shapes whose
  reference fixtures are committed (tests/golden), compared token for token
  on every rank; a mismatch makes the run exit non-zero.
* roofline: the decode step (one megakernel launch per token when the
  library plans it): (weight + KV bytes read per token per rank) / time per
  token vs the measured HBM peak; roofline_gemv: the prefill GEMV on the
  LM-head weights; roofline_prefill_gemm: the tensor-core GEMM.
* N > 1: fused_ar (fused AllReduce + residual + RMSNorm vs NCCL all_reduce,
  next to the measured NVLink one-way latency) and embed_argmax (the masked
  embedding and the distributed argmax vs the reference's torch + NCCL
  formulation of the same operations).
* cpu_baseline (N=1): the reference's CPU path restated per rank
  (oracle/rank.py) on the host cores, on a bounded sample.
``--impl reference`` times that CPU path as the reference arm: one Gloo
process per rank with cores // N threads each (rank 0 of a torchrun launch
spawns them; the other ranks exit at once).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import socket
import statistics
import subprocess
import sys
import tempfile
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

MEASURED_PEAKS = os.path.join(REPO, "MEASURED_PEAKS.json")
GOLDEN = os.path.join(REPO, "tests", "golden")
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
NVLINK_GBS = 900.0  # nominal per direction per GPU


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--model", default=None, choices=["qwen2.5-0.5b", "qwen2.5-7b", "tiny"],
                   help="default: qwen2.5-0.5b at N <= 2, qwen2.5-7b at N >= 4")
    p.add_argument("--batch", type=int, default=None, help="one batch size (default: 1; 7B: 1, 8, 32)")
    p.add_argument("--prompt", type=int, default=None)
    p.add_argument("--new-tokens", type=int, default=None)
    p.add_argument("--dtype", default="bf16", choices=["bf16", "fp32"])
    p.add_argument("--gen-device", default=None, help="where synthetic weights are drawn (cpu|cuda)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true")
    p.add_argument("--no-collectives", action="store_true", help="N > 1: skip the fused_ar / embed_argmax blocks")
    p.add_argument("--no-pdl", action="store_true")
    p.add_argument("--out", default=None, help="also write the JSON line here")
    p.add_argument("--workload", default="decode", choices=["decode", "fused_ar", "prefill_gemm"],
                   help="decode (default), the fused AllReduce+residual+RMSNorm microbenchmark alone, or the "
                        "tensor-core prefill GEMM sweep")
    p.add_argument("--gemm-shapes", default=None,
                   help="prefill_gemm: comma-separated names of the shapes to run (default: all)")
    p.add_argument("--iters", type=int, default=10000, help="fused_ar: iterations per size")
    return p.parse_args(argv)


def workload(args, world: int):
    """(model name, config, prompt length, new tokens, batch sizes)."""
    from minitp_b200 import config as mcfg

    name = args.model or ("qwen2.5-0.5b" if world <= 2 else "qwen2.5-7b")
    if name == "qwen2.5-7b":
        cfg, prompt, new, batches = mcfg.qwen25_7b(), 1024, 256, [1, 8, 32]
    elif name == "tiny":
        cfg, prompt, new, batches = mcfg.baseline_tiny(), 8, 16, [1]
    else:
        cfg, prompt, new, batches = mcfg.qwen25_05b(), 128, 128, [1]
    if args.batch:
        batches = [args.batch]
    return name, cfg, args.prompt or prompt, args.new_tokens or new, batches


def peaks():
    try:
        with open(MEASURED_PEAKS) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def peak_tflops():
    """Dense bf16 peak: the burst cuBLAS figure (a GEMM timed alone)."""
    try:
        with open(MEASURED_PEAKS) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (burst)"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


def free_port() -> int:
    """A rendezvous port below Linux's ephemeral range (32768+), so NCCL/Gloo sockets cannot take it."""
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


def time_prefill_gemm(epi: str, M: int, N: int, K: int, dev, reps: int = 20) -> dict:
    """Device time per launch of the tensor-core GEMM (gemm_tc_kernel).

    `epi` "swiglu" runs ops.linear_swiglu (N = 2 x intermediate rows of W),
    "store" runs ops.linear. The launches are captured in a CUDA graph so the
    host does not pace them, and they cycle over enough distinct weight copies
    (> 256 MiB in all) that every launch reads its weights from HBM, not L2.
    """
    from minitp_b200 import ops

    wbytes = N * K * 2
    copies = max(2, min(64, (256 << 20) // wbytes + 1))
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    ws = [(torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16) for _ in range(copies)]
    fn = (lambda w: ops.linear_swiglu(x, w)) if epi == "swiglu" else (lambda w: ops.linear(x, w))
    for w in ws[:3]:
        fn(w)  # eager calls set the kernel attributes before capture
    torch.cuda.synchronize()
    n = max(reps, copies)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(n):
            fn(ws[i % copies])
    graph.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(3):
        graph.replay()
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1e3 / (3 * n)
    del graph
    flops = 2.0 * M * N * K
    peak, peak_kind = peak_tflops()
    tflops = flops / (us * 1e-6) / 1e12
    byts = wbytes + M * K * 2 + M * (N // 2 if epi == "swiglu" else N) * 2
    return {"bound": "tensor", "kernel": f"gemm_tc_kernel ({epi})", "M": M, "N": N, "K": K,
            "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s", "frac": round(tflops / peak, 4),
            "peak_kind": peak_kind, "us_per_launch": round(us, 3), "flops_per_launch": flops,
            "hbm_gbs": round(byts / (us * 1e-6) / 1e9, 1), "bytes_per_launch": byts,
            "timing": f"CUDA graph of {n} launches over {copies} weight copies, CUDA events"}


# ---------------------------------------------------------------------- #
# clocks
# ---------------------------------------------------------------------- #
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.path = tempfile.mktemp(prefix="mtpb_clocks_", suffix=".csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.idx)], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.remove(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------- #
# bytes per token, launches
# ---------------------------------------------------------------------- #
def weight_bytes_per_token(model) -> int:
    """Weight bytes one decode step streams on this rank (all GEMV weights + LM head)."""
    n = model.lm_head.weight.numel()
    for layer in model.model.layers:
        a, m = layer.self_attn, layer.mlp
        n += a.qkv_proj.weight.numel() + a.o_proj.weight.numel()
        n += m.gate_up_proj.weight.numel() + m.down_proj.weight.numel()
    return n * model.lm_head.weight.element_size()


def kv_bytes_per_token(model, batch: int, avg_len: float) -> float:
    a = model.model.layers[0].self_attn
    per_pos = 2 * a.kv_heads_local * a.head_dim * model.lm_head.weight.element_size()
    return per_pos * avg_len * batch * len(model.model.layers)


# DRAM bytes (read + write) of one decode-step launch measured by ncu
# (dram__bytes_read.sum + dram__bytes_write.sum), keyed by (model, batch, TP,
# kernel revision). Configurations without a capture of the current kernel
# report null.
MK_TRAFFIC: dict = {("qwen2.5-0.5b", 1, 1, 2): 994_579_200, ("qwen2.5-0.5b", 1, 1, 3): 994_149_376}
MK_REVISION = 3


def measured_traffic(model_name: str, batch: int, world: int, step_launches: int):
    if step_launches != 1:
        return None
    return MK_TRAFFIC.get((model_name, batch, world, MK_REVISION))


def decode_launches(model, batch: int, cap: int) -> int:
    from minitp_b200 import _lib

    nk = ctypes.c_int(0)
    _lib.call("mtpb_model_decode_kernels", model.native(), batch, cap, ctypes.byref(nk))
    return nk.value


def prefill_launch_count(n_layers: int, chunks: int, consume_pass: bool) -> int:
    """Kernel launches of a prefill through the kernel chain.

    Per chunk: the embedding, 5 per layer (QKV, attention, O, gate/up, down)
    and, when the chunk's rows do not fit the GEMV's shared-memory staging, a
    separate AllReduce-consume pass in front of QKV and gate/up; then the
    final norm's consume pass and the LM head of the last chunk.
    """
    per_chunk = 1 + 5 * n_layers + (2 * n_layers if consume_pass else 0)
    return chunks * per_chunk + (1 if consume_pass else 0) + 1


def launches_per_generation(prefill: int, new_tokens: int, step_launches: int) -> int:
    """Launches of one fixed-length generation: the prefill, the greedy pick of its
    last position (argmax rows + finish), the decode position seed and the decode
    steps (`step_launches` each: 1 when the decode megakernel runs them)."""
    return prefill + 2 + 1 + (new_tokens - 1) * step_launches


def prefill_launches(model, batch: int, prompt_len: int, comm) -> int:
    """Prefill launches for this model and shape (chunked by the communicator slot)."""
    cfg = model.cfg
    esz = model.lm_head.weight.element_size()
    row = batch * cfg.hidden_size * esz
    tc = max(1, min(prompt_len, comm.slot_bytes() // row))
    consume = batch * tc * cfg.hidden_size * esz > 64 * 1024  # GEMV x staging limit
    return prefill_launch_count(cfg.num_hidden_layers, math.ceil(prompt_len / tc), consume)


# ---------------------------------------------------------------------- #
# parity before timing
# ---------------------------------------------------------------------- #
# name: (config factory, batch, prompt, new tokens); fp32 runs whose reference
# ids are committed in tests/golden
PARITY_MODELS = {
    "q05b": ("qwen25_05b", None, 1, 128, 128),
    "q05b_b4": ("qwen25_05b", None, 4, 32, 16),
    "q7b_l2": ("qwen25_7b", 2, 1, 16, 8),
}
# world -> [(run, fixture)]: the reference's own TP=N run where one exists;
# at TP=8 (and 0.5B at TP=4) the reference rejects the head count, so the
# padded runs are held to the reference's TP=1 ids
PARITY_RUNS = {
    1: [("q05b", "model_q05b_tp1_fp32.npz")],
    2: [("q05b", "model_q05b_tp2_fp32.npz"), ("q05b_b4", "model_q05b_b4_tp2_fp32.npz")],
    4: [("q7b_l2", "model_q7b_l2_tp4_fp32.npz"), ("q05b_b4", "model_q05b_b4_tp1_fp32.npz")],
    8: [("q7b_l2", "model_q7b_l2_tp1_fp32.npz"), ("q05b_b4", "model_q05b_b4_tp1_fp32.npz")],
}


def run_parity(ctx, world: int) -> list[dict]:
    import numpy as np
    import torch.distributed as dist

    from minitp_b200 import config as mcfg
    from minitp_b200.generation import generate_greedy
    from minitp_b200.weight_loader import load_synthetic_tp

    out = []
    for run, fixture in PARITY_RUNS.get(world, []):
        fac, layers, b, p, n = PARITY_MODELS[run]
        cfg = getattr(mcfg, fac)(layers) if layers else getattr(mcfg, fac)()
        model = load_synthetic_tp(cfg, ctx, dtype=torch.float32, device=ctx.device)
        with np.load(os.path.join(GOLDEN, fixture)) as g:
            prompt, want = torch.from_numpy(g["prompt"]), torch.from_numpy(g["tokens"])
        got = generate_greedy(model, prompt.to(ctx.device), n, early_stop=False)
        launches = decode_launches(model, b, p + n)
        ctx.comm().raise_on_error()
        equal = torch.tensor([int(torch.equal(got.cpu(), want))], device=ctx.device)
        if world > 1:
            allg = [torch.empty_like(got) for _ in range(world)]
            dist.all_gather(allg, got.contiguous())
            agree = all(torch.equal(x, allg[0]) for x in allg)
            dist.all_reduce(equal, op=dist.ReduceOp.MIN)
        else:
            agree = True
        out.append({"run": run, "fixture": fixture, "tp": world, "dtype": "fp32",
                    "tokens_equal": bool(equal.item()), "ranks_agree": bool(agree),
                    "new_tokens": n, "decode_launches": launches, "heads_padded": bool(model.cfg.is_padded)})
        model.release_native()
        del model, got
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------- #
# decode timing
# ---------------------------------------------------------------------- #
def decode_bench(model, ctx, model_name, batch, prompt_len, new_tokens, args, flush, with_e2e):
    """Device-timed decode (graph replays of the session's captured step), step time, e2e."""
    import torch.distributed as dist

    from minitp_b200.generation import GenerationState, decode_session, generate_greedy
    from minitp_b200.synthetic import make_prompt

    dev = ctx.device
    world = ctx.tp_size
    ids_host = make_prompt(model.cfg.vocab_size, batch, prompt_len).pin_memory()
    ids = ids_host.to(dev)
    sess = decode_session(model, batch, prompt_len + new_tokens, dev)

    def one_step():
        st = GenerationState(model, ids, new_tokens, session=sess)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        logits = st.prefill(last_only=True)
        tok = st.select_next(logits)
        ev[3].record()  # time to first token: prefill + greedy pick of its last position
        st.append(tok)
        st.start_device_decode(tok)
        replays = new_tokens - 1
        if st._graph is None:  # the first call of the shape: eager step, then capture (warm-up)
            st.device_step()
            st.capture()
            replays -= 1
        ev[1].record()
        for _ in range(replays):
            st.graph_step()
        ev[2].record()
        return st, ev, replays

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(1, args.warmup)):
        st, _, _ = one_step()
        st.release()
        flush.zero_()
    barrier()
    ctx.comm().raise_on_error()

    sampler = ClockSampler(dev.index if dev.index is not None else 0)
    sampler.start()
    decode_ms, step_ms, ttft_ms = [], [], []
    barrier()
    for _ in range(args.steps):
        flush.zero_()  # L2 flush between timed steps (256 MiB > 126 MB L2)
        st, ev, replays = one_step()
        torch.cuda.synchronize()
        decode_ms.append(ev[1].elapsed_time(ev[2]) / max(1, replays))
        step_ms.append(ev[0].elapsed_time(ev[2]))
        ttft_ms.append(ev[0].elapsed_time(ev[3]))
        st.release()
    barrier()
    clocks = sampler.stop()
    ctx.comm().raise_on_error()
    t = torch.tensor([statistics.mean(decode_ms), statistics.mean(step_ms), statistics.mean(ttft_ms)],
                     dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_token, ms_per_step, ttft = t.tolist()
    res = {"batch": batch, "ms_per_token": ms_per_token, "ms_per_step": ms_per_step, "ttft_ms": ttft, "clocks": clocks,
           "tok_s": batch / (ms_per_token / 1e3), "launches": decode_launches(model, batch, prompt_len + new_tokens),
           "prefill_launches": prefill_launches(model, batch, prompt_len, ctx.comm())}
    if with_e2e:
        e2e_ms = []
        e2e_warm = 1
        for i in range(e2e_warm + max(2, min(args.steps, 5))):
            flush.zero_()
            barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = generate_greedy(model, ids_host.to(dev, non_blocking=True), new_tokens, early_stop=False)
            out.to("cpu", non_blocking=False)
            e.record()
            torch.cuda.synchronize()
            if i >= e2e_warm:
                e2e_ms.append(s.elapsed_time(e))
        te = torch.tensor([statistics.mean(e2e_ms)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        res["e2e"] = {"value": round(batch * new_tokens / (te.item() / 1e3), 2), "unit": "tok/s",
                      "h2d_bytes_per_step": ids_host.numel() * ids_host.element_size(),
                      "d2h_bytes_per_step": batch * (prompt_len + new_tokens) * 8,
                      "definition": "generate_greedy from pinned host ids to host output ids, incl. prefill",
                      "warmup": e2e_warm, "samples_ms": [round(x, 3) for x in e2e_ms]}
    return res


# ---------------------------------------------------------------------- #
# collectives (N > 1)
# ---------------------------------------------------------------------- #
def _graph_time_us(fn, reps_total: int, chunk: int, dev) -> float:
    """Device time per call of `fn`, replayed from a CUDA graph of `chunk` calls (max over ranks)."""
    import torch.distributed as dist

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(chunk):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    reps = max(1, reps_total // chunk)
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    s.record()
    for _ in range(reps):
        graph.replay()
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1e3 / (reps * chunk)
    del graph
    t = torch.tensor([us], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def nvlink_floor(ctx, iters: int = 20000, warm: int = 1000) -> dict:
    """One-way latency of one 8-byte LL word between ranks 0 and 1 (ping-pong, device-timed)."""
    import torch.distributed as dist

    from minitp_b200 import _lib

    comm = ctx.comm()
    ns = torch.zeros(1, dtype=torch.int64, device=ctx.device)
    dist.barrier()
    if ctx.tp_rank in (0, 1):
        _lib.call("mtpb_comm_pingpong", comm.handle, 1 - ctx.tp_rank, iters, warm, ns.data_ptr(),
                  _lib.stream_ptr(ctx.device))
    torch.cuda.synchronize()
    dist.all_reduce(ns, op=dist.ReduceOp.MAX)
    comm.raise_on_error()
    rt = ns.item() / (iters - warm) / 1e3
    return {"one_way_us": round(rt / 2, 3), "round_trip_us": round(rt, 3), "iters": iters - warm,
            "how": "one 8-byte LL word bounced between ranks 0 and 1 over NVLink, %globaltimer on the device"}


def fused_ar_block(ctx, iters: int, floor_us: float | None) -> list[dict]:
    """Fused AllReduce + residual + RMSNorm vs NCCL all_reduce, [rows, 896] bf16."""
    import torch.distributed as dist

    from minitp_b200 import _lib
    from minitp_b200.synthetic_cases import fused_ar_case

    comm = ctx.comm()
    dev = ctx.device
    world = ctx.tp_size
    out = []
    for rows in (1, 8, 64, 128, 512, 2048):
        partials, residual, gain = fused_ar_case(rows, 896, world, seed=1000 + rows)
        p = partials[ctx.tp_rank].to(dev)
        r = residual.to(dev)
        g = gain.to(dev)
        out_res = torch.empty_like(p)
        out_norm = torch.empty_like(p)
        nccl_t = p.clone()

        def fused():
            _lib.call("mtpb_allreduce_residual_rmsnorm", comm.handle, p.data_ptr(), r.data_ptr(), g.data_ptr(),
                      None, out_res.data_ptr(), out_norm.data_ptr(), rows, 896, 1e-6, _lib.MTPB_BF16,
                      _lib.stream_ptr(dev))

        def nccl():
            dist.all_reduce(nccl_t)

        f_us = _graph_time_us(fused, iters, 100, dev)
        n_us = _graph_time_us(nccl, iters, 100, dev)
        comm.raise_on_error()
        m = rows * 896 * 2
        line = {"rows": rows, "bytes": m, "fused_us": round(f_us, 3), "nccl_allreduce_us": round(n_us, 3),
                "ratio_fused_over_nccl": round(f_us / n_us, 3),
                "fused_send_gbs": round((world - 1) * m / (f_us * 1e-6) / 1e9, 2),
                "fused_send_frac_of_900": round((world - 1) * m / (f_us * 1e-6) / 1e9 / NVLINK_GBS, 4),
                "iters": max(1, iters // 100) * 100}
        if floor_us:
            line["fused_over_floor"] = round(f_us / floor_us, 2)
        out.append(line)
    torch.cuda.synchronize()
    dist.barrier()
    return out


def embed_argmax_block(ctx, iters: int = 2000) -> list[dict]:
    """Vocab-parallel embedding + distributed argmax vs the reference's formulation.

    Ours: ops.embedding (masked local lookup + NVLink reduce in one kernel) and
    ops.argmax (packed-key argmax over the shard + O(tp) NVLink gather). The
    reference's (minitp/parallel/embedding.py:44-50, 118-172): F.embedding of
    the masked ids, a mask multiply and an NCCL all_reduce; NaN cleanup, a
    local max, the bitpack key and an NCCL all_gather_into_tensor. Both run
    from CUDA graphs on the same box; ids and embeddings are compared.
    """
    import torch.distributed as dist
    import torch.nn.functional as F

    from minitp_b200 import ops
    from minitp_b200.parallel.linear import shard_range
    from minitp_b200.synthetic_cases import argmax_logits

    comm = ctx.comm()
    dev = ctx.device
    world, rank = ctx.tp_size, ctx.tp_rank
    hbm, _ = peaks()
    out = []
    for vocab in (151936, 151937):
        s, e = shard_range(vocab, rank, world)
        gen = torch.Generator(device=dev)
        gen.manual_seed(vocab)
        table = (torch.randn(e - s, 896, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        for batch in (1, 8, 64):
            g = torch.Generator().manual_seed(vocab * 7 + batch)
            ids = torch.randint(0, vocab, (batch, 1), generator=g).to(dev)
            logits = argmax_logits(vocab, batch, seed=vocab + batch)[:, s:e].contiguous().to(dev)
            gather_buf = torch.empty(world, batch, dtype=torch.int64, device=dev)

            def ref_embed():
                mask = (ids >= s) & (ids < e)
                x = F.embedding((ids - s) * mask, table) * mask.unsqueeze(-1).to(table.dtype)
                dist.all_reduce(x)
                return x

            def ref_argmax():
                clean = torch.where(torch.isnan(logits), torch.full_like(logits, float("-inf")), logits)
                values, idx = clean.max(dim=-1)
                gid = idx + s
                vals = torch.where(values == 0, torch.zeros_like(values), values)
                bits = vals.float().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
                key = torch.where(bits < 0x80000000, bits, ((~bits) & 0xFFFFFFFF) - 0x80000000)
                packed = (key << 32) | (0xFFFFFFFF - gid.to(torch.int64))
                dist.all_gather_into_tensor(gather_buf, packed)
                winner = gather_buf.max(dim=0).values
                return 0xFFFFFFFF - (winner & 0xFFFFFFFF)

            mine_e = ops.embedding(ids, table, s, e, vocab, comm)
            mine_a = ops.argmax(logits, s, comm).view(-1)
            ref_e, ref_a = ref_embed(), ref_argmax()
            torch.cuda.synchronize()
            t = {
                "embed_us": _graph_time_us(lambda: ops.embedding(ids, table, s, e, vocab, comm), iters, 50, dev),
                "ref_embed_us": _graph_time_us(ref_embed, iters, 50, dev),
                "argmax_us": _graph_time_us(lambda: ops.argmax(logits, s, comm), iters, 50, dev),
                "ref_argmax_us": _graph_time_us(ref_argmax, iters, 50, dev),
            }
            comm.raise_on_error()
            read = batch * (e - s) * 4
            out.append({"vocab": vocab, "batch": batch, **{k: round(v, 3) for k, v in t.items()},
                        "embed_equal": bool(torch.equal(mine_e, ref_e)), "ids_equal": bool(torch.equal(mine_a, ref_a)),
                        "argmax_read_bytes": read, "argmax_hbm_gbs": round(read / (t["argmax_us"] * 1e-6) / 1e9, 1),
                        "argmax_frac_of_hbm": round(read / (t["argmax_us"] * 1e-6) / 1e9 / hbm, 4)})
    torch.cuda.synchronize()
    dist.barrier()
    return out


# ---------------------------------------------------------------------- #
# the reference's CPU path (Gloo ranks)
# ---------------------------------------------------------------------- #
def _ref_worker(rank, world, port, out_path, cfg_kw, dtype_name, batch, prompt_len, sample, fill_cache, threads,
                warmup, steps):
    import torch.distributed as dist

    from oracle.model import OracleConfig
    from oracle.rank import OracleRank

    torch.set_num_threads(threads)
    if world > 1:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg = OracleConfig(**cfg_kw)
        dt = torch.bfloat16 if dtype_name == "bf16" else torch.float32
        t0 = time.perf_counter()
        m = OracleRank(cfg, rank, world, dtype=dt, weights="fill")
        build_s = time.perf_counter() - t0
        g = torch.Generator().manual_seed(0)
        ids = torch.randint(0, cfg.vocab_size, (batch, prompt_len), generator=g)
        times = []
        for i in range(warmup + steps):
            if fill_cache:
                m.reset(batch, prompt_len + sample + 1, fill_len=prompt_len)
                tok = ids[:, -1]
            else:
                m.reset(batch, prompt_len + sample + 1)
                tok = m.select(m.forward(ids)[:, -1])
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            for _ in range(sample):
                tok = m.select(m.forward(tok[:, None])[:, -1])
            dt_s = time.perf_counter() - t0
            if i >= warmup:
                times.append(dt_s)
        torch.save({"times": times, "build_s": build_s}, f"{out_path}.{rank}")
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


def cpu_reference(cfg, world: int, dtype_name: str, batch: int, prompt_len: int, sample: int, fill_cache: bool,
                  warmup: int, steps: int) -> dict:
    """Decode tok/s of the reference's CPU path: `world` Gloo processes, cores // world threads each."""
    import torch.multiprocessing as mp

    cores = os.cpu_count() or 1
    threads = max(1, cores // world)
    cfg_kw = {k: getattr(cfg, k) for k in (
        "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
        "head_dim", "vocab_size", "rms_norm_eps", "rope_theta", "max_position_embeddings", "tie_word_embeddings")}
    port = free_port()
    out_path = os.path.join(tempfile.gettempdir(), f"mtpb_ref_{os.getpid()}_{port}")
    if world > 1:
        mp.start_processes(_ref_worker, args=(world, port, out_path, cfg_kw, dtype_name, batch, prompt_len, sample,
                                              fill_cache, threads, warmup, steps),
                           nprocs=world, join=True, start_method="spawn")
    else:
        _ref_worker(0, 1, port, out_path, cfg_kw, dtype_name, batch, prompt_len, sample, fill_cache, threads,
                    warmup, steps)
    res = []
    for r in range(world):
        res.append(torch.load(f"{out_path}.{r}", weights_only=False))
        os.remove(f"{out_path}.{r}")
    per_step = [max(x["times"][i] for x in res) for i in range(steps)]  # max over ranks
    value = batch * sample / statistics.median(per_step)
    how = (f"KV cache pre-filled to {prompt_len} positions (no CPU prefill)" if fill_cache
           else f"prefill of {prompt_len} untimed")
    return {"value": value, "cores": threads * world, "threads_per_rank": threads, "ranks": world,
            "sample": f"per step: {how}, then {sample} timed greedy decode steps of batch {batch}; "
                      f"{world} Gloo process(es) x {threads} threads; max over ranks; median of {steps} steps",
            "timed_s": round(sum(per_step), 2)}


def reference_sample(cfg, prompt_len: int, new_tokens: int) -> tuple[int, bool]:
    """(decode steps per sample, pre-fill the KV cache instead of a CPU prefill)."""
    params = cfg.num_hidden_layers * cfg.hidden_size * (4 * cfg.hidden_size + 3 * cfg.intermediate_size)
    if params > 2e9:  # 7B: a CPU prefill of the prompt would take minutes
        return 3, True
    return min(32, max(1, new_tokens - 1)), False


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # rank 0 runs the Gloo ranks itself
    world = args.gpus
    name, cfg, prompt_len, new_tokens, batches = workload(args, world)
    batch = batches[0]
    if cfg.num_attention_heads % world:
        # minitp/config.py:50-61 (ModelConfig.validate)
        msg = f"ValueError: num_attention_heads={cfg.num_attention_heads} not divisible by tp_size={world}"
        print(json.dumps({"impl": "reference", "unavailable": f"the reference rejects {name} at TP={world}: {msg}",
                          "n_gpus": world}), flush=True)
        return
    sample, fill = reference_sample(cfg, prompt_len, new_tokens)
    r = cpu_reference(cfg, world, args.dtype, batch, prompt_len, sample, fill, max(1, args.warmup), args.steps)
    value = r["value"]
    line = {
        "impl": "reference", "metric": "decode tok/s", "value": round(value, 3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * batch * sample / value, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": args.dtype, "data": "synthetic (random weights, uniform prompt ids)",
        "config": {"workload": f"{name} decode, B={batch}, prompt {prompt_len}, {new_tokens} new tokens, TP={world}",
                   "model": name, "global_batch": batch, "seq_len": prompt_len + new_tokens,
                   "parallelism": f"tp{world} (Gloo CPU ranks)"},
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": r["cores"], "kind": "port",
                         "sample": r["sample"] + "; oracle/rank.py restates the reference's per-rank CPU path"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------- #
# B200 arm
# ---------------------------------------------------------------------- #
def run_b200(args):
    import torch.distributed as dist

    from minitp_b200 import _lib, ops
    from minitp_b200.build import build
    from minitp_b200.distributed.context import init_context
    from minitp_b200.weight_loader import load_synthetic_tp

    if int(os.environ.get("RANK", "0")) == 0:
        build()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    ctx = init_context(timeout_s=120.0)
    if world > 1:
        dist.barrier()  # rank 0 built the library before anyone loads it
    lib = _lib.load()
    if args.no_pdl:
        lib.mtpb_set_pdl(0)
    dev = ctx.device
    name, cfg, prompt_len, new_tokens, batches = workload(args, world)
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32

    parity = [] if args.no_parity else run_parity(ctx, world)
    parity_ok = all(x["tokens_equal"] and x["ranks_agree"] for x in parity)

    gen_dev = args.gen_device or ("cuda" if name == "qwen2.5-7b" else "cpu")
    model = load_synthetic_tp(cfg, ctx, dtype=dtype, device=dev, seed=0, gen_device=gen_dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    runs = []
    for i, b in enumerate(batches):
        runs.append(decode_bench(model, ctx, name, b, prompt_len, new_tokens, args, flush, with_e2e=(i == 0)))
    main = runs[0]
    batch = main["batch"]
    ms_per_token = main["ms_per_token"]
    step_launches = main["launches"]

    # the prefill GEMV, timed live: the LM-head weights over this rank's vocab shard
    x = torch.randn(batch, cfg.hidden_size, device=dev).to(dtype)
    w = model.lm_head.weight
    for _ in range(3):
        ops.linear(x, w)
    reps = 50
    ks, ke = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    flush.zero_()
    torch.cuda.synchronize()
    ks.record()
    for _ in range(reps):
        ops.linear(x, w)
    ke.record()
    torch.cuda.synchronize()
    k_ms = ks.elapsed_time(ke) / reps
    peak, peak_kind = peaks()
    k_bytes = w.numel() * w.element_size() + x.numel() * x.element_size() + batch * w.shape[0] * w.element_size()
    k_gbs = k_bytes / (k_ms / 1e3) / 1e9

    gu = model.model.layers[0].mlp.gate_up_proj.weight
    tc_line = None
    if dtype == torch.bfloat16 and batch * prompt_len >= 64:
        tc_line = time_prefill_gemm("swiglu", batch * prompt_len, gu.shape[0], gu.shape[1], dev)

    wb = weight_bytes_per_token(model)
    kvb = kv_bytes_per_token(model, batch, prompt_len + new_tokens / 2)
    tok_gbs = (wb + kvb) / (ms_per_token / 1e3) / 1e9

    coll = {}
    if world > 1 and not args.no_collectives:
        floor = nvlink_floor(ctx)
        coll["nvlink_floor"] = floor
        coll["fused_ar"] = fused_ar_block(ctx, args.iters, floor["one_way_us"])
        coll["embed_argmax"] = embed_argmax_block(ctx)

    line = None
    if ctx.is_rank_zero:
        line = {
            "metric": "decode tok/s", "value": round(main["tok_s"], 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(main["ms_per_step"], 4),
            "us_per_token": round(ms_per_token * 1e3, 3), "ttft_ms": round(main["ttft_ms"], 3),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": args.dtype,
            "data": "synthetic (seeded random weights N(0,0.02) and uniform prompt ids)",
            "config": {
                "workload": f"{name} decode, B={batch}, prompt {prompt_len}, {new_tokens} new tokens, TP={world}",
                "model": name, "global_batch": batch, "seq_len": prompt_len + new_tokens,
                "parallelism": f"tp{world}", "heads_padded": bool(model.cfg.is_padded),
                "l2": "flushed between timed steps (256 MiB write)",
                "decode": ("CUDA graph replay of the device-resident decode step (persistent megakernel)"
                           if step_launches == 1 else f"CUDA graph replay of the kernel chain ({step_launches} "
                                                      "launches per step)"),
                "step": "prefill (eager) + greedy selection + decode graph replays; graph captured in warm-up",
            },
            "e2e": main["e2e"],
            "parity": parity,
            "roofline": {"bound": "hbm",
                         "kernel": "decode_mk_kernel" if step_launches == 1 else "decode kernel chain",
                         "achieved": round(tok_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(tok_gbs / peak, 4),
                         "traffic": measured_traffic(name, batch, world, step_launches),
                         "peak_kind": peak_kind,
                         "bytes_per_launch": round(wb + kvb), "weight_bytes": wb, "kv_bytes": round(kvb),
                         "us_per_launch": round(ms_per_token * 1e3, 3),
                         "timing": "CUDA events over the graph replays of the decode step"},
            "roofline_gemv": {"bound": "hbm", "kernel": "gemv_kernel (LM-head weights, prefill GEMV)",
                              "achieved": round(k_gbs, 1), "peak": peak, "unit": "GB/s",
                              "frac": round(k_gbs / peak, 4), "bytes_per_launch": k_bytes,
                              "us_per_launch": round(k_ms * 1e3, 3)},
            "roofline_prefill_gemm": tc_line,
            "gpu_launches": launches_per_generation(main["prefill_launches"], new_tokens, step_launches) * args.steps,
            "clocks": main["clocks"],
        }
        if len(runs) > 1:
            line["batches"] = []
            for r in runs:
                kv_r = kv_bytes_per_token(model, r["batch"], prompt_len + new_tokens / 2)
                gbs = (wb + kv_r) / (r["ms_per_token"] / 1e3) / 1e9
                line["batches"].append({
                    "batch": r["batch"], "tok_s": round(r["tok_s"], 2), "us_per_token": round(r["ms_per_token"] * 1e3, 3),
                    "ttft_ms": round(r["ttft_ms"], 3),
                    "ms_per_step": round(r["ms_per_step"], 3), "decode_launches_per_token": r["launches"],
                    "decode_path": "megakernel" if r["launches"] == 1 else "kernel chain",
                    "roofline_frac": round(gbs / peak, 4), "bytes_per_token": round(wb + kv_r), "clocks": r["clocks"]})
        line.update(coll)
        if world == 1 and not args.no_cpu_baseline:
            sample, fill = reference_sample(cfg, prompt_len, new_tokens)
            r = cpu_reference(cfg, 1, args.dtype, batch, prompt_len, sample, fill, 1, 3)
            line["cpu_baseline"] = {"value": round(r["value"], 3), "unit": "tok/s", "cores": r["cores"],
                                    "kind": "port", "sample": r["sample"] + "; oracle/rank.py (the reference's "
                                                                            "per-rank CPU path restated)"}
    if world > 1:
        dist.barrier()
    model.release_native()
    if line is not None:
        s = json.dumps(line)
        print(s, flush=True)
        if args.out:
            with open(args.out, "w") as f:
                f.write(s + "\n")
    ctx.destroy()
    if not parity_ok:
        print("parity: a fixture's greedy ids were not reproduced", file=sys.stderr, flush=True)
        sys.exit(3)


def run_fused_ar(args):
    """The fused AllReduce microbenchmark alone: one JSON line per size on rank 0."""
    import torch.distributed as dist

    from minitp_b200.build import build
    from minitp_b200.distributed.context import init_context

    if int(os.environ.get("RANK", "0")) == 0:
        build()
    ctx = init_context(timeout_s=120.0)
    if ctx.tp_size < 2:
        if ctx.is_rank_zero:
            print(json.dumps({"workload": "fused_ar", "skipped": "needs >= 2 GPUs"}))
        return
    dist.barrier()
    floor = nvlink_floor(ctx)
    for line in fused_ar_block(ctx, args.iters, floor["one_way_us"]):
        if ctx.is_rank_zero:
            print(json.dumps({"workload": "fused_ar", "tp": ctx.tp_size, "nvlink_one_way_us": floor["one_way_us"],
                              **line}), flush=True)
    ctx.destroy()


# (name, epilogue, M, N, K): prefill projections of the two model shapes.
# 0.5B: gate/up (2 x 4864) and down at the 128-token prompt and a 2048-token
# chunk; 7B at TP=4: QKV, gate/up (2 x 4736) and down at B=1 x 1024 and
# B=8 x 1024 prompt rows.
PREFILL_GEMM_SHAPES = [
    ("05b_gateup_m128", "swiglu", 128, 9728, 896),
    ("05b_gateup_m2048", "swiglu", 2048, 9728, 896),
    ("05b_down_m2048", "store", 2048, 896, 4864),
    ("05b_qkv_m2048", "store", 2048, 1152, 896),
    ("7b_tp4_qkv_m1024", "store", 1024, 1152, 3584),
    ("7b_tp4_gateup_m1024", "swiglu", 1024, 9472, 3584),
    ("7b_tp4_down_m1024", "store", 1024, 3584, 4736),
    ("7b_tp4_gateup_m8192", "swiglu", 8192, 9472, 3584),
    ("7b_tp4_down_m8192", "store", 8192, 3584, 4736),
]


def run_prefill_gemm(args):
    """Tensor-core prefill GEMM sweep on one GPU: one JSON line per shape."""
    from minitp_b200.build import build

    build()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    want = set(args.gemm_shapes.split(",")) if args.gemm_shapes else None
    for name, epi, M, N, K in PREFILL_GEMM_SHAPES:
        if want and name not in want:
            continue
        r = time_prefill_gemm(epi, M, N, K, dev)
        r = {"workload": "prefill_gemm", "shape": name, **r}
        print(json.dumps(r), flush=True)


def main(argv=None):
    args = parse_args(argv)
    if args.workload == "fused_ar":
        run_fused_ar(args)
        return
    if args.workload == "prefill_gemm":
        run_prefill_gemm(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
