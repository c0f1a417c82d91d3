"""Decode throughput of the B200 TP path: ``python bench.py --gpus N --steps K --warmup W``.

One step = one fixed-length greedy generation over a batch of synthetic
prompts (Qwen2.5-0.5B shape by default: B=1, prompt 128, 128 new tokens,
bf16, seeded random weights) at TP = N (one process per GPU under torchrun).
The prefill runs eagerly; the 127 decode steps are replays of one CUDA graph
of the device-resident decode step.

Reported (rank 0, one JSON line):
* value: decode tokens/s = B * decode steps / decode time, where the decode
  time is measured with CUDA events per step and the max over ranks is taken.
* e2e: the same metric through ``generate_greedy``, starting from pinned host
  prompt ids and ending with the output ids copied back to the host.
* roofline: the dominant kernel (the LM-head GEMV streams the largest weight
  of the token), timed live with CUDA events over repeated launches;
  achieved = its weight bytes / launch time. roofline_token: (weight + KV)
  bytes read per token per rank / measured time per token.
* cpu_baseline: the CPU oracle port of the reference (rank 0, N=1 only) on
  a bounded sample (prefill + 8 decode tokens).
``--impl reference`` times that CPU port as the reference arm.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

MEASURED_PEAKS = os.path.join(REPO, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--model", default="qwen2.5-0.5b", choices=["qwen2.5-0.5b", "qwen2.5-7b", "tiny"])
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--prompt", type=int, default=None)
    p.add_argument("--new-tokens", type=int, default=None)
    p.add_argument("--dtype", default="bf16", choices=["bf16", "fp32"])
    p.add_argument("--gen-device", default=None, help="where synthetic weights are drawn (cpu|cuda)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-pdl", action="store_true")
    p.add_argument("--out", default=None, help="also write the JSON line here")
    p.add_argument("--workload", default="decode", choices=["decode", "fused_ar", "prefill_gemm"],
                   help="decode (default), the fused AllReduce+residual+RMSNorm microbenchmark, or the "
                        "tensor-core prefill GEMM sweep")
    p.add_argument("--gemm-shapes", default=None,
                   help="prefill_gemm: comma-separated names of the shapes to run (default: all)")
    p.add_argument("--iters", type=int, default=10000, help="fused_ar: iterations per size")
    return p.parse_args(argv)


def workload(args):
    from minitp_b200 import config as mcfg

    if args.model == "qwen2.5-7b":
        cfg, prompt, new = mcfg.qwen25_7b(), 1024, 256
    elif args.model == "tiny":
        cfg, prompt, new = mcfg.baseline_tiny(), 8, 16
    else:
        cfg, prompt, new = mcfg.qwen25_05b(), 128, 128
    return cfg, args.prompt or prompt, args.new_tokens or new


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
# bytes per token
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


# DRAM bytes (read + write) of one decode_mk_kernel launch from an ncu capture
# (profiles/decode_mk_kernel_qwen05b_tp1_b1.md), keyed by (model, batch, TP).
MK_TRAFFIC = {("qwen2.5-0.5b", 1, 1): 994_280_704}


def measured_traffic(args, world: int, step_launches: int):
    if step_launches != 1:
        return None
    return MK_TRAFFIC.get((args.model, args.batch, world))


def launches_per_generation(n_layers: int, new_tokens: int, prefill_tokens: int, step_launches: int) -> int:
    """minitp_b200 kernel launches of one fixed-length generation.

    Prefill runs the kernel chain; every decode step makes `step_launches`
    launches (1 when the decode megakernel runs it, as the library reports).
    """
    prefill = 1 + n_layers * 5 + (2 * n_layers + 1 if prefill_tokens > 1 else 0) + 1
    select = 2  # argmax rows + finish
    seed = 1  # decode position store
    return prefill + select + seed + (new_tokens - 1) * step_launches


# ---------------------------------------------------------------------- #
# CPU baseline (oracle port of the reference)
# ---------------------------------------------------------------------- #
_ORACLE_MODELS: dict = {}


def cpu_oracle_decode(cfg, batch, prompt_len, sample_tokens, dtype, tp, threads, passes=1):
    """Decode tok/s of the oracle port on the host cores.

    Each pass: fresh KV caches, prefill of the prompt (untimed), then
    ``sample_tokens`` timed greedy decode steps. The model (synthetic weights)
    is built once per shape and kept for later calls.
    """
    from oracle.model import OracleConfig, OracleModel, checkpoint_tensors, prompt

    torch.set_num_threads(threads)
    key = (repr(cfg), str(dtype), tp)
    model = _ORACLE_MODELS.get(key)
    if model is None:
        model = OracleModel(OracleConfig.of(cfg), checkpoint_tensors(cfg), tp=tp, dtype=dtype)
        _ORACLE_MODELS.clear()
        _ORACLE_MODELS[key] = model
    ids = prompt(cfg.vocab_size, batch, prompt_len)
    dt = 0.0
    for _ in range(passes):
        model.reset(batch, prompt_len + sample_tokens + 1)
        logits = model.forward(ids, torch.arange(prompt_len))
        tok = model.select(logits[:, -1])
        t0 = time.perf_counter()
        for i in range(sample_tokens):
            logits = model.forward(tok[:, None], torch.tensor([prompt_len + i]))
            tok = model.select(logits[:, -1])
        dt += time.perf_counter() - t0
    return batch * sample_tokens * passes / dt, dt


def run_reference(args, cfg, prompt_len, new_tokens):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    sample = max(1, new_tokens - 1)  # every decode step of one generation
    vals = []
    for _ in range(max(args.warmup, 0)):
        cpu_oracle_decode(cfg, args.batch, prompt_len, 2, dtype, args.gpus, threads)
    for _ in range(args.steps):
        v, _ = cpu_oracle_decode(cfg, args.batch, prompt_len, sample, dtype, args.gpus, threads)
        vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": "decode tok/s", "value": round(value, 3), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * args.batch / value, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": args.dtype, "data": "synthetic (seeded random weights and prompts)",
        "config": {"workload": f"{args.model} B={args.batch} P={prompt_len} new={new_tokens} tp={args.gpus}",
                   "model": args.model, "global_batch": args.batch, "seq_len": prompt_len + new_tokens,
                   "parallelism": f"tp{args.gpus} (emulated in one process)"},
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"per step: prefill {prompt_len} (untimed) + {sample} decode steps, oracle port "
                                   f"of the reference CPU path, tp={args.gpus} emulated"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------- #
# B200 arm
# ---------------------------------------------------------------------- #
def run_b200(args, cfg, prompt_len, new_tokens):
    import torch.distributed as dist

    from minitp_b200 import _lib, ops
    from minitp_b200.build import build
    from minitp_b200.distributed.context import init_context
    from minitp_b200.generation import GenerationState, generate_greedy
    from minitp_b200.synthetic import make_prompt
    from minitp_b200.weight_loader import load_synthetic_tp

    if int(os.environ.get("RANK", "0")) == 0:
        build()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        # rank 0 built the library; the others wait for it through the store
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    ctx = init_context(timeout_s=120.0)
    if world > 1:
        dist.barrier()
    lib = _lib.load()
    if args.no_pdl:
        lib.mtpb_set_pdl(0)
    dev = ctx.device
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    gen_dev = args.gen_device or ("cuda" if args.model == "qwen2.5-7b" else "cpu")
    model = load_synthetic_tp(cfg, ctx, dtype=dtype, device=dev, seed=0, gen_device=gen_dev)
    ids_host = make_prompt(cfg.vocab_size, args.batch, prompt_len).pin_memory()
    ids = ids_host.to(dev)
    comm = ctx.comm()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def one_step(timed: bool):
        st = GenerationState(model, ids, new_tokens)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        logits = st.prefill(last_only=True)
        tok = st.select_next(logits)
        st.append(tok)
        st.start_device_decode(tok)
        st.device_step()
        st.capture()
        ev[1].record()
        for _ in range(new_tokens - 2):
            st.graph_step()
        ev[2].record()
        return st, ev

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        one_step(False)
        flush.zero_()
    barrier()
    comm.raise_on_error()

    sampler = ClockSampler(dev.index if dev.index is not None else 0)
    sampler.start()
    decode_ms, step_ms = [], []
    barrier()
    for _ in range(args.steps):
        flush.zero_()  # L2 flush between timed steps (256 MiB > 126 MB L2)
        st, ev = one_step(True)
        torch.cuda.synchronize()
        decode_ms.append(ev[1].elapsed_time(ev[2]) / max(1, new_tokens - 2))
        step_ms.append(ev[0].elapsed_time(ev[2]))
        st.release()
    barrier()
    clocks = sampler.stop()
    comm.raise_on_error()

    # max over ranks
    t = torch.tensor([statistics.mean(decode_ms), statistics.mean(step_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_token, ms_per_step = t.tolist()
    value = args.batch / (ms_per_token / 1e3)

    # e2e through the public API: pinned host ids in, host ids out
    e2e_ms = []
    e2e_warm = 2
    for i in range(e2e_warm + max(2, min(args.steps, 5))):
        flush.zero_()
        barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = generate_greedy(model, ids_host.to(dev, non_blocking=True), new_tokens, early_stop=False)
        host = out.to("cpu", non_blocking=False)
        e.record()
        torch.cuda.synchronize()
        if i >= e2e_warm:  # the first calls are untimed warm-up, as for the device-timed steps
            e2e_ms.append(s.elapsed_time(e))
    te = torch.tensor([statistics.mean(e2e_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = args.batch * new_tokens / (te.item() / 1e3)

    # decode launches per step as the library plans them (1 = megakernel)
    nk = ctypes.c_int(0)
    _lib.call("mtpb_model_decode_kernels", model.native(), args.batch, prompt_len + new_tokens, ctypes.byref(nk))
    step_launches = nk.value

    # the prefill GEMV, timed live: the LM-head weights over this rank's vocab shard
    x = torch.randn(args.batch, cfg.hidden_size, device=dev).to(dtype)
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
    k_bytes = w.numel() * w.element_size() + x.numel() * x.element_size() + args.batch * w.shape[0] * w.element_size()
    k_gbs = k_bytes / (k_ms / 1e3) / 1e9

    # the prefill GEMM (tensor cores) at this workload's prefill rows, gate/up shape
    gu = model.model.layers[0].mlp.gate_up_proj.weight
    tc_line = None
    if dtype == torch.bfloat16 and args.batch * prompt_len >= 64:
        tc_line = time_prefill_gemm("swiglu", args.batch * prompt_len, gu.shape[0], gu.shape[1], dev)

    wb = weight_bytes_per_token(model)
    kvb = kv_bytes_per_token(model, args.batch, prompt_len + new_tokens / 2)
    tok_gbs = (wb + kvb) / (ms_per_token / 1e3) / 1e9

    line = None
    if ctx.is_rank_zero:
        line = {
            "metric": "decode tok/s", "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "us_per_token": round(ms_per_token * 1e3, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": args.dtype,
            "data": "synthetic (seeded random weights N(0,0.02) and uniform prompt ids)",
            "config": {
                "workload": f"{args.model} decode, B={args.batch}, prompt {prompt_len}, {new_tokens} new tokens, "
                            f"TP={world}",
                "model": args.model, "global_batch": args.batch, "seq_len": prompt_len + new_tokens,
                "parallelism": f"tp{world}", "heads_padded": bool(model.cfg.is_padded),
                "l2": "flushed between timed steps (256 MiB write)",
                "decode": "CUDA graph replay of the device-resident decode step (persistent megakernel)",
            },
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": ids_host.numel() * ids_host.element_size(),
                    "d2h_bytes_per_step": args.batch * (prompt_len + new_tokens) * 8,
                    "definition": "generate_greedy from pinned host ids to host output ids, incl. prefill",
                    "warmup": e2e_warm, "samples_ms": [round(x, 3) for x in e2e_ms]},
            "roofline": {"bound": "hbm",
                         "kernel": "decode_mk_kernel" if step_launches == 1 else "decode kernel chain",
                         "achieved": round(tok_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(tok_gbs / peak, 4), "traffic": measured_traffic(args, world, step_launches),
                         "peak_kind": peak_kind,
                         "bytes_per_launch": round(wb + kvb), "weight_bytes": wb, "kv_bytes": round(kvb),
                         "us_per_launch": round(ms_per_token * 1e3, 3),
                         "timing": "CUDA events over the graph replays of the decode step (one launch each)"},
            "roofline_gemv": {"bound": "hbm", "kernel": "gemv_kernel (LM-head weights, prefill GEMV)",
                              "achieved": round(k_gbs, 1), "peak": peak, "unit": "GB/s",
                              "frac": round(k_gbs / peak, 4), "bytes_per_launch": k_bytes,
                              "us_per_launch": round(k_ms * 1e3, 3)},
            "roofline_prefill_gemm": tc_line,
            "gpu_launches": launches_per_generation(cfg.num_hidden_layers, new_tokens, prompt_len,
                                                    step_launches) * args.steps,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            ns = max(1, new_tokens - 1)
            v, dt = cpu_oracle_decode(cfg, args.batch, prompt_len, ns, dtype, 1, threads, passes=3)
            line["cpu_baseline"] = {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                                    "sample": f"3 x (prefill {prompt_len} untimed + {ns} decode steps), "
                                              f"{dt:.1f} s timed, oracle port of the reference CPU path"}
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


def run_fused_ar(args):
    """Fused AllReduce + residual + RMSNorm vs NCCL all_reduce, [rows, 896] bf16.

    Both are replayed from CUDA graphs of `chunk` back-to-back calls, so the
    numbers are device time per call (max over ranks), not host launch time.
    Prints one JSON line per size on rank 0.
    """
    import torch.distributed as dist

    from minitp_b200 import ops
    from minitp_b200.build import build
    from minitp_b200.distributed.context import init_context
    from minitp_b200.synthetic_cases import fused_ar_case

    if int(os.environ.get("RANK", "0")) == 0:
        build()
    ctx = init_context(timeout_s=120.0)
    world = ctx.tp_size
    if world < 2:
        if ctx.is_rank_zero:
            print(json.dumps({"workload": "fused_ar", "skipped": "needs >= 2 GPUs"}))
        return
    dist.barrier()
    comm = ctx.comm()
    dev = ctx.device
    results = []
    chunk = 100
    for rows in (1, 8, 64, 128, 512, 2048):
        partials, residual, gain = fused_ar_case(rows, 896, world, seed=1000 + rows)
        p = partials[ctx.tp_rank].to(dev)
        r = residual.to(dev)
        g = gain.to(dev)
        out_res = torch.empty_like(p)
        out_norm = torch.empty_like(p)
        nccl_t = p.clone()
        from minitp_b200 import _lib

        def fused():
            _lib.call("mtpb_allreduce_residual_rmsnorm", comm.handle, p.data_ptr(), r.data_ptr(), g.data_ptr(),
                      None, out_res.data_ptr(), out_norm.data_ptr(), rows, 896, 1e-6, _lib.MTPB_BF16,
                      _lib.stream_ptr(dev))

        def nccl():
            dist.all_reduce(nccl_t)

        times = {}
        for name, fn in (("fused", fused), ("nccl", nccl)):
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
            reps = max(1, args.iters // chunk)
            s, e = torch.cuda.Event(True), torch.cuda.Event(True)
            s.record()
            for _ in range(reps):
                graph.replay()
            e.record()
            torch.cuda.synchronize()
            us = s.elapsed_time(e) * 1e3 / (reps * chunk)
            t = torch.tensor([us], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times[name] = t.item()
            del graph
        comm.raise_on_error()
        m = rows * 896 * 2
        line = {"workload": "fused_ar", "metric": "fused AR+residual+RMSNorm latency", "rows": rows,
                "bytes": m, "tp": world, "unit": "us", "fused_us": round(times["fused"], 3),
                "nccl_allreduce_us": round(times["nccl"], 3),
                "ratio_fused_over_nccl": round(times["fused"] / times["nccl"], 3),
                "fused_nvlink_send_gbs": round((world - 1) * m / (times["fused"] * 1e-6) / 1e9, 2),
                "iters": (max(1, args.iters // chunk)) * chunk}
        results.append(line)
        if ctx.is_rank_zero:
            print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
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
    cfg, prompt_len, new_tokens = workload(args)
    if args.impl == "reference":
        run_reference(args, cfg, prompt_len, new_tokens)
    else:
        run_b200(args, cfg, prompt_len, new_tokens)


if __name__ == "__main__":
    main()
