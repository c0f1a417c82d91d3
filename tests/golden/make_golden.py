"""Record parity fixtures by running the reference implementation (mini-TP).

Run in a container where the reference source tree is readable:

    python tests/golden/make_golden.py --reference /path/to/mini-tp [--only NAME ...]

The reference package ``minitp`` is imported unmodified from that tree and
driven through its public API, on CPU: in-process for TP=1, and as Gloo ranks
(``tests/tp_harness.run_tp``) for TP>1. Inputs come from the seeded protocols
in ``minitp_b200.synthetic`` and ``minitp_b200.synthetic_cases``, so the
fixtures store outputs (plus input checksums), not the inputs themselves.

Fixtures written to ``tests/golden/``:

* ``model_<cfg>_tp<N>_<dtype>.npz``: greedy decode through
  ``GenerationState`` (minitp/generation.py:70-130), the same loop as
  ``generate_greedy`` with ``early_stop=False`` (generation.py:133-171).
  Stores the token ids, the full (rank-gathered) logits of the prefill's last
  position and of the first and last decode steps, and per-step top-2 values
  and ids.
* ``argmax_tp<N>.npz``: ``VocabParallelLMHead.distributed_argmax`` with the
  bitpack encoding (minitp/parallel/embedding.py:118-172) on the seeded
  tie-injected logits, plus the reference test suite's constructed
  21M-vocab cases (tests/test_vocab_layers.py:350-383).
* ``embedding_tp<N>.npz``: ``VocabParallelEmbedding.forward``
  (embedding.py:44-50).
* ``fused_ar_tp<N>.npz``: the RowParallel reduce (collectives.py:147-157), then
  the decoder residual add (layer.py:64) and ``RMSNorm`` (layer.py:36-42).
* ``rope.npz``: ``RotaryEmbedding.apply`` (rope.py:47-64).
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
import tempfile
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from minitp_b200 import config as mcfg  # noqa: E402
from minitp_b200.synthetic import make_prompt, save_checkpoint  # noqa: E402
from minitp_b200.synthetic_cases import argmax_logits, embedding_case, fused_ar_case  # noqa: E402
from tests.tp_harness import run_tp  # noqa: E402

DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16}


def _ref_import(ref_root: str):
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)


def _ref_ctx(rank: int, tp: int):
    import torch.distributed as dist
    from minitp.distributed.context import ParallelContext

    pg = dist.group.WORLD if tp > 1 else None
    return ParallelContext(rank, rank, tp, rank, tp, torch.device("cpu"), pg)


def _gather_last(local: torch.Tensor, tp: int) -> torch.Tensor:
    """Concatenate every rank's ``[B, V/tp]`` logits (even vocab split)."""
    if tp == 1:
        return local.float().clone()
    import torch.distributed as dist

    parts = [torch.empty_like(local) for _ in range(tp)]
    dist.all_gather(parts, local.contiguous())
    return torch.cat(parts, dim=-1).float()


def checksum(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()[:16]


# ---------------------------------------------------------------------- #
# model decode
# ---------------------------------------------------------------------- #
def _w_model(rank, tp, ref_root, cfg_kw, ckpt_dir, dtype_name, batch, prompt_len, n_new, seed):
    _ref_import(ref_root)
    from minitp.config import ModelConfig as RC
    from minitp.generation import GenerationState, generate_greedy
    from minitp.weight_loader import load_qwen2_tp

    rc = RC(**cfg_kw)
    rc.validate(tp)
    ctx = _ref_ctx(rank, tp)
    model = load_qwen2_tp(ckpt_dir, rc, ctx, dtype=DTYPES[dtype_name], loader="selective").eval()
    ids = make_prompt(rc.vocab_size, batch, prompt_len, seed)
    out = {}
    with torch.inference_mode():
        state = GenerationState(model, ids, n_new)
        logits = state.prefill()
        out["prefill_last_logits"] = _gather_last(logits[:, -1], tp).numpy()
        top_v, top_i, step_logits = [], [], {}
        for step in range(n_new):
            full = _gather_last(logits[:, -1], tp)
            tv, ti = full.topk(2, dim=-1)
            top_v.append(tv.numpy())
            top_i.append(ti.numpy())
            if step in (1, n_new - 1):
                step_logits[step] = full.numpy()
            tok = state.select_next(logits)
            pos = state.append(tok)
            if step + 1 < n_new:
                logits = state.decode_step(tok, pos)
        tokens = state.out_ids.clone()
        # the shipped entry point must give the same sequence
        again = generate_greedy(model, ids, n_new, early_stop=False)
        assert torch.equal(again, tokens), "generate_greedy diverged from GenerationState loop"
    out["tokens"] = tokens.numpy()
    out["top2_values"] = np.stack(top_v)  # [n_new, B, 2]: logits that chose token `step`
    out["top2_ids"] = np.stack(top_i)
    out["decode1_logits"] = step_logits[1]
    out["decode_last_logits"] = step_logits[n_new - 1]
    out["prompt"] = ids.numpy()
    return out


MODEL_RUNS = {
    # name: (cfg factory, batch, prompt_len, n_new, [(tp, dtype)])
    "tiny": (mcfg.baseline_tiny, 1, 8, 16, [(1, "fp32"), (2, "fp32"), (1, "bf16"), (2, "bf16")]),
    "q05b": (mcfg.qwen25_05b, 1, 128, 128, [(1, "fp32"), (2, "fp32"), (1, "bf16"), (2, "bf16")]),
    "q05b_b4": (mcfg.qwen25_05b, 4, 32, 16, [(1, "fp32"), (2, "fp32")]),
    "q7b_l2": (lambda: mcfg.qwen25_7b(num_layers=2), 1, 16, 8,
               [(1, "fp32"), (4, "fp32"), (1, "bf16")]),
}


def make_model_goldens(ref_root: str, names: list[str]) -> None:
    for name in names:
        factory, batch, plen, n_new, runs = MODEL_RUNS[name]
        cfg = factory()
        cfg_kw = {k: getattr(cfg, k) for k in (
            "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
            "num_key_value_heads", "head_dim", "vocab_size", "rms_norm_eps", "rope_theta",
            "max_position_embeddings", "tie_word_embeddings")}
        with tempfile.TemporaryDirectory(prefix="mtpb_ck_") as ckpt:
            t0 = time.time()
            save_checkpoint(cfg, ckpt, seed=0)
            print(f"[{name}] checkpoint written in {time.time() - t0:.1f}s", flush=True)
            for tp, dt in runs:
                t0 = time.time()
                args = (ref_root, cfg_kw, ckpt, dt, batch, plen, n_new, 0)
                if tp == 1:
                    torch.set_num_threads(os.cpu_count() or 1)
                    res = _w_model(0, 1, *args)
                else:
                    res = run_tp(tp, _w_model, *args)[0]
                res["config"] = np.array(repr(cfg_kw))
                # keep fixtures small: full-vocab logits only for TP=1 runs (TP>1
                # runs keep tokens, top-2 and float64 checksums), and only the
                # prefill logits when batch > 1
                for k in ("prefill_last_logits", "decode1_logits", "decode_last_logits"):
                    res[k.replace("_logits", "_sum")] = np.array(np.asarray(res[k], np.float64).sum())
                    if tp > 1 or (batch > 1 and k != "prefill_last_logits"):
                        del res[k]
                path = os.path.join(HERE, f"model_{name}_tp{tp}_{dt}.npz")
                np.savez_compressed(path, **res)
                print(f"[{name}] tp={tp} {dt}: {time.time() - t0:.1f}s tokens "
                      f"{res['tokens'][0, plen:plen + 8].tolist()} -> {path}", flush=True)


# ---------------------------------------------------------------------- #
# distributed argmax
# ---------------------------------------------------------------------- #
ARGMAX_CASES = [(v, b) for v in (151936, 151937) for b in (1, 8, 64)]


def _w_argmax(rank, tp, ref_root):
    _ref_import(ref_root)
    from minitp.parallel.embedding import VocabParallelLMHead
    from minitp.parallel.linear import shard_range

    ctx = _ref_ctx(rank, tp)
    out = {}
    for vocab, batch in ARGMAX_CASES:
        logits = argmax_logits(vocab, batch, seed=vocab + batch)
        head = VocabParallelLMHead(4, vocab, ctx, init_weights=False)
        s, e = shard_range(vocab, rank, tp)
        got = head.distributed_argmax(logits[:, s:e].contiguous(), encoding="bitpack")
        out[f"ids_v{vocab}_b{batch}"] = got.squeeze(-1).numpy()
        out[f"sum_v{vocab}_b{batch}"] = np.array(float(logits.double().sum()))
    # constructed cases of the reference suite (tests/test_vocab_layers.py:350-383)
    vocab = 21_000_000
    head = VocabParallelLMHead(4, vocab, ctx, init_weights=False)
    s, e = shard_range(vocab, rank, tp)
    got = []
    for case in big_vocab_cases():
        got.append(int(head.distributed_argmax(case[..., s:e].contiguous(), encoding="bitpack")))
    out["ids_big"] = np.array(got)
    return out


def big_vocab_cases() -> list[torch.Tensor]:
    vocab = 21_000_000
    base = torch.full((1, vocab), -1e30)
    cases = []
    for vid in (12095, 16_777_216, 16_777_217, 20_000_001, 20_979_201):
        c = base.clone()
        c[0, vid] = 3.5
        cases.append(c)
    tie = base.clone()
    tie[0, 5] = 7.0
    tie[0, vocab - 5] = 7.0
    cases.append(tie)
    neg = torch.full((1, vocab), -50.0)
    neg[0, vocab - 2] = -0.25
    cases.append(neg)
    nan_case = base.clone()
    nan_case[0, 6] = 9.0
    nan_case[0, 100] = float("nan")
    cases.append(nan_case)
    return cases


def make_argmax_goldens(ref_root: str) -> None:
    for tp in (2, 4, 8):
        t0 = time.time()
        res = run_tp(tp, _w_argmax, ref_root)
        for r in range(1, tp):
            for k, v in res[r].items():
                assert np.array_equal(v, res[0][k]), (tp, r, k)
        np.savez_compressed(os.path.join(HERE, f"argmax_tp{tp}.npz"), **res[0])
        print(f"[argmax] tp={tp}: {time.time() - t0:.1f}s big={res[0]['ids_big'].tolist()}", flush=True)


# ---------------------------------------------------------------------- #
# vocab-parallel embedding
# ---------------------------------------------------------------------- #
EMBED_CASES = [(v, b) for v in (151936, 151937) for b in (1, 8, 64)]


def _w_embed(rank, tp, ref_root):
    _ref_import(ref_root)
    from minitp.parallel.embedding import VocabParallelEmbedding
    from minitp.parallel.linear import shard_range

    ctx = _ref_ctx(rank, tp)
    out = {}
    for vocab, batch in EMBED_CASES:
        table, ids = embedding_case(vocab, 896, batch, seed=vocab * 7 + batch)
        emb = VocabParallelEmbedding(vocab, 896, ctx, init_weights=False).to(torch.bfloat16)
        s, e = shard_range(vocab, rank, tp)
        with torch.no_grad():
            emb.weight.copy_(table[s:e])
            y = emb(ids)
        out[f"out_v{vocab}_b{batch}"] = y.view(torch.int16).numpy()
        out[f"ids_v{vocab}_b{batch}"] = ids.numpy()
    return out


def make_embedding_goldens(ref_root: str) -> None:
    for tp in (2, 4, 8):
        t0 = time.time()
        res = run_tp(tp, _w_embed, ref_root)
        np.savez_compressed(os.path.join(HERE, f"embedding_tp{tp}.npz"), **res[0])
        print(f"[embedding] tp={tp}: {time.time() - t0:.1f}s", flush=True)


# ---------------------------------------------------------------------- #
# RowParallel reduce + residual + RMSNorm
# ---------------------------------------------------------------------- #
FUSED_AR_ROWS = (1, 8, 64, 128, 512, 2048)


def _w_fused_ar(rank, tp, ref_root):
    _ref_import(ref_root)
    from minitp.distributed import all_reduce
    from minitp.layer import RMSNorm

    out = {}
    for rows in FUSED_AR_ROWS:
        partials, residual, gain = fused_ar_case(rows, 896, tp, seed=1000 + rows)
        t = partials[rank].clone()
        reduced = all_reduce(t)  # in-place SUM over ranks (collectives.py:147-157)
        x = residual + reduced  # decoder residual add (layer.py:64)
        norm = RMSNorm(896, 1e-6, init_weights=False).to(torch.bfloat16)
        with torch.no_grad():
            norm.weight.copy_(gain)
            y = norm(x)
        if rows <= 64:
            out[f"residual_r{rows}"] = x.view(torch.int16).numpy()
            out[f"normed_r{rows}"] = y.view(torch.int16).numpy()
        else:  # large cases: a row sample plus float64 sums keep the fixture small
            sample = sorted({0, 1, rows // 2, rows - 1})
            out[f"sample_rows_r{rows}"] = np.array(sample)
            out[f"residual_r{rows}"] = x[sample].view(torch.int16).numpy()
            out[f"normed_r{rows}"] = y[sample].view(torch.int16).numpy()
            out[f"residual_sum_r{rows}"] = np.array(float(x.double().sum()))
            out[f"normed_sum_r{rows}"] = np.array(float(y.double().sum()))
    return out


def make_fused_ar_goldens(ref_root: str) -> None:
    for tp in (2, 4, 8):
        t0 = time.time()
        res = run_tp(tp, _w_fused_ar, ref_root)
        for r in range(1, tp):
            for k, v in res[r].items():
                assert np.array_equal(v, res[0][k]), (tp, r, k)
        np.savez_compressed(os.path.join(HERE, f"fused_ar_tp{tp}.npz"), **res[0])
        print(f"[fused_ar] tp={tp}: {time.time() - t0:.1f}s", flush=True)


# ---------------------------------------------------------------------- #
# RoPE
# ---------------------------------------------------------------------- #
def make_rope_goldens(ref_root: str) -> None:
    _ref_import(ref_root)
    from minitp.rope import RotaryEmbedding

    out = {}
    for hd in (16, 64, 128):
        rot = RotaryEmbedding(hd, 1e6, 4096)
        g = torch.Generator()
        g.manual_seed(hd)
        q = torch.randn(2, 4, 5, hd, generator=g)
        k = torch.randn(2, 1, 5, hd, generator=g)
        pos = torch.tensor([0, 1, 95, 1000, 4095])
        for dt in ("fp32", "bf16"):
            qq, kk = q.to(DTYPES[dt]), k.to(DTYPES[dt])
            qr, kr = rot.apply(qq, kk, pos)
            out[f"q_hd{hd}_{dt}"] = qr.float().numpy()
            out[f"k_hd{hd}_{dt}"] = kr.float().numpy()
        out[f"cos_hd{hd}"] = rot.cos_cache[pos].numpy()
        out[f"sin_hd{hd}"] = rot.sin_cache[pos].numpy()
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **out)
    print("[rope] done", flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MINITP_REFERENCE"),
                    help="source tree of the reference (default: $MINITP_REFERENCE)")
    ap.add_argument("--only", nargs="*", default=None,
                    help="subset of: rope argmax embedding fused_ar " + " ".join(MODEL_RUNS))
    a = ap.parse_args()
    if not a.reference:
        raise SystemExit("give the reference source tree with --reference or $MINITP_REFERENCE")
    ref = os.path.abspath(a.reference)
    if not os.path.isdir(os.path.join(ref, "minitp")):
        raise SystemExit(f"reference package not found under {ref}")
    want = a.only or ["rope", "argmax", "embedding", "fused_ar", *MODEL_RUNS]
    if "rope" in want:
        make_rope_goldens(ref)
    if "argmax" in want:
        make_argmax_goldens(ref)
    if "embedding" in want:
        make_embedding_goldens(ref)
    if "fused_ar" in want:
        make_fused_ar_goldens(ref)
    models = [m for m in want if m in MODEL_RUNS]
    if models:
        make_model_goldens(ref, models)


if __name__ == "__main__":
    main()
