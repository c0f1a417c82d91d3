"""Pin the CPU oracle to outputs recorded from the reference (tests/golden, make_golden.py).

The oracle is the checker of every GPU parity test, so it must reproduce the
reference first: ids and lookups bit-exactly, floats within the reference's
own tolerances.
"""

import numpy as np
import pytest
import torch

from tests.conftest import golden
from minitp_b200 import config as mcfg
from minitp_b200.synthetic_cases import argmax_logits, embedding_case, fused_ar_case
from oracle import model as om
from oracle.argmax import distributed_argmax, shard_range


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_argmax_oracle_matches_reference(tp):
    g = golden(f"argmax_tp{tp}.npz")
    for vocab in (151936, 151937):
        for batch in (1, 8, 64):
            x = argmax_logits(vocab, batch, seed=vocab + batch)
            # same inputs (float64 sum; the summation order depends on the thread count)
            assert abs(float(x.double().sum()) - float(g[f"sum_v{vocab}_b{batch}"])) < 1e-8
            got = distributed_argmax(x.numpy(), tp)
            assert np.array_equal(got, g[f"ids_v{vocab}_b{batch}"]), (vocab, batch)
            # every tie row resolved to the lower id, and the bitpack == torch.argmax w/o NaN
            assert np.array_equal(got, x.argmax(-1).numpy())


def test_argmax_oracle_big_vocab_cases():
    """The reference suite's constructed 21M-vocab cases (ids > 2^24, ties, negatives, NaN)."""
    from tests.golden.make_golden import big_vocab_cases

    g = golden("argmax_tp2.npz")
    got = [int(distributed_argmax(c.numpy(), 2)[0]) for c in big_vocab_cases()]
    assert got == g["ids_big"].tolist() == [12095, 16777216, 16777217, 20000001, 20979201, 5, 20999998, 6]


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_embedding_oracle_matches_reference(tp):
    g = golden(f"embedding_tp{tp}.npz")
    for vocab in (151936, 151937):
        for batch in (1, 8, 64):
            table, ids = embedding_case(vocab, 896, batch, seed=vocab * 7 + batch)
            assert np.array_equal(ids.numpy(), g[f"ids_v{vocab}_b{batch}"])
            shards = [table[slice(*shard_range(vocab, r, tp))] for r in range(tp)]
            got = om.embedding(ids, shards, vocab)
            assert np.array_equal(got.view(torch.int16).numpy(), g[f"out_v{vocab}_b{batch}"])


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_fused_ar_oracle_matches_reference(tp):
    g = golden(f"fused_ar_tp{tp}.npz")
    for rows in (1, 8, 64, 128, 512, 2048):
        partials, residual, gain = fused_ar_case(rows, 896, tp, seed=1000 + rows)
        x, y = om.allreduce_residual_rmsnorm(list(partials), residual, gain, 1e-6)
        if f"sample_rows_r{rows}" in g:
            sel = g[f"sample_rows_r{rows}"]
            x, y = x[sel], y[sel]
        want_x = torch.from_numpy(g[f"residual_r{rows}"]).view(torch.bfloat16)
        want_y = torch.from_numpy(g[f"normed_r{rows}"]).view(torch.bfloat16)
        if tp == 2:
            assert torch.equal(x, want_x)  # two-rank bf16 sum: one rounding, bit-exact
        else:
            # for tp > 2 Gloo rounds each of its tp-1 running sums to bf16 (the
            # oracle rounds once), then the residual add rounds again; every
            # value here is below 8 in magnitude, so each rounding is off by
            # at most half an ulp of 2^-5: bound tp * 2^-6
            atol = tp * 2 ** -6
            torch.testing.assert_close(x.float(), want_x.float(), atol=atol, rtol=0)
        atol = 2 ** -5 if tp == 2 else tp * 2 ** -6
        torch.testing.assert_close(y.float(), want_y.float(), atol=atol, rtol=2 ** -6)


def test_rope_oracle_matches_reference():
    g = golden("rope.npz")
    for hd in (16, 64, 128):
        cos, sin = om.rope_tables(hd, 1e6, 4096)
        pos = torch.tensor([0, 1, 95, 1000, 4095])
        assert np.array_equal(cos[pos].numpy(), g[f"cos_hd{hd}"])
        assert np.array_equal(sin[pos].numpy(), g[f"sin_hd{hd}"])
        gen = torch.Generator().manual_seed(hd)
        q = torch.randn(2, 4, 5, hd, generator=gen)
        k = torch.randn(2, 1, 5, hd, generator=gen)
        for dt, tdt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
            qr = om.apply_rope(q.to(tdt), cos[pos], sin[pos])
            kr = om.apply_rope(k.to(tdt), cos[pos], sin[pos])
            assert np.array_equal(qr.float().numpy(), g[f"q_hd{hd}_{dt}"])
            assert np.array_equal(kr.float().numpy(), g[f"k_hd{hd}_{dt}"])


def _oracle_generate(cfg, batch, plen, n, tp, dtype):
    torch.set_num_threads(max(1, torch.get_num_threads()))
    m = om.OracleModel(om.OracleConfig.of(cfg), om.checkpoint_tensors(cfg), tp=tp, dtype=dtype)
    ids = om.prompt(cfg.vocab_size, batch, plen)
    return ids, *m.generate(ids, n, keep_logits=True)


@pytest.mark.parametrize("tp,dt", [(1, "fp32"), (2, "fp32"), (1, "bf16"), (2, "bf16")])
def test_tiny_model_oracle_matches_reference(tp, dt):
    g = golden(f"model_tiny_tp{tp}_{dt}.npz")
    ids, out, kept = _oracle_generate(mcfg.baseline_tiny(), 1, 8, 16, tp, torch.float32 if dt == "fp32"
                                      else torch.bfloat16)
    assert np.array_equal(ids.numpy(), g["prompt"])
    assert np.array_equal(out.numpy(), g["tokens"])
    if "prefill_last_logits" in g:
        tol = 1e-4 if dt == "fp32" else 0.5
        ref = g["prefill_last_logits"]
        err = np.abs(kept[0].numpy() - ref).max()
        assert (err / np.abs(ref).max() if dt == "fp32" else err) < tol
    # checksum of all logits (the only logits record of TP>1 fixtures): fp32 within
    # 1e-2 in total; bf16 within 1e-3 per logit on average
    total_tol = 1e-2 if dt == "fp32" else 1e-3 * kept[0].numel()
    assert abs(float(kept[0].double().sum()) - float(g["prefill_last_sum"])) < total_tol


def test_q05b_fp32_oracle_matches_reference_tokens():
    """Qwen2.5-0.5B shape, fp32, TP=1: 128 greedy tokens identical to the reference's."""
    g = golden("model_q05b_tp1_fp32.npz")
    ids, out, kept = _oracle_generate(mcfg.qwen25_05b(), 1, 128, 128, 1, torch.float32)
    assert np.array_equal(out.numpy(), g["tokens"])
    ref = g["prefill_last_logits"]
    assert np.abs(kept[0].numpy() - ref).max() / np.abs(ref).max() < 1e-4


def _w_oracle_rank(rank, world, name, dtype):
    from minitp_b200 import config as mcfg
    from oracle.model import OracleConfig, prompt
    from oracle.rank import OracleRank

    # q05b: the first 16 of the fixture's 128 greedy steps (a greedy run is prefix-consistent)
    fac, b, p, n = {"tiny": (mcfg.baseline_tiny, 1, 8, 16), "q05b": (mcfg.qwen25_05b, 1, 128, 16)}[name]
    cfg = OracleConfig.of(fac())
    dt = torch.float32 if dtype == "fp32" else torch.bfloat16
    m = OracleRank(cfg, rank, world, dtype=dt)
    return m.generate(prompt(cfg.vocab_size, b, p), n).numpy()


@pytest.mark.distributed
@pytest.mark.parametrize("name,tp,dtype", [("tiny", 1, "fp32"), ("tiny", 2, "fp32"), ("tiny", 2, "bf16"),
                                           ("q05b", 2, "fp32")])
def test_oracle_rank_gloo_matches_reference(name, tp, dtype):
    """The per-rank Gloo restatement (the bench's reference arm) reproduces the reference's ids."""
    from tests.tp_harness import run_tp

    res = run_tp(tp, _w_oracle_rank, name, dtype)
    g = golden(f"model_{name}_tp{tp}_{dtype}.npz")
    for r in range(tp):
        assert np.array_equal(res[r], g["tokens"][:, :res[r].shape[1]]), r
