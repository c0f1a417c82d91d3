"""Multi-GPU parity (>= 2 GPUs): the NVLink kernels against the reference's TP fixtures.

* fused AllReduce + residual + RMSNorm: bit-exact at TP=2 (the reference's
  two-rank bf16 sum rounds once), within the derived rounding bound above;
* embedding and argmax ids: bit-exact, identical on every rank;
* greedy tokens of the TP=2 model: identical to the reference's TP=2 run (fp32);
* a rank that skips a collective makes its peer's bounded wait expire.
"""

import numpy as np
import pytest
import torch

from tests import mp_worker
from tests.conftest import golden

pytestmark = [pytest.mark.gpu, pytest.mark.multi_gpu]


def _world():
    return min(torch.cuda.device_count(), 8)


def test_collectives_match_reference():
    world = 2
    res = mp_worker.run(world, mp_worker.w_collectives)
    g = golden(f"fused_ar_tp{world}.npz")
    ga = golden(f"argmax_tp{world}.npz")
    ge = golden(f"embedding_tp{world}.npz")
    for r in range(1, world):  # identical on every rank
        for k in res[0]:
            assert np.array_equal(res[r][k], res[0][k]), k
    out = res[0]
    for rows in (1, 8, 64, 128, 512, 2048):
        x, y = out[f"res_r{rows}"], out[f"norm_r{rows}"]
        if f"sample_rows_r{rows}" in g:
            sel = g[f"sample_rows_r{rows}"]
            x, y = x[sel], y[sel]
        assert np.array_equal(x, g[f"residual_r{rows}"]), rows  # two-rank bf16 sum: bit-exact
        yf = torch.from_numpy(y).view(torch.bfloat16).float()
        wf = torch.from_numpy(g[f"normed_r{rows}"]).view(torch.bfloat16).float()
        torch.testing.assert_close(yf, wf, atol=0, rtol=2 ** -7)
    for vocab in (151936, 151937):
        for batch in (1, 8, 64):
            assert np.array_equal(out[f"emb_v{vocab}_b{batch}"], ge[f"out_v{vocab}_b{batch}"])
            assert np.array_equal(out[f"argmax_v{vocab}_b{batch}"], ga[f"ids_v{vocab}_b{batch}"])
    assert out["argmax_big"].tolist() == ga["ids_big"].tolist()


@pytest.mark.parametrize("name", ["tiny", "q05b", "q05b_b4"])
def test_tp2_fp32_tokens_match_reference(name):
    res = mp_worker.run(2, mp_worker.w_generate, name, "fp32")
    g = golden(f"model_{name}_tp2_fp32.npz")
    g1 = golden(f"model_{name}_tp1_fp32.npz")
    for r in range(2):
        assert np.array_equal(res[r]["tokens"], g["tokens"]), r
        assert int(res[r]["decode_launches"]) == 1  # the decode megakernel ran
    ref = g1["prefill_last_logits"]
    assert np.abs(res[0]["prefill_last_logits"] - ref).max() / np.abs(ref).max() < 1e-4


def test_tp2_bf16_tokens_and_decode_logits_match_reference():
    """0.5B bf16 at TP=2 against the reference's own TP=2 bf16 run.

    Free-running ids equal the reference's up to its first near-tie; with the
    reference's ids fed to every decode step, each step's top logit is within
    0.5 of the reference's and the ids agree except at near-ties.
    """
    from tests.teacher import check_teacher_tops, check_tokens_up_to_near_tie, merge_rank_tops

    res = mp_worker.run(2, mp_worker.w_teacher, "q05b", "model_q05b_tp2_bf16.npz")
    g = golden("model_q05b_tp2_bf16.npz")
    assert np.array_equal(res[0]["tokens"], res[1]["tokens"])
    for r in range(2):
        assert int(res[r]["decode_launches"]) == 1
    check_tokens_up_to_near_tie(res[0]["tokens"], g["tokens"], g["top2_values"], g["prompt"].shape[1])
    best, best_id = merge_rank_tops([x["top_vals"] for x in res], [x["top_ids"] for x in res])
    check_teacher_tops(best, best_id, g["top2_values"], g["top2_ids"])


def test_tp2_bf16_prefill_logits():
    res = mp_worker.run(2, mp_worker.w_generate, "q05b", "bf16")
    g1 = golden("model_q05b_tp1_bf16.npz")
    assert np.abs(res[0]["prefill_last_logits"] - g1["prefill_last_logits"]).max() < 0.5
    assert np.array_equal(res[0]["tokens"], res[1]["tokens"])


@pytest.mark.parametrize("world,name", [(2, "q05b"), (4, "q7b_l2")])
def test_two_shot_sites_match_one_shot(world, name):
    """The model's AllReduce sites outside the projections in the reduce-scatter + all-gather form:
    prefill logits and greedy tokens bit-identical to the one-shot form, on every rank (bf16)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = mp_worker.run(world, mp_worker.w_two_shot, name)
    for r in range(world):
        assert np.array_equal(res[r]["one_logits"], res[r]["two_logits"]), r
        assert np.array_equal(res[r]["one_tokens"], res[r]["two_tokens"]), r
        assert np.array_equal(res[r]["two_tokens"], res[0]["two_tokens"]), r


def test_tp2_fp32_tokens_two_shot_sites():
    """The TP=2 model with every AllReduce site outside a projection in the two-shot form (prefill
    sites and the final norm): tokens equal the reference's TP=2 run."""
    res = mp_worker.run(2, mp_worker.w_generate, "q05b", "fp32", 0, True)
    g = golden("model_q05b_tp2_fp32.npz")
    for r in range(2):
        assert np.array_equal(res[r]["tokens"], g["tokens"]), r


def test_peer_timeout_is_reported():
    res = mp_worker.run(2, mp_worker.w_peer_timeout)
    assert bool(res[0]["ok_before"]) and bool(res[1]["ok_before"])
    assert np.all(res[0]["first_sum"] == 2.0)
    assert bool(res[0]["raised"])


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs >= 4 GPUs")
def test_tp4_padded_tokens_match_tp1():
    """0.5B at TP=4 needs Q-head padding (14 heads); tokens must equal the TP=1 reference's."""
    res = mp_worker.run(4, mp_worker.w_generate, "q05b_b4", "fp32")
    g1 = golden("model_q05b_b4_tp1_fp32.npz")
    for r in range(4):
        assert np.array_equal(res[r]["tokens"], g1["tokens"]), r
        assert bool(res[r]["heads_padded"])


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs >= 4 GPUs")
def test_tp4_7b_tokens_match_reference_tp4():
    """7B shape (2 layers, fp32) at TP=4: the reference's own TP=4 run (no padding, 1 KV head per rank),
    with the prefill's AllReduce sites in the two-shot form."""
    res = mp_worker.run(4, mp_worker.w_generate, "q7b_l2", "fp32", 0, True)
    g = golden("model_q7b_l2_tp4_fp32.npz")
    g1 = golden("model_q7b_l2_tp1_fp32.npz")
    for r in range(4):
        assert np.array_equal(res[r]["tokens"], g["tokens"]), r
        assert int(res[r]["decode_launches"]) == 1
        assert not bool(res[r]["heads_padded"])
    ref = g1["prefill_last_logits"]
    assert np.abs(res[0]["prefill_last_logits"] - ref).max() / np.abs(ref).max() < 1e-4


@pytest.mark.skipif(torch.cuda.device_count() < 8, reason="needs 8 GPUs")
def test_tp8_7b_padded_replicated_tokens_match_tp1():
    """7B shape at TP=8, which the reference rejects (28 heads): Q heads padded to 32 and each
    of the 4 KV heads replicated on 2 ranks. Tokens must equal the reference's TP=1 run."""
    res = mp_worker.run(8, mp_worker.w_generate, "q7b_l2", "fp32")
    g1 = golden("model_q7b_l2_tp1_fp32.npz")
    for r in range(8):
        assert np.array_equal(res[r]["tokens"], g1["tokens"]), r
        assert int(res[r]["decode_launches"]) == 1
        assert bool(res[r]["heads_padded"])
    ref = g1["prefill_last_logits"]
    assert np.abs(res[0]["prefill_last_logits"] - ref).max() / np.abs(ref).max() < 1e-4
