"""Teacher-forced decode logits and the near-tie rule of the bf16 parity checks.

bf16 runs sum the GEMV products in another order than the reference's
cuBLAS, so a greedy id may flip where the reference's top two logits are
within a few bf16 ulps; after such a flip the two sequences diverge and
later logits are not comparable. Feeding the reference's own ids to every
decode step ("teacher forcing") keeps the inputs identical, so the logits of
every step can be checked against the reference's top-2 values recorded in
the fixture (minitp/generation.py:54-67 picks the top-1 of those logits).
"""

from __future__ import annotations

import numpy as np
import torch

# a greedy id may differ only where the reference's top-2 gap is this many
# bf16 ulps (at the top logit's magnitude) or less
NEAR_TIE_ULPS = 4


def bf16_ulp(x: float) -> float:
    return float(2.0 ** (np.floor(np.log2(abs(x))) - 7)) if x != 0 else 2.0 ** -133


def local_top2(logits: torch.Tensor, vstart: int) -> tuple[np.ndarray, np.ndarray]:
    """Top-2 values (fp32) and global ids of local logits ``[B, V_local]``; ties -> lowest id."""
    lf = logits.float()
    vals, idx = torch.topk(lf, 2, dim=-1, sorted=True)
    # torch.topk does not promise the lowest index among equal values: fix ties
    first = torch.argmax(lf, dim=-1)  # lowest index of the maximum
    idx[:, 0] = first
    return vals.cpu().numpy(), (idx + vstart).cpu().numpy()


def teacher_forced_tops(model, prompt: torch.Tensor, ref_tokens: torch.Tensor, n: int, keep_steps=()):
    """Per-step local top-2 of the decode logits, fed the reference's ids.

    Step 0 is the prefill's last position; step s >= 1 is the decode step
    whose input is ``ref_tokens[:, P + s - 1]``, run through the library's
    decode step (the decode megakernel when it plans the shape) with a logits
    output. Returns (values [n, B, 2], global ids [n, B, 2], {step: local
    logits [B, V_local] fp32} for the steps in ``keep_steps``).
    """
    from minitp_b200 import _lib
    from minitp_b200.generation import GenerationState

    b, p = prompt.shape
    vstart = int(model.lm_head.vocab_start)
    st = GenerationState(model, prompt, n)
    lg = st.prefill(last_only=True)[:, -1]
    vals, ids, kept = [], [], {}
    v, i = local_top2(lg, vstart)
    vals.append(v)
    ids.append(i)
    if 0 in keep_steps:
        kept[0] = lg.float().cpu().numpy()
    tok = ref_tokens[:, p].clone()
    st.append(tok)
    st.start_device_decode(tok)
    vloc = model.lm_head.weight.shape[0]
    out = torch.empty(b, vloc, dtype=model.lm_head.weight.dtype, device=prompt.device)
    kp, vp = st.kv.pointer_arrays()
    stream = _lib.stream_ptr(prompt.device)
    for s in range(1, n):
        st._tok.copy_(ref_tokens[:, p + s - 1])  # the decode step overwrites it with its own pick
        st.kv.check_room(1)
        _lib.call("mtpb_model_decode_step", model.native(), st._tok.data_ptr(), b, kp, vp, st.kv.max_seq_len,
                  None, 0, out.data_ptr(), stream)
        st.kv.advance(1)
        v, i = local_top2(out, vstart)
        vals.append(v)
        ids.append(i)
        if s in keep_steps:
            kept[s] = out.float().cpu().numpy()
    torch.cuda.synchronize()
    st.release()
    return np.stack(vals), np.stack(ids), kept


def merge_rank_tops(vals: list[np.ndarray], ids: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
    """Global top-1 value and id per (step, row) from every rank's local top-2 (lowest id on ties)."""
    v = np.stack([x[..., 0] for x in vals])  # [ranks, n, B]
    i = np.stack([x[..., 0] for x in ids])
    best = v.max(axis=0)
    cand = np.where(v == best[None], i, np.iinfo(np.int64).max)
    return best, cand.min(axis=0)


def check_tokens_up_to_near_tie(got: np.ndarray, want: np.ndarray, top2_values: np.ndarray, prompt_len: int):
    """Generated ids equal the reference's up to its first near-tie (then stop comparing)."""
    for row in range(got.shape[0]):
        g, w = got[row, prompt_len:], want[row, prompt_len:prompt_len + got.shape[1] - prompt_len]
        bad = np.flatnonzero(g != w)
        if bad.size:
            s = int(bad[0])
            top = top2_values[s, row].astype(np.float64)
            assert top[0] - top[1] <= NEAR_TIE_ULPS * bf16_ulp(top[0]), \
                f"row {row} step {s}: ids differ without a reference near-tie (top2 {top.tolist()})"


def check_teacher_tops(best: np.ndarray, best_id: np.ndarray, top2_values: np.ndarray, top2_ids: np.ndarray,
                       atol: float = 0.5):
    """Every step's top logit within `atol` of the reference's; ids equal unless a near-tie."""
    n = best.shape[0]
    ref_v = top2_values[:n].astype(np.float64)
    err = np.abs(best - ref_v[..., 0])
    assert err.max() < atol, f"top logit off by {err.max():.3f} at step {int(np.argmax(err.max(axis=-1)))}"
    diff = np.argwhere(best_id != top2_ids[:n, :, 0])
    for s, row in diff:
        top = ref_v[s, row]
        assert top[0] - top[1] <= NEAR_TIE_ULPS * bf16_ulp(top[0]), \
            f"step {s} row {row}: teacher-forced id differs without a near-tie (top2 {top.tolist()})"
