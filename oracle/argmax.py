"""Greedy argmax oracle in numpy integer arithmetic.

Restates ``VocabParallelLMHead.distributed_argmax`` with the bitpack
encoding (reference minitp/parallel/embedding.py:118-172) and its TP=1 fast
path (``local_logits.argmax``, embedding.py:146-147).
"""

from __future__ import annotations

import numpy as np


def shard_range(size: int, rank: int, tp: int) -> tuple[int, int]:
    """minitp/parallel/linear.py:13-17."""
    base, rem = divmod(size, tp)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def _keys(values: np.ndarray) -> np.ndarray:
    """Monotone fp32 -> signed key (embedding.py:159-166), -0.0 normalised to +0.0."""
    v = np.where(values == 0, np.float32(0), values.astype(np.float32))
    bits = v.view(np.uint32).astype(np.int64)
    neg = ((~bits) & 0xFFFFFFFF) - 0x80000000
    return np.where(bits < 0x80000000, bits, neg)


def local_best(local_logits: np.ndarray, vocab_start: int) -> np.ndarray:
    """Packed int64 of one rank: NaN -> -inf, first max, (key << 32) | (2^32-1 - id).

    embedding.py:152-167.
    """
    x = np.asarray(local_logits, dtype=np.float32)
    clean = np.where(np.isnan(x), np.float32(-np.inf), x)
    idx = clean.argmax(axis=-1)  # first occurrence of the max
    vals = np.take_along_axis(clean, idx[..., None], axis=-1)[..., 0]
    gid = idx.astype(np.int64) + vocab_start
    return (_keys(vals) << 32) | (0xFFFFFFFF - gid)


def distributed_argmax(full_logits: np.ndarray, tp: int) -> np.ndarray:
    """Ids ``[...]`` of the bitpack path for a vocab sharded over ``tp`` ranks.

    tp == 1 follows torch.argmax (NaN wins, first occurrence), as the
    reference's fast path does (embedding.py:146-147).
    """
    x = np.asarray(full_logits, dtype=np.float32)
    v = x.shape[-1]
    if tp == 1:
        nan = np.isnan(x)
        first_nan = nan.argmax(axis=-1)
        plain = x.argmax(axis=-1)
        return np.where(nan.any(axis=-1), first_nan, plain).astype(np.int64)
    packed = []
    for r in range(tp):
        s, e = shard_range(v, r, tp)
        packed.append(local_best(x[..., s:e], s))
    winner = np.max(np.stack(packed, axis=-1), axis=-1)  # embedding.py:169-171
    return (0xFFFFFFFF - (winner & 0xFFFFFFFF)).astype(np.int64)
