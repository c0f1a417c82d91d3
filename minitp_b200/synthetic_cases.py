"""Seeded inputs for the operator microbenchmarks and their parity tests.

Each generator is deterministic on the CPU (``torch.Generator``), so a parity
fixture recorded from the reference can be checked on another machine by
regenerating the same inputs from the seed.
"""

from __future__ import annotations

import torch


def argmax_logits(vocab: int, batch: int, seed: int = 0, tie_frac: float = 0.1) -> torch.Tensor:
    """fp32 logits ``[batch, vocab]`` ~ N(0, 3) with exact cross-shard ties.

    In every ``round(1/tie_frac)``-th row two ids receive the same value, above
    every other logit of the row. Both ids then hold the row maximum, so the
    lower id must win. The pair alternates between:

    * a "far" pair, one id in the first eighth of the vocab and one in the last
      eighth. They sit in different shards for tp = 2, 4 and 8.
    * an "adjacent" pair straddling the tp=2 shard boundary (last id of shard 0,
      first id of shard 1).
    """
    g = torch.Generator()
    g.manual_seed(seed)
    x = torch.randn(batch, vocab, generator=g) * 3.0
    every = max(1, round(1.0 / tie_frac)) if tie_frac > 0 else 0
    if every:
        half = (vocab + 1) // 2  # shard_range(vocab, 0, 2) end
        eighth = max(1, vocab // 8)
        for row in range(0, batch, every):
            top = float(x[row].max()) + 1.0
            if (row // every) % 2 == 0:
                a = int(torch.randint(0, eighth, (1,), generator=g))
                b = int(torch.randint(vocab - eighth, vocab, (1,), generator=g))
            else:
                a, b = half - 1, half
            x[row, a] = top
            x[row, b] = top
    return x


def embedding_case(vocab: int, hidden: int, batch: int, seed: int = 0):
    """bf16 table ``[vocab, hidden]`` ~ N(0, 0.02) and ids ``[batch, 1]`` uniform in [0, vocab)."""
    g = torch.Generator()
    g.manual_seed(seed)
    table = (torch.randn(vocab, hidden, generator=g) * 0.02).to(torch.bfloat16)
    ids = torch.randint(0, vocab, (batch, 1), generator=g)
    return table, ids


def fused_ar_case(rows: int, hidden: int, tp: int, seed: int = 0, dtype=torch.bfloat16):
    """Per-rank partials ``[tp, rows, hidden]`` ~ N(0,1), residual ~ N(0,1), gain ~ N(1, 0.1)."""
    g = torch.Generator()
    g.manual_seed(seed)
    partials = torch.randn(tp, rows, hidden, generator=g).to(dtype)
    residual = torch.randn(rows, hidden, generator=g).to(dtype)
    gain = (1.0 + 0.1 * torch.randn(hidden, generator=g)).to(dtype)
    return partials, residual, gain
