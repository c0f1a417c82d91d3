"""Vocab-parallel embedding and LM head, plus distributed greedy argmax.

Reference: minitp/parallel/embedding.py:24-228. Same constructors, shard
ranges (uneven vocab: contiguous ranges, rank 0 first), return shapes and
errors. The lookup, the logits and the argmax run in minitp_b200 kernels;
the argmax exchanges one packed int64 per row and rank over NVLink.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from minitp_b200 import ops
from minitp_b200.distributed import all_gather
from minitp_b200.distributed.context import ParallelContext
from minitp_b200.parallel.linear import shard_range

# The reference's module default (embedding.py:21). Every encoding gives the
# same ids on this path (one packed key per row and rank); "fp32" keeps the
# reference's guard for vocabularies above 2**24.
ARGMAX_ENCODING = "bitpack"
_ENCODINGS = ("bitpack", "fp32", "fp64", "split")


def _comm(ctx: ParallelContext):
    return ctx.comm() if ctx.device.type == "cuda" else None


class VocabParallelEmbedding(nn.Module):
    def __init__(
        self, vocab_size: int, hidden_size: int, ctx: ParallelContext, init_weights: bool = True
    ) -> None:
        super().__init__()
        self.vocab_size = vocab_size
        self.hidden_size = hidden_size
        self.ctx = ctx
        start, end = shard_range(vocab_size, ctx.tp_rank, ctx.tp_size)
        self.vocab_start, self.vocab_end = start, end
        self.weight = nn.Parameter(
            torch.zeros(end - start, hidden_size) if init_weights else torch.empty(end - start, hidden_size)
        )
        self.tp1_fast = True  # kept for the reference's feature flags

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        return ops.embedding(ids, self.weight, self.vocab_start, self.vocab_end, self.vocab_size, _comm(self.ctx))


class VocabParallelLMHead(nn.Module):
    def __init__(
        self,
        hidden_size: int,
        vocab_size: int,
        ctx: ParallelContext,
        gather_logits: bool = False,
        init_weights: bool = True,
    ) -> None:
        super().__init__()
        self.vocab_size = vocab_size
        self.hidden_size = hidden_size
        self.ctx = ctx
        self.gather_logits = gather_logits
        start, end = shard_range(vocab_size, ctx.tp_rank, ctx.tp_size)
        self.vocab_start, self.vocab_end = start, end
        self.weight = nn.Parameter(
            torch.zeros(end - start, hidden_size) if init_weights else torch.empty(end - start, hidden_size)
        )

    def _max_local_vocab(self) -> int:
        base, rem = divmod(self.vocab_size, self.ctx.tp_size)
        return base + (1 if rem else 0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        local = ops.linear(x, self.weight)
        if not self.gather_logits or self.ctx.tp_size == 1:
            return local
        return self.gather(local)

    def gather(self, local: torch.Tensor) -> torch.Tensor:
        """Full-vocab logits from every rank's shard (debug / correctness path)."""
        out = torch.empty(*local.shape[:-1], self.vocab_size, dtype=local.dtype, device=local.device)
        if self.vocab_size % self.ctx.tp_size == 0:
            all_gather(out, local, self.ctx.process_group)
            return out
        mx = self._max_local_vocab()
        padded = torch.nn.functional.pad(local, (0, mx - local.shape[-1]))
        gathered = torch.empty(*local.shape[:-1], self.ctx.tp_size * mx, dtype=local.dtype, device=local.device)
        all_gather(gathered, padded, self.ctx.process_group)
        for r in range(self.ctx.tp_size):
            s, e = shard_range(self.vocab_size, r, self.ctx.tp_size)
            out[..., s:e] = gathered[..., r * mx : r * mx + (e - s)]
        return out

    @torch.no_grad()
    def distributed_argmax(self, local_logits: torch.Tensor, encoding: str | None = None) -> torch.Tensor:
        """Greedy next-token id over the sharded vocab -> ``[..., 1]`` long, same on all ranks.

        Reference: embedding.py:118-213. Ties resolve to the smallest id; with
        tp > 1 a NaN logit cannot win, with tp == 1 NaN behaves as in
        ``torch.argmax``.
        """
        enc = encoding or ARGMAX_ENCODING
        if enc not in _ENCODINGS:
            raise ValueError(f"unknown argmax encoding {enc!r}")
        if enc == "fp32" and self.ctx.tp_size > 1 and self.vocab_size > 2**24:
            raise ValueError(
                f"fp32 argmax encoding cannot represent ids >= 2**24 exactly "
                f"(vocab_size={self.vocab_size}); use the bitpack encoding"
            )
        return ops.argmax(local_logits, self.vocab_start, _comm(self.ctx))
