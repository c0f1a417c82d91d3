"""TP layers (reference: minitp/parallel)."""

from minitp_b200.parallel.embedding import VocabParallelEmbedding, VocabParallelLMHead
from minitp_b200.parallel.fused import FusedGateUpColumnParallelLinear, FusedQKVColumnParallelLinear
from minitp_b200.parallel.linear import ColumnParallelLinear, RowParallelLinear, shard_range

__all__ = [
    "ColumnParallelLinear",
    "RowParallelLinear",
    "FusedQKVColumnParallelLinear",
    "FusedGateUpColumnParallelLinear",
    "VocabParallelEmbedding",
    "VocabParallelLMHead",
    "shard_range",
]
