"""Process-group context and collective wrappers (reference: minitp/distributed)."""

from minitp_b200.distributed.collectives import (
    CommStats,
    all_gather,
    all_gather_dim0,
    all_reduce,
    broadcast,
    comm_summary,
    drain_comm_stats,
    get_comm_stats,
    reduce_scatter,
    reset_comm_stats,
    set_profiling,
)
from minitp_b200.distributed.context import ParallelContext, context_for, init_context

__all__ = [
    "CommStats",
    "ParallelContext",
    "context_for",
    "init_context",
    "all_reduce",
    "all_gather",
    "all_gather_dim0",
    "reduce_scatter",
    "broadcast",
    "set_profiling",
    "get_comm_stats",
    "drain_comm_stats",
    "comm_summary",
    "reset_comm_stats",
]
