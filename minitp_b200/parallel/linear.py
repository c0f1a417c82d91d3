"""Column- and Row-parallel linear layers.

Same constructors, parameter shapes, sharding and error messages as the
reference (minitp/parallel/linear.py:13-122). The forward runs on the
weight-streaming GEMV kernel; RowParallel's reduction (and the bias, added
once after it) runs in one NVLink AllReduce kernel.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from minitp_b200 import _lib, ops
from minitp_b200.distributed import all_gather
from minitp_b200.distributed.context import ParallelContext


def shard_range(size: int, tp_rank: int, tp_size: int) -> tuple[int, int]:
    """Contiguous [start, end) of a rank; the first ``size % tp`` ranks get one extra.

    Reference: minitp/parallel/linear.py:13-17.
    """
    base, rem = divmod(size, tp_size)
    start = tp_rank * base + min(tp_rank, rem)
    return start, start + base + (1 if tp_rank < rem else 0)


def comm_of(ctx: ParallelContext):
    """The NVLink communicator of ``ctx`` (world-1 communicator for TP=1)."""
    return ctx.comm() if (ctx.tp_size > 1 or ctx.device.type == "cuda") else None


class ColumnParallelLinear(nn.Module):
    """Y = XW with the output dimension sharded (reference linear.py:20-70)."""

    def __init__(
        self,
        input_size: int,
        output_size: int,
        ctx: ParallelContext,
        bias: bool = True,
        gather_output: bool = False,
        init_weights: bool = True,
    ) -> None:
        super().__init__()
        if output_size % ctx.tp_size != 0:
            raise ValueError(f"output_size={output_size} not divisible by tp_size={ctx.tp_size}")
        self.input_size = input_size
        self.output_size = output_size
        self.ctx = ctx
        self.gather_output = gather_output
        self.output_size_local = output_size // ctx.tp_size
        self.output_start, _ = shard_range(output_size, ctx.tp_rank, ctx.tp_size)
        self.weight = nn.Parameter(torch.empty(self.output_size_local, input_size))
        if bias:
            self.bias = nn.Parameter(torch.empty(self.output_size_local))
        else:
            self.register_parameter("bias", None)
        if init_weights:
            nn.init.kaiming_uniform_(self.weight, a=5**0.5)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        local = ops.linear(x, self.weight, self.bias)
        if not self.gather_output or self.ctx.tp_size == 1:
            return local
        out = torch.empty(*local.shape[:-1], self.output_size, dtype=local.dtype, device=local.device)
        return all_gather(out, local, self.ctx.process_group)


class RowParallelLinear(nn.Module):
    """Y = XW with the input dimension sharded; partial sums reduced, bias once.

    Reference: minitp/parallel/linear.py:73-122. The reduction and the bias
    add run in one kernel (``mtpb_allreduce_residual_rmsnorm`` without the
    residual and the norm).
    """

    def __init__(
        self,
        input_size: int,
        output_size: int,
        ctx: ParallelContext,
        bias: bool = True,
        input_is_parallel: bool = True,
        reduce_output: bool = True,
        init_weights: bool = True,
    ) -> None:
        super().__init__()
        if input_size % ctx.tp_size != 0:
            raise ValueError(f"input_size={input_size} not divisible by tp_size={ctx.tp_size}")
        self.input_size = input_size
        self.output_size = output_size
        self.ctx = ctx
        self.input_is_parallel = input_is_parallel
        self.reduce_output = reduce_output
        self.input_size_local = input_size // ctx.tp_size
        self.weight = nn.Parameter(torch.empty(output_size, self.input_size_local))
        if bias:
            self.bias = nn.Parameter(torch.empty(output_size))
        else:
            self.register_parameter("bias", None)
        if init_weights:
            nn.init.kaiming_uniform_(self.weight, a=5**0.5)

    def partial(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's un-reduced ``x_local @ W_local^T`` (no bias)."""
        if not self.input_is_parallel and self.ctx.tp_size > 1:
            x = x.split(self.input_size_local, dim=-1)[self.ctx.tp_rank]
        return ops.linear(x, self.weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        local = self.partial(x)
        reduce = self.reduce_output and self.ctx.tp_size > 1
        if not reduce and self.bias is None:
            return local
        _lib.require_cuda(local)
        comm = self.ctx.comm() if reduce else None
        out, _ = ops.allreduce_residual_rmsnorm(local, None, None, 0.0, comm, bias=self.bias)
        return out
