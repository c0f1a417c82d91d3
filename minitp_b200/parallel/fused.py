"""Per-rank packed projections (reference: minitp/parallel/fused.py:26-113).

Packed row layouts, fixed at load time:
- FusedQKV:    [q_shard; k_shard; v_shard] -> q_local + 2*kv_local rows
- FusedGateUp: [gate_shard; up_shard]      -> 2*inter_local rows
The forward is one GEMV; the split returns views, as in the reference.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from minitp_b200 import ops
from minitp_b200.distributed.context import ParallelContext


class FusedQKVColumnParallelLinear(nn.Module):
    def __init__(
        self,
        hidden_size: int,
        q_out_local: int,
        kv_out_local: int,
        ctx: ParallelContext,
        bias: bool = True,
        init_weights: bool = True,
    ) -> None:
        super().__init__()
        if hidden_size % ctx.tp_size != 0:
            raise ValueError(f"hidden_size={hidden_size} not divisible by tp_size={ctx.tp_size}")
        self.hidden_size = hidden_size
        self.q_out_local = q_out_local
        self.kv_out_local = kv_out_local
        self.ctx = ctx
        out_rows = q_out_local + 2 * kv_out_local
        self.weight = nn.Parameter(torch.empty(out_rows, hidden_size))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_rows))
        else:
            self.register_parameter("bias", None)
        if init_weights:
            nn.init.kaiming_uniform_(self.weight, a=5**0.5)

    def out_features(self) -> int:
        return self.weight.shape[0]

    def forward(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        y = ops.linear(x, self.weight, self.bias)
        q, k, v = torch.split(y, [self.q_out_local, self.kv_out_local, self.kv_out_local], dim=-1)
        return q, k, v


class FusedGateUpColumnParallelLinear(nn.Module):
    def __init__(
        self,
        hidden_size: int,
        intermediate_local: int,
        ctx: ParallelContext,
        bias: bool = False,
        init_weights: bool = True,
    ) -> None:
        super().__init__()
        if intermediate_local * ctx.tp_size == 0 or hidden_size % ctx.tp_size != 0:
            raise ValueError(f"hidden_size={hidden_size} not divisible by tp_size={ctx.tp_size}")
        self.hidden_size = hidden_size
        self.intermediate_local = intermediate_local
        self.ctx = ctx
        self.weight = nn.Parameter(torch.empty(2 * intermediate_local, hidden_size))
        if bias:
            self.bias = nn.Parameter(torch.empty(2 * intermediate_local))
        else:
            self.register_parameter("bias", None)
        if init_weights:
            nn.init.kaiming_uniform_(self.weight, a=5**0.5)

    def forward(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        y = ops.linear(x, self.weight, self.bias)
        return torch.chunk(y, 2, dim=-1)

    def swiglu(self, x: torch.Tensor) -> torch.Tensor:
        """``silu(gate) * up`` fused into the GEMV epilogue (no bias support)."""
        if self.bias is not None:
            raise NotImplementedError("fused SwiGLU epilogue has no bias; Qwen2 gate/up carry none")
        return ops.linear_swiglu(x, self.weight)
