"""Qwen2 SwiGLU MLP (reference: minitp/mlp.py:18-38).

gate/up is one GEMV with ``silu(gate) * up`` in its epilogue; down is
RowParallel (``partial`` returns the un-reduced output for the fused
AllReduce + residual path of the decoder layer).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from minitp_b200.config import ModelConfig
from minitp_b200.distributed.context import ParallelContext
from minitp_b200.parallel.fused import FusedGateUpColumnParallelLinear
from minitp_b200.parallel.linear import RowParallelLinear


class TPQwen2MLP(nn.Module):
    def __init__(self, cfg: ModelConfig, ctx: ParallelContext, init_weights: bool = True) -> None:
        super().__init__()
        self.intermediate_local = cfg.intermediate_size // ctx.tp_size
        self.gate_up_proj = FusedGateUpColumnParallelLinear(
            cfg.hidden_size, self.intermediate_local, ctx, bias=False, init_weights=init_weights
        )
        self.down_proj = RowParallelLinear(
            cfg.intermediate_size, cfg.hidden_size, ctx, bias=False, init_weights=init_weights
        )
        self.use_fused_gateup = True

    def partial(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj.partial(self.gate_up_proj.swiglu(x))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(self.gate_up_proj.swiglu(x))
