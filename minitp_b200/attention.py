"""Qwen2 GQA attention over the rank's local heads (reference: minitp/attention.py:22-106).

One fused kernel computes the packed QKV projection, adds the bias, rotates
q and k (RoPE) and appends K/V to the cache. One split-KV kernel then
attends each local query head to its KV head. The cache is never expanded
or repeat-interleaved: query heads of a group share one K/V read. o_proj is
RowParallel. ``partial`` returns its un-reduced output, so the decoder layer
can fuse the AllReduce with the residual add and the next RMSNorm.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from minitp_b200 import ops
from minitp_b200.config import ModelConfig
from minitp_b200.distributed.context import ParallelContext
from minitp_b200.kv_cache import KVCache
from minitp_b200.parallel.fused import FusedQKVColumnParallelLinear
from minitp_b200.parallel.linear import RowParallelLinear
from minitp_b200.rope import RotaryEmbedding


class TPQwen2Attention(nn.Module):
    def __init__(self, cfg: ModelConfig, ctx: ParallelContext, init_weights: bool = True) -> None:
        super().__init__()
        self.cfg = cfg
        self.ctx = ctx
        tp = ctx.tp_size
        self.q_heads_local = cfg.num_attention_heads // tp
        self.kv_replication = cfg.kv_replication(tp)
        self.kv_heads_local = max(1, cfg.num_key_value_heads // tp)
        self.head_dim = cfg.head_dim
        self.q_local = self.q_heads_local * self.head_dim
        self.kv_local = self.kv_heads_local * self.head_dim
        if self.q_heads_local % self.kv_heads_local != 0:
            raise ValueError(
                f"local q heads {self.q_heads_local} not divisible by local kv heads {self.kv_heads_local}"
            )
        self.qkv_proj = FusedQKVColumnParallelLinear(
            cfg.hidden_size, self.q_local, self.kv_local, ctx, bias=True, init_weights=init_weights
        )
        self.o_proj = RowParallelLinear(
            cfg.num_attention_heads * cfg.head_dim, cfg.hidden_size, ctx, bias=False, init_weights=init_weights
        )
        self.use_fused_qkv = True
        self._rotary: RotaryEmbedding | None = None

    def _tables(self, rotary: RotaryEmbedding | None, device) -> RotaryEmbedding:
        if rotary is not None:
            return rotary
        if self._rotary is None or self._rotary.cos_cache.device != device:
            self._rotary = RotaryEmbedding(self.head_dim, self.cfg.rope_theta, self.cfg.max_position_embeddings, device)
        return self._rotary

    def attend(self, x, positions, kv_cache: KVCache | None, layer_idx: int, rotary=None) -> torch.Tensor:
        """Attention output ``[B, T, q_local]`` before o_proj."""
        b, t, _ = x.shape
        if kv_cache is None:  # attend over the T new tokens only (cache_len 0)
            kv_cache = KVCache(1, b, self.kv_heads_local, self.head_dim, t, x.dtype, x.device)
            layer_idx = 0
        kv_cache.check_room(t)
        cache_len = kv_cache.seq_len
        rot = self._tables(rotary, x.device)
        q = ops.qkv_rope(
            x, self.qkv_proj.weight, self.qkv_proj.bias, kv_cache.k[layer_idx], kv_cache.v[layer_idx],
            self.q_heads_local, self.kv_heads_local, cache_len, positions, rot.cos_cache, rot.sin_cache,
        )
        return ops.attention(q, kv_cache.k[layer_idx], kv_cache.v[layer_idx], self.q_heads_local,
                             self.kv_heads_local, cache_len)

    def partial(self, x, positions, kv_cache, layer_idx, rotary=None) -> torch.Tensor:
        """This rank's un-reduced o_proj output."""
        return self.o_proj.partial(self.attend(x, positions, kv_cache, layer_idx, rotary))

    def forward(self, x, positions, kv_cache: KVCache | None, layer_idx: int, rotary=None) -> torch.Tensor:
        return self.o_proj(self.attend(x, positions, kv_cache, layer_idx, rotary))
