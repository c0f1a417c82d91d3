"""RMSNorm, the TP decoder layer and the full TP Qwen2 model.

Reference: minitp/layer.py:19-124. Module tree, parameter names and
state_dict keys are the reference's, so checkpoints load unchanged.

``TPQwen2ForCausalLM.forward`` runs the whole model as one chain of
minitp_b200 kernels. The chain is built by the native sequencer
(``mtpb_model_forward``) over the module's own parameter tensors:
  embedding (push) -> per layer: [AR + residual + RMSNorm + fused QKV/RoPE/KV]
  -> attention -> [o_proj GEMV + NVLink push] -> [AR + residual + RMSNorm +
  gate/up + SwiGLU] -> [down GEMV + push] -> AR + final norm + LM head.
Every RowParallel AllReduce is fused into the kernel that consumes it.
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn as nn

from minitp_b200 import _lib, ops
from minitp_b200.attention import TPQwen2Attention
from minitp_b200.config import ModelConfig
from minitp_b200.distributed.context import ParallelContext
from minitp_b200.kv_cache import KVCache
from minitp_b200.mlp import TPQwen2MLP
from minitp_b200.parallel.embedding import VocabParallelEmbedding, VocabParallelLMHead
from minitp_b200.rope import RotaryEmbedding


class RMSNorm(nn.Module):
    """``T(x * rsqrt(mean(x^2) + eps) * w)`` in fp32 math (reference layer.py:19-42)."""

    def __init__(self, hidden_size: int, eps: float, init_weights: bool = True) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size) if init_weights else torch.empty(hidden_size))
        self.eps = eps
        self.implementation = "fused"  # a single minitp_b200 kernel

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rmsnorm(x, self.weight, self.eps)


class TPQwen2DecoderLayer(nn.Module):
    """``x = x + attn(norm1(x)); x = x + mlp(norm2(x))`` (reference layer.py:45-65).

    Both RowParallel reductions are fused with the residual add that follows
    them, and the first with the post-attention RMSNorm.
    """

    def __init__(self, cfg: ModelConfig, ctx: ParallelContext, init_weights: bool = True) -> None:
        super().__init__()
        self.ctx = ctx
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, init_weights=init_weights)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, init_weights=init_weights)
        self.self_attn = TPQwen2Attention(cfg, ctx, init_weights=init_weights)
        self.mlp = TPQwen2MLP(cfg, ctx, init_weights=init_weights)

    def forward(self, x, positions, kv_cache: KVCache | None, layer_idx: int, rotary=None) -> torch.Tensor:
        comm = self.ctx.comm() if self.ctx.tp_size > 1 else None
        h = self.input_layernorm(x)
        attn = self.self_attn.partial(h, positions, kv_cache, layer_idx, rotary)
        ln2 = self.post_attention_layernorm
        x1, h2 = ops.allreduce_residual_rmsnorm(attn, x, ln2.weight, ln2.eps, comm)
        x2, _ = ops.allreduce_residual_rmsnorm(self.mlp.partial(h2), x1, None, 0.0, comm)
        return x2


class TPQwen2ForCausalLM(nn.Module):
    def __init__(self, cfg: ModelConfig, ctx: ParallelContext, init_weights: bool = True) -> None:
        super().__init__()
        self.cfg = cfg
        self.ctx = ctx
        self.init_weights = init_weights
        self.rotary: RotaryEmbedding | None = None
        self.use_rotary_cache = True
        self.model = nn.Module()
        self.model.embed_tokens = VocabParallelEmbedding(cfg.vocab_size, cfg.hidden_size, ctx, init_weights)
        self.model.layers = nn.ModuleList(
            TPQwen2DecoderLayer(cfg, ctx, init_weights) for _ in range(cfg.num_hidden_layers)
        )
        self.model.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, init_weights)
        self.lm_head = VocabParallelLMHead(cfg.hidden_size, cfg.vocab_size, ctx, init_weights=init_weights)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight
        self._native_handle = None
        self._native_key = None
        self._native_keepalive = None

    # ------------------------------------------------------------------
    # native model (weights stay in this module's parameters)
    # ------------------------------------------------------------------
    def _rotary_tables(self, device) -> RotaryEmbedding:
        if self.rotary is None or self.rotary.cos_cache.device != device:
            self.rotary = RotaryEmbedding(self.cfg.head_dim, self.cfg.rope_theta,
                                          self.cfg.max_position_embeddings, device)
        return self.rotary

    def native(self) -> int:
        """Handle of the native model over the current parameter tensors (rebuilt if they moved)."""
        params = [self.model.embed_tokens.weight, self.lm_head.weight, self.model.norm.weight]
        for layer in self.model.layers:
            a, m = layer.self_attn, layer.mlp
            params += [layer.input_layernorm.weight, a.qkv_proj.weight, a.qkv_proj.bias, a.o_proj.weight,
                       layer.post_attention_layernorm.weight, m.gate_up_proj.weight, m.down_proj.weight]
        key = tuple(0 if p is None else p.data_ptr() for p in params)
        if self._native_handle is not None and key == self._native_key:
            return self._native_handle
        dev = self.model.embed_tokens.weight.device
        _lib.require_cuda(self.model.embed_tokens.weight)
        dtype = self.model.embed_tokens.weight.dtype
        for p in params:
            if p is not None and (p.dtype != dtype or not p.is_contiguous() or p.device != dev):
                raise _lib.MinitpB200Error("native model: parameters must be contiguous, one dtype, one device")
        self.release_native()
        cfg, ctx = self.cfg, self.ctx
        rot = self._rotary_tables(dev)
        attn0 = self.model.layers[0].self_attn
        d = _lib.ModelDesc(
            dtype=_lib.dtype_code(dtype), hidden=cfg.hidden_size,
            inter_local=self.model.layers[0].mlp.intermediate_local, n_layers=cfg.num_hidden_layers,
            hq_local=attn0.q_heads_local, hkv_local=attn0.kv_heads_local, head_dim=cfg.head_dim,
            vocab_start=self.lm_head.vocab_start, vocab_end=self.lm_head.vocab_end, vocab_size=cfg.vocab_size,
            eps=cfg.rms_norm_eps, embed=self.model.embed_tokens.weight.data_ptr(),
            lm_head=self.lm_head.weight.data_ptr(), final_norm=self.model.norm.weight.data_ptr(),
            cos_tab=rot.cos_cache.data_ptr(), sin_tab=rot.sin_cache.data_ptr(), rope_len=rot.max_seq_len,
        )
        h = ctypes.c_void_p()
        with torch.cuda.device(dev):
            comm = ctx.comm()
            _lib.call("mtpb_model_create", ctypes.byref(d), comm.handle, ctypes.byref(h))
            for i, layer in enumerate(self.model.layers):
                a, m = layer.self_attn, layer.mlp
                ld = _lib.LayerDesc(
                    ln1=layer.input_layernorm.weight.data_ptr(), qkv_w=a.qkv_proj.weight.data_ptr(),
                    qkv_b=_lib.ptr(a.qkv_proj.bias), o_w=a.o_proj.weight.data_ptr(),
                    ln2=layer.post_attention_layernorm.weight.data_ptr(),
                    gu_w=m.gate_up_proj.weight.data_ptr(), down_w=m.down_proj.weight.data_ptr(),
                )
                _lib.call("mtpb_model_set_layer", h.value, i, ctypes.byref(ld))
        self._native_handle = h.value
        self._native_key = key
        self._native_keepalive = rot
        return self._native_handle

    def release_native(self) -> None:
        # decode sessions hold graphs captured over the native model's buffers
        self.__dict__.pop("_decode_sessions", None)
        if self._native_handle is not None:
            torch.cuda.synchronize(self.model.embed_tokens.weight.device)
            _lib.load().mtpb_model_destroy(self._native_handle)
            self._native_handle = None
            self._native_key = None

    def __del__(self):
        try:
            self.release_native()
        except Exception:
            pass

    # ------------------------------------------------------------------
    def forward(
        self,
        input_ids: torch.Tensor,  # [B, T]
        positions: torch.Tensor | None = None,  # [T]
        kv_cache: KVCache | None = None,
        gather_logits: bool = False,
        last_only: bool = False,
    ) -> torch.Tensor:
        """Logits ``[B, T, V_local]`` (``[B, 1, V_local]`` with ``last_only``).

        Reference: minitp/layer.py:91-124. ``last_only`` computes the LM head
        for the last token only (what greedy selection consumes); the other
        rows are not materialised.
        """
        _lib.require_cuda(input_ids)
        b, t = input_ids.shape
        h = self.native()
        kv = kv_cache
        if kv is None:
            attn0 = self.model.layers[0].self_attn
            kv = KVCache(self.cfg.num_hidden_layers, b, attn0.kv_heads_local, self.cfg.head_dim, t,
                         self.model.embed_tokens.weight.dtype, input_ids.device)
        kv.check_room(t)
        rope_pos = None
        if positions is not None:
            rope_pos = positions.reshape(-1)
            if rope_pos.dtype != torch.int64:
                rope_pos = rope_pos.to(torch.int64)
            rope_pos = rope_pos.contiguous()
        elif t > 1 and kv.seq_len > 0:
            # the reference numbers multi-token inputs from 0 when no positions are given
            rope_pos = torch.arange(t, device=input_ids.device)
        ids = input_ids.contiguous()
        if ids.dtype != torch.int64:
            ids = ids.to(torch.int64)
        rows = b if last_only else b * t
        vloc = self.lm_head.vocab_end - self.lm_head.vocab_start
        logits = torch.empty(rows, vloc, dtype=self.model.embed_tokens.weight.dtype, device=input_ids.device)
        kp, vp = kv.pointer_arrays()
        _lib.call("mtpb_model_forward", h, ids.data_ptr(), b, t, _lib.ptr(rope_pos), kv.seq_len, kp, vp,
                  kv.max_seq_len, logits.data_ptr(), 1 if last_only else 0, _lib.stream_ptr(input_ids.device))
        if kv_cache is not None:
            kv_cache.advance(t)
        out = logits.view(b, 1 if last_only else t, vloc)
        if gather_logits and self.ctx.tp_size > 1:
            return self.lm_head.gather(out)
        return out
