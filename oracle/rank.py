"""One rank of the reference's CPU/Gloo decode path (test infrastructure and CPU baseline).

Restates, for ONE tensor-parallel rank in its own process, what the
reference's modules do per decode step, with real ``torch.distributed``
collectives on the Gloo backend (the reference's CPU path,
minitp/distributed/context.py:61-76):

* VocabParallelEmbedding: masked local lookup, SUM all_reduce
  (minitp/parallel/embedding.py:44-50);
* per layer: RMSNorm (layer.py:36-42), fused QKV F.linear with bias
  (parallel/fused.py:57-61), RoPE in fp32 (rope.py:47-64), KV-cache write
  (kv_cache.py:43-55), GQA expand / repeat_interleave +
  F.scaled_dot_product_attention (attention.py:77-103), o_proj partial +
  all_reduce (parallel/linear.py:111-122), residual (layer.py:64), RMSNorm,
  gate/up F.linear, silu * up, down partial + all_reduce, residual
  (mlp.py:34-38, layer.py:65);
* final RMSNorm, local LM-head logits (embedding.py:87-90) and the bitpack
  distributed argmax with one O(tp) all_gather (embedding.py:118-172; Gloo
  takes the list form of collectives.py:185-214).

It is not part of the product: ``tests/`` check it against the reference's
fixtures, and ``bench.py --impl reference`` times it as the reference's CPU
path (one process per rank, ``cores // tp`` threads each).

Weights: ``weights="seeded"`` slices the seeded synthetic checkpoint (the
protocol of the parity fixtures); ``weights="fill"`` fills every shard from a
small random tile (same shapes and dtype, same arithmetic cost, no
generator pass over billions of values), for timing large shapes.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn.functional as F

from oracle.argmax import shard_range
from oracle.model import OracleConfig, checkpoint_tensors, kv_head_rows, rmsnorm, rope_tables


def _fill(shape, dtype, seed: int) -> torch.Tensor:
    """A tensor of `shape` tiled from a 1 Mi-element N(0, 0.02) block (fast to build)."""
    g = torch.Generator().manual_seed(seed)
    tile = (torch.randn(1 << 20, generator=g) * 0.02).to(dtype)
    n = math.prod(shape)
    out = torch.empty(n, dtype=dtype)
    for o in range(0, n, tile.numel()):
        k = min(tile.numel(), n - o)
        out[o:o + k] = tile[:k]
    return out.view(shape)


class OracleRank:
    """The reference TP model as seen by rank ``rank`` of ``tp`` (Gloo collectives)."""

    def __init__(self, cfg: OracleConfig, rank: int, tp: int, dtype: torch.dtype = torch.float32,
                 weights: str = "seeded", tensors: dict | None = None, group=None) -> None:
        if cfg.num_attention_heads % tp:
            # the reference's ModelConfig.validate (minitp/config.py:50-61)
            raise ValueError(f"num_attention_heads={cfg.num_attention_heads} not divisible by tp_size={tp}")
        self.cfg, self.rank, self.tp, self.dtype, self.group = cfg, rank, tp, dtype, group
        hd, H, I, V = cfg.head_dim, cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
        self.hq = cfg.num_attention_heads // tp
        self.hkv = max(1, cfg.num_key_value_heads // tp)
        self.vstart, self.vend = shard_range(V, rank, tp)
        q0, q1 = shard_range(cfg.num_attention_heads * hd, rank, tp)
        k0, kn = kv_head_rows(cfg.num_key_value_heads, hd, rank, tp)
        i0, i1 = shard_range(I, rank, tp)
        cast = lambda t: t.to(dtype).contiguous()  # noqa: E731
        if weights == "seeded":
            t = tensors if tensors is not None else checkpoint_tensors(cfg)
            self.embed = cast(t["model.embed_tokens.weight"][self.vstart:self.vend])
            head = t["model.embed_tokens.weight"] if cfg.tie_word_embeddings else t["lm_head.weight"]
            self.lm_head = cast(head[self.vstart:self.vend])
            self.norm = cast(t["model.norm.weight"])
            self.layers = []
            for i in range(cfg.num_hidden_layers):
                p = f"model.layers.{i}."
                self.layers.append(dict(
                    ln1=cast(t[p + "input_layernorm.weight"]), ln2=cast(t[p + "post_attention_layernorm.weight"]),
                    qkv_w=cast(torch.cat([t[p + "self_attn.q_proj.weight"][q0:q1],
                                          t[p + "self_attn.k_proj.weight"][k0:k0 + kn],
                                          t[p + "self_attn.v_proj.weight"][k0:k0 + kn]])),
                    qkv_b=cast(torch.cat([t[p + "self_attn.q_proj.bias"][q0:q1],
                                          t[p + "self_attn.k_proj.bias"][k0:k0 + kn],
                                          t[p + "self_attn.v_proj.bias"][k0:k0 + kn]])),
                    o_w=cast(t[p + "self_attn.o_proj.weight"][:, q0:q1]),
                    gu_w=cast(torch.cat([t[p + "mlp.gate_proj.weight"][i0:i1], t[p + "mlp.up_proj.weight"][i0:i1]])),
                    down_w=cast(t[p + "mlp.down_proj.weight"][:, i0:i1])))
        elif weights == "fill":
            s = 1000 * rank
            nq, nkv, il = q1 - q0, kn, i1 - i0
            self.embed = _fill((self.vend - self.vstart, H), dtype, s + 1)
            self.lm_head = self.embed if cfg.tie_word_embeddings else _fill((self.vend - self.vstart, H), dtype, s + 2)
            self.norm = torch.ones(H, dtype=dtype)
            self.layers = []
            for i in range(cfg.num_hidden_layers):
                self.layers.append(dict(
                    ln1=torch.ones(H, dtype=dtype), ln2=torch.ones(H, dtype=dtype),
                    qkv_w=_fill((nq + 2 * nkv, H), dtype, s + 10 * i + 3),
                    qkv_b=_fill((nq + 2 * nkv,), dtype, s + 10 * i + 4),
                    o_w=_fill((H, nq), dtype, s + 10 * i + 5),
                    gu_w=_fill((2 * il, H), dtype, s + 10 * i + 6),
                    down_w=_fill((H, il), dtype, s + 10 * i + 7)))
        else:
            raise ValueError(f"unknown weights mode {weights!r}")
        self.cos, self.sin = rope_tables(hd, cfg.rope_theta, cfg.max_position_embeddings)
        self.k = self.v = None
        self.seq_len = 0

    # ------------------------------------------------------------------ collectives
    def _all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.tp > 1:
            dist.all_reduce(t, group=self.group)  # collectives.py:147-157
        return t

    def reset(self, batch: int, max_seq: int, fill_len: int = 0) -> None:
        """Fresh KV caches [B, hkv, max_seq, hd] (kv_cache.py:18-41); `fill_len` slots pre-filled
        with N(0, 1) values and the cursor set past them (timing runs without a prefill)."""
        L, hd = self.cfg.num_hidden_layers, self.cfg.head_dim
        z = lambda: torch.zeros(batch, self.hkv, max_seq, hd, dtype=self.dtype)  # noqa: E731
        self.k = [z() for _ in range(L)]
        self.v = [z() for _ in range(L)]
        if fill_len:
            g = torch.Generator().manual_seed(7 + self.rank)
            blk = torch.randn(batch, self.hkv, fill_len, hd, generator=g).to(self.dtype)
            for buf in (*self.k, *self.v):
                buf[:, :, :fill_len] = blk
        self.seq_len = fill_len

    # ------------------------------------------------------------------ model
    @torch.no_grad()
    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        """Local logits [B, T, V_local] of this rank (layer.py:91-124)."""
        cfg, hd = self.cfg, self.cfg.head_dim
        b, t = ids.shape
        start, end = self.seq_len, self.seq_len + t
        pos = torch.arange(start, end)
        cos, sin = self.cos[pos], self.sin[pos]
        # embedding.py:44-50
        if self.tp > 1:
            mask = (ids >= self.vstart) & (ids < self.vend)
            x = F.embedding((ids - self.vstart) * mask, self.embed) * mask.unsqueeze(-1).to(self.dtype)
            x = self._all_reduce(x)
        else:
            x = F.embedding(ids, self.embed)
        for li, w in enumerate(self.layers):
            h = rmsnorm(x, w["ln1"], cfg.rms_norm_eps)
            y = F.linear(h, w["qkv_w"], w["qkv_b"])
            q, k, v = torch.split(y, [self.hq * hd, self.hkv * hd, self.hkv * hd], dim=-1)
            q = q.reshape(b, t, self.hq, hd).transpose(1, 2)
            k = k.reshape(b, t, self.hkv, hd).transpose(1, 2)
            v = v.reshape(b, t, self.hkv, hd).transpose(1, 2)
            q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
            self.k[li][:, :, start:end] = k
            self.v[li][:, :, start:end] = v
            kk, vv = self.k[li][:, :, :end], self.v[li][:, :, :end]
            if self.hq != self.hkv:
                if self.hkv == 1:
                    kk = kk.expand(b, self.hq, end, hd)
                    vv = vv.expand(b, self.hq, end, hd)
                else:
                    kk = kk.repeat_interleave(self.hq // self.hkv, dim=1)
                    vv = vv.repeat_interleave(self.hq // self.hkv, dim=1)
            if t == 1:
                o = F.scaled_dot_product_attention(q, kk, vv)
            elif start == 0:
                o = F.scaled_dot_product_attention(q, kk, vv, is_causal=True)
            else:
                m = torch.ones(t, end, dtype=torch.bool).tril(diagonal=start)
                o = F.scaled_dot_product_attention(q, kk, vv, attn_mask=m)
            o = o.transpose(1, 2).reshape(b, t, self.hq * hd)
            x = x + self._all_reduce(F.linear(o, w["o_w"]))
            h = rmsnorm(x, w["ln2"], cfg.rms_norm_eps)
            gate, up = torch.chunk(F.linear(h, w["gu_w"]), 2, dim=-1)
            x = x + self._all_reduce(F.linear(F.silu(gate) * up, w["down_w"]))
        self.seq_len = end
        h = rmsnorm(x, self.norm, cfg.rms_norm_eps)
        return F.linear(h, self.lm_head)

    @staticmethod
    def _rope(x, cos, sin):
        """rope.py:53-64 (rotate_half in fp32, cast back)."""
        xf = x.float()
        x1, x2 = xf.chunk(2, dim=-1)
        return (xf * cos[None, None] + torch.cat([-x2, x1], dim=-1) * sin[None, None]).to(x.dtype)

    @torch.no_grad()
    def select(self, local_last: torch.Tensor) -> torch.Tensor:
        """Greedy ids [B] identical on every rank (embedding.py:118-172, bitpack)."""
        if self.tp == 1:
            return local_last.argmax(dim=-1)
        clean = torch.where(torch.isnan(local_last), torch.full_like(local_last, float("-inf")), local_last)
        values, idx = clean.max(dim=-1)
        gid = idx + self.vstart
        vals = torch.where(values == 0, torch.zeros_like(values), values)
        bits = vals.float().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        key = torch.where(bits < 0x80000000, bits, ((~bits) & 0xFFFFFFFF) - 0x80000000)
        packed = (key << 32) | (0xFFFFFFFF - gid.to(torch.int64))
        parts = [torch.empty_like(packed) for _ in range(self.tp)]
        dist.all_gather(parts, packed, group=self.group)  # collectives.py:185-214 (list form off NCCL)
        winner = torch.stack(parts, dim=-1).max(dim=-1).values
        return (0xFFFFFFFF - (winner & 0xFFFFFFFF)).to(torch.long)

    @torch.no_grad()
    def generate(self, ids: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
        """Fixed-length greedy decode (generation.py:133-171, early_stop=False)."""
        b, p = ids.shape
        self.reset(b, p + max_new_tokens)
        out = torch.empty(b, p + max_new_tokens, dtype=torch.long)
        out[:, :p] = ids
        logits = self.forward(ids)
        for step in range(max_new_tokens):
            tok = self.select(logits[:, -1])
            out[:, p + step] = tok
            if step + 1 < max_new_tokens:
                logits = self.forward(tok[:, None])
        return out


__all__ = ["OracleRank"]
