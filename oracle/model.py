"""CPU restatement of the reference TP Qwen2 decode path (torch on CPU).

Follows minitp v0.4 operation by operation, with the same rounding points in
the model dtype (fp32 or bf16). TP is emulated: rank r holds the reference's
shards (minitp/weight_loader.py:154-269) and every RowParallel / vocab
AllReduce is a rank-ordered sum of the per-rank partials
(minitp/parallel/linear.py:111-122, embedding.py:44-50).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from oracle.argmax import distributed_argmax, shard_range


@dataclass(frozen=True)
class OracleConfig:
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    vocab_size: int
    rms_norm_eps: float
    rope_theta: float
    max_position_embeddings: int
    tie_word_embeddings: bool

    @classmethod
    def of(cls, cfg) -> OracleConfig:
        return cls(**{k: getattr(cfg, k) for k in cls.__dataclass_fields__})


def kv_head_rows(num_kv_heads: int, head_dim: int, rank: int, tp: int) -> tuple[int, int]:
    """minitp/weight_loader.py:52-58."""
    if num_kv_heads % tp == 0:
        heads = num_kv_heads // tp
        return rank * heads * head_dim, heads * head_dim
    group = tp // num_kv_heads
    return (rank // group) * head_dim, head_dim


# ---------------------------------------------------------------------- #
# primitives
# ---------------------------------------------------------------------- #
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """minitp/layer.py:36-42."""
    dtype = x.dtype
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * w.float()).to(dtype)


def rope_tables(head_dim: int, theta: float, max_seq_len: int) -> tuple[torch.Tensor, torch.Tensor]:
    """minitp/rope.py:27-34."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    pos = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, H, T, hd]; cos/sin [T, hd]: minitp/rope.py:53-64 (rotate_half, fp32 math)."""
    xf = x.float()
    x1, x2 = xf.chunk(2, dim=-1)
    rot = torch.cat([-x2, x1], dim=-1)
    return (xf * cos[None, None] + rot * sin[None, None]).to(x.dtype)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cache_len: int) -> torch.Tensor:
    """GQA attention, q [B, hq, T, hd], k/v [B, hkv, L, hd] (minitp/attention.py:71-103).

    Query t (absolute slot cache_len + t) attends keys [0, cache_len + t];
    softmax(q k^T / sqrt(hd)) v in fp32, output cast to the model dtype.
    """
    b, hq, t, hd = q.shape
    hkv = k.shape[1]
    group = hq // hkv
    kf = k.float().repeat_interleave(group, dim=1)
    vf = v.float().repeat_interleave(group, dim=1)
    s = torch.matmul(q.float(), kf.transpose(-1, -2)) / math.sqrt(hd)
    L = k.shape[2]
    mask = torch.ones(t, L, dtype=torch.bool).tril(diagonal=cache_len)
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, vf).to(q.dtype)


def rank_sum(parts: list[torch.Tensor]) -> torch.Tensor:
    """AllReduce SUM of per-rank tensors in rank order (minitp/distributed/collectives.py:147-157).

    Partials are accumulated in fp32 and rounded once to the model dtype,
    which is what a two-rank bf16 reduction does.
    """
    acc = parts[0].float()
    for p in parts[1:]:
        acc = acc + p.float()
    return acc.to(parts[0].dtype)


def embedding(ids: torch.Tensor, table_shards: list[torch.Tensor], vocab: int) -> torch.Tensor:
    """Masked local lookups summed over ranks (minitp/parallel/embedding.py:44-50)."""
    tp = len(table_shards)
    if tp == 1:
        return F.embedding(ids, table_shards[0])
    parts = []
    for r, tab in enumerate(table_shards):
        s, e = shard_range(vocab, r, tp)
        mask = (ids >= s) & (ids < e)
        local = (ids - s).clamp(min=0) * mask
        parts.append(F.embedding(local, tab) * mask.unsqueeze(-1).to(tab.dtype))
    return rank_sum(parts)


def allreduce_residual_rmsnorm(partials, residual, gain, eps):
    """RowParallel reduce + residual add + RMSNorm (linear.py:111-122, layer.py:64, layer.py:36-42)."""
    x = residual + rank_sum(list(partials))
    return x, rmsnorm(x, gain, eps)


# ---------------------------------------------------------------------- #
# model
# ---------------------------------------------------------------------- #
class OracleModel:
    """The reference TP model with ``tp`` emulated ranks, built from HF-named fp32 tensors."""

    def __init__(self, cfg: OracleConfig, tensors: dict[str, torch.Tensor], tp: int = 1,
                 dtype: torch.dtype = torch.float32) -> None:
        if cfg.num_attention_heads % tp or cfg.hidden_size % tp or cfg.intermediate_size % tp:
            raise ValueError("oracle: config not divisible by tp (the reference rejects it)")
        self.cfg, self.tp, self.dtype = cfg, tp, dtype
        hd = cfg.head_dim
        self.hq = cfg.num_attention_heads // tp
        self.hkv = max(1, cfg.num_key_value_heads // tp)
        cast = lambda t: t.to(dtype).contiguous()  # noqa: E731
        V = cfg.vocab_size
        self.embed = [cast(tensors["model.embed_tokens.weight"][slice(*shard_range(V, r, tp))]) for r in range(tp)]
        head = tensors["model.embed_tokens.weight"] if cfg.tie_word_embeddings else tensors["lm_head.weight"]
        self.lm_head = [cast(head[slice(*shard_range(V, r, tp))]) for r in range(tp)]
        self.norm = cast(tensors["model.norm.weight"])
        self.layers = []
        I = cfg.intermediate_size
        for i in range(cfg.num_hidden_layers):
            p = f"model.layers.{i}."
            ranks = []
            for r in range(tp):
                q0, q1 = shard_range(cfg.num_attention_heads * hd, r, tp)
                k0, kn = kv_head_rows(cfg.num_key_value_heads, hd, r, tp)
                i0, i1 = shard_range(I, r, tp)
                qkv_w = torch.cat([tensors[p + "self_attn.q_proj.weight"][q0:q1],
                                   tensors[p + "self_attn.k_proj.weight"][k0:k0 + kn],
                                   tensors[p + "self_attn.v_proj.weight"][k0:k0 + kn]])
                qkv_b = torch.cat([tensors[p + "self_attn.q_proj.bias"][q0:q1],
                                   tensors[p + "self_attn.k_proj.bias"][k0:k0 + kn],
                                   tensors[p + "self_attn.v_proj.bias"][k0:k0 + kn]])
                gate_up = torch.cat([tensors[p + "mlp.gate_proj.weight"][i0:i1],
                                     tensors[p + "mlp.up_proj.weight"][i0:i1]])
                ranks.append(dict(
                    qkv_w=cast(qkv_w), qkv_b=cast(qkv_b),
                    o_w=cast(tensors[p + "self_attn.o_proj.weight"][:, q0:q1]),
                    gu_w=cast(gate_up), down_w=cast(tensors[p + "mlp.down_proj.weight"][:, i0:i1]),
                ))
            self.layers.append(dict(ln1=cast(tensors[p + "input_layernorm.weight"]),
                                    ln2=cast(tensors[p + "post_attention_layernorm.weight"]), ranks=ranks))
        self.cos, self.sin = rope_tables(hd, cfg.rope_theta, cfg.max_position_embeddings)
        self.k = self.v = None
        self.seq_len = 0

    def reset(self, batch: int, max_seq: int) -> None:
        """Fresh per-rank KV caches [B, hkv, max_seq, hd] (minitp/kv_cache.py:18-41)."""
        L, hd = self.cfg.num_hidden_layers, self.cfg.head_dim
        z = lambda: torch.zeros(batch, self.hkv, max_seq, hd, dtype=self.dtype)  # noqa: E731
        self.k = [[z() for _ in range(self.tp)] for _ in range(L)]
        self.v = [[z() for _ in range(self.tp)] for _ in range(L)]
        self.seq_len = 0

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, positions: torch.Tensor | None = None) -> torch.Tensor:
        """Full-vocab logits ``[B, T, V]`` (fp32 view of the dtype result); layer.py:91-124."""
        cfg, tp, hd = self.cfg, self.tp, self.cfg.head_dim
        b, t = ids.shape
        start = self.seq_len
        if positions is None:
            positions = torch.arange(start, start + t)
        cos, sin = self.cos[positions], self.sin[positions]
        x = embedding(ids, self.embed, cfg.vocab_size)
        end = start + t
        for li, layer in enumerate(self.layers):
            h = rmsnorm(x, layer["ln1"], cfg.rms_norm_eps)
            parts = []
            for r, w in enumerate(layer["ranks"]):
                y = F.linear(h, w["qkv_w"], w["qkv_b"])  # fused.py:57-61
                q, k, v = torch.split(y, [self.hq * hd, self.hkv * hd, self.hkv * hd], dim=-1)
                q = q.reshape(b, t, self.hq, hd).transpose(1, 2)
                k = k.reshape(b, t, self.hkv, hd).transpose(1, 2)
                v = v.reshape(b, t, self.hkv, hd).transpose(1, 2)
                q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
                self.k[li][r][:, :, start:end] = k  # kv_cache.py:53-55
                self.v[li][r][:, :, start:end] = v
                o = attention(q, self.k[li][r][:, :, :end], self.v[li][r][:, :, :end], start)
                o = o.transpose(1, 2).reshape(b, t, self.hq * hd)
                parts.append(F.linear(o, w["o_w"]))  # linear.py:117
            x = x + rank_sum(parts)  # layer.py:64
            h = rmsnorm(x, layer["ln2"], cfg.rms_norm_eps)
            parts = []
            for w in layer["ranks"]:
                gate, up = torch.chunk(F.linear(h, w["gu_w"]), 2, dim=-1)  # fused.py:102-104
                parts.append(F.linear(F.silu(gate) * up, w["down_w"]))  # mlp.py:38
            x = x + rank_sum(parts)  # layer.py:65
        self.seq_len = end  # layer.py:115-116
        h = rmsnorm(x, self.norm, cfg.rms_norm_eps)
        return torch.cat([F.linear(h, w) for w in self.lm_head], dim=-1).float()  # embedding.py:87-90

    def select(self, logits_last: torch.Tensor) -> torch.Tensor:
        """Greedy ids of the last position (minitp/generation.py:54-59)."""
        return torch.from_numpy(distributed_argmax(logits_last.numpy(), self.tp))

    @torch.no_grad()
    def generate(self, ids: torch.Tensor, max_new_tokens: int, keep_logits: bool = False):
        """Fixed-length greedy decode (generation.py:133-171 with early_stop=False)."""
        b, p = ids.shape
        self.reset(b, p + max_new_tokens)
        out = torch.empty(b, p + max_new_tokens, dtype=torch.long)
        out[:, :p] = ids
        logits = self.forward(ids, torch.arange(p))
        kept = []
        for step in range(max_new_tokens):
            last = logits[:, -1]
            if keep_logits:
                kept.append(last.clone())
            tok = self.select(last)
            out[:, p + step] = tok
            if step + 1 < max_new_tokens:
                logits = self.forward(tok[:, None], torch.tensor([p + step]))
        return (out, kept) if keep_logits else out


def checkpoint_tensors(cfg, seed: int = 0) -> dict[str, torch.Tensor]:
    """The seeded synthetic checkpoint: one generator, draw order of the HF names.

    Restated from the protocol used by the parity fixtures: embed; per layer
    q/k/v weight+bias, o, gate, up, down (~N(0, 0.02)); norms are ones;
    untied lm_head last.
    """
    g = torch.Generator()
    g.manual_seed(seed)
    h, inter, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    q, kv = cfg.num_attention_heads * hd, cfg.num_key_value_heads * hd
    out: dict[str, torch.Tensor] = {}

    def draw(name, shape):
        out[name] = torch.randn(shape, generator=g) * 0.02

    draw("model.embed_tokens.weight", (cfg.vocab_size, h))
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        out[p + "input_layernorm.weight"] = torch.ones(h)
        draw(p + "self_attn.q_proj.weight", (q, h))
        draw(p + "self_attn.q_proj.bias", (q,))
        draw(p + "self_attn.k_proj.weight", (kv, h))
        draw(p + "self_attn.k_proj.bias", (kv,))
        draw(p + "self_attn.v_proj.weight", (kv, h))
        draw(p + "self_attn.v_proj.bias", (kv,))
        draw(p + "self_attn.o_proj.weight", (h, q))
        out[p + "post_attention_layernorm.weight"] = torch.ones(h)
        draw(p + "mlp.gate_proj.weight", (inter, h))
        draw(p + "mlp.up_proj.weight", (inter, h))
        draw(p + "mlp.down_proj.weight", (h, inter))
    out["model.norm.weight"] = torch.ones(h)
    if not cfg.tie_word_embeddings:
        draw("lm_head.weight", (cfg.vocab_size, h))
    return out


def prompt(vocab: int, batch: int, length: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator()
    g.manual_seed(seed)
    return torch.randint(0, vocab, (batch, length), generator=g)


__all__ = ["OracleConfig", "OracleModel", "allreduce_residual_rmsnorm", "apply_rope", "attention",
           "checkpoint_tensors", "embedding", "prompt", "rank_sum", "rmsnorm", "rope_tables"]
