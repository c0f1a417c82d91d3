"""Qwen2 model configuration and tensor-parallel sharding math.

Mirrors ``minitp/config.py`` (reference): the same frozen dataclass fields,
``from_hf``, ``validate``, ``local_heads`` and ``kv_replication``, with the same
``ValueError`` messages (they contain "divisible"). One addition: Q-head
padding (``padded_for``), which the reference does not have. It makes layouts
such as 28 Q heads at tp=8 shardable without changing the result.
"""

from __future__ import annotations

from dataclasses import dataclass, replace


def _rope_theta(hf_config) -> float:
    theta = getattr(hf_config, "rope_theta", None)
    if theta is None:  # transformers >= 5 keeps it in rope_parameters
        theta = hf_config.rope_parameters["rope_theta"]
    return float(theta)


@dataclass(frozen=True)
class ModelConfig:
    """Field-for-field the reference ``ModelConfig`` (minitp/config.py:17-29).

    ``orig_num_attention_heads`` is set only on padded configs: it is the Q head
    count of the checkpoint before zero heads were inserted (0 = not padded).
    """

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
    tie_word_embeddings: bool = True
    orig_num_attention_heads: int = 0

    @classmethod
    def from_hf(cls, hf_config, tp_size: int = 1) -> ModelConfig:
        """minitp/config.py:31-48."""
        cfg = cls(
            hidden_size=hf_config.hidden_size,
            intermediate_size=hf_config.intermediate_size,
            num_hidden_layers=hf_config.num_hidden_layers,
            num_attention_heads=hf_config.num_attention_heads,
            num_key_value_heads=hf_config.num_key_value_heads,
            head_dim=getattr(hf_config, "head_dim", None)
            or hf_config.hidden_size // hf_config.num_attention_heads,
            vocab_size=hf_config.vocab_size,
            rms_norm_eps=hf_config.rms_norm_eps,
            rope_theta=_rope_theta(hf_config),
            max_position_embeddings=hf_config.max_position_embeddings,
            tie_word_embeddings=getattr(hf_config, "tie_word_embeddings", True),
        )
        cfg.validate(tp_size)
        return cfg

    # ------------------------------------------------------------------ #
    # TP validation (minitp/config.py:50-68)
    # ------------------------------------------------------------------ #
    def validate(self, tp_size: int) -> None:
        checks = {
            "hidden_size": self.hidden_size,
            "num_attention_heads": self.num_attention_heads,
            "intermediate_size": self.intermediate_size,
        }
        for name, value in checks.items():
            if value % tp_size != 0:
                raise ValueError(
                    f"{name}={value} not divisible by tp_size={tp_size}; "
                    "tensor-parallel sharding would be incorrect"
                )
        if self.num_key_value_heads % tp_size != 0 and tp_size % self.num_key_value_heads != 0:
            raise ValueError(
                f"num_key_value_heads={self.num_key_value_heads} incompatible with "
                f"tp_size={tp_size}: need kv%tp==0 (shard) or tp%kv==0 (replicate)"
            )

    def local_heads(self, tp_size: int) -> tuple[int, int]:
        """(q_heads_per_rank, kv_heads_per_rank); minitp/config.py:70-72."""
        return self.num_attention_heads // tp_size, max(1, self.num_key_value_heads // tp_size)

    def kv_replication(self, tp_size: int) -> int:
        """Ranks sharing each KV head; minitp/config.py:74-78."""
        if self.num_key_value_heads % tp_size == 0:
            return 1
        return tp_size // self.num_key_value_heads

    # ------------------------------------------------------------------ #
    # Q-head padding (no counterpart in the reference)
    # ------------------------------------------------------------------ #
    @property
    def is_padded(self) -> bool:
        return self.orig_num_attention_heads > 0

    @property
    def checkpoint_q_heads(self) -> int:
        """Q heads stored in the checkpoint (before any padding)."""
        return self.orig_num_attention_heads or self.num_attention_heads

    def needs_padding(self, tp_size: int) -> bool:
        try:
            self.validate(tp_size)
            return False
        except ValueError:
            return True

    def padded_for(self, tp_size: int) -> ModelConfig:
        """Return a config whose Q heads are padded so ``tp_size`` can shard it.

        Each GQA group of ``g = q/kv`` query heads is padded to ``g'`` heads, the
        smallest multiple of the number of ranks that share one KV head. The
        inserted heads get zero q rows, zero q bias and zero o_proj columns, so
        they contribute exactly 0 to the o_proj output: the model's result is
        unchanged. Example: 28 q / 4 kv at tp=8 gives g=7 -> g'=8, 32 heads,
        4 per rank, every KV head replicated on 2 ranks.

        ``hidden_size`` and ``intermediate_size`` are not padded; they must
        still divide by ``tp_size``.
        """
        q, kv = self.checkpoint_q_heads, self.num_key_value_heads
        if q % kv != 0:
            raise ValueError(f"num_attention_heads={q} not divisible by num_key_value_heads={kv}")
        base = replace(self, num_attention_heads=q, orig_num_attention_heads=0)
        if not base.needs_padding(tp_size):
            return base
        if kv % tp_size != 0 and tp_size % kv != 0:
            raise ValueError(
                f"num_key_value_heads={kv} incompatible with tp_size={tp_size}: "
                "need kv%tp==0 (shard) or tp%kv==0 (replicate)"
            )
        g = q // kv
        share = tp_size // kv if tp_size % kv == 0 else 1  # ranks per KV head
        if kv % tp_size == 0:
            # KV heads shard evenly; q_local = g * kv/tp is already integral
            g_pad = g
        else:
            g_pad = -(-g // share) * share
        cfg = replace(self, num_attention_heads=g_pad * kv, orig_num_attention_heads=q)
        cfg.validate(tp_size)
        return cfg

    def padded_head_map(self) -> list[int]:
        """For each padded Q head, the checkpoint head it holds (-1 = zero head)."""
        if not self.is_padded:
            return list(range(self.num_attention_heads))
        kv = self.num_key_value_heads
        g, g_pad = self.orig_num_attention_heads // kv, self.num_attention_heads // kv
        out = []
        for grp in range(kv):
            for j in range(g_pad):
                out.append(grp * g + j if j < g else -1)
        return out


def tiny_config(tp_size: int = 1) -> ModelConfig:
    """Tiny random Qwen2-ish config for fast layer-level tests (minitp/config.py:81-97)."""
    cfg = ModelConfig(
        hidden_size=64,
        intermediate_size=128,
        num_hidden_layers=2,
        num_attention_heads=4,
        num_key_value_heads=2,
        head_dim=16,
        vocab_size=128,
        rms_norm_eps=1e-6,
        rope_theta=10000.0,
        max_position_embeddings=256,
        tie_word_embeddings=False,
    )
    cfg.validate(tp_size)
    return cfg


# ---------------------------------------------------------------------- #
# The workload configurations the benchmarks and parity tests run.
# ---------------------------------------------------------------------- #
def baseline_tiny() -> ModelConfig:
    """Tiny Qwen2: 2 layers, H64, I128, 4q/2kv, hd16, V1000, theta 1e6, tied."""
    return ModelConfig(
        hidden_size=64, intermediate_size=128, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=16,
        vocab_size=1000, rms_norm_eps=1e-6, rope_theta=1e6,
        max_position_embeddings=4096, tie_word_embeddings=True,
    )


def qwen25_05b(num_layers: int = 24) -> ModelConfig:
    """Qwen2.5-0.5B shape: H896, I4864, 14q/2kv, hd64, V151936, tied."""
    return ModelConfig(
        hidden_size=896, intermediate_size=4864, num_hidden_layers=num_layers,
        num_attention_heads=14, num_key_value_heads=2, head_dim=64,
        vocab_size=151936, rms_norm_eps=1e-6, rope_theta=1e6,
        max_position_embeddings=32768, tie_word_embeddings=True,
    )


def qwen25_7b(num_layers: int = 28) -> ModelConfig:
    """Qwen2.5-7B shape: H3584, I18944, 28q/4kv, hd128, V152064, untied."""
    return ModelConfig(
        hidden_size=3584, intermediate_size=18944, num_hidden_layers=num_layers,
        num_attention_heads=28, num_key_value_heads=4, head_dim=128,
        vocab_size=152064, rms_norm_eps=1e-6, rope_theta=1e6,
        max_position_embeddings=32768, tie_word_embeddings=False,
    )


CONFIGS = {
    "tiny": baseline_tiny,
    "qwen2.5-0.5b": qwen25_05b,
    "qwen2.5-7b": qwen25_7b,
}
