"""Load HF-named Qwen2 checkpoints onto per-rank shards (reference: minitp/weight_loader.py).

Same shard helpers (``shard_len``, ``kv_head_rows``, ``fused_qkv_local_sizes``),
the same packed layouts (``qkv_proj = [q; k; v]``, ``gate_up_proj = [gate; up]``)
and the same ``load_qwen2_tp`` signature. Each rank reads only its slices of a
safetensors checkpoint.

Additions:
* Q-head padding (``pad_heads=True``): when ``num_attention_heads`` does not
  divide by tp, the config is padded (``ModelConfig.padded_for``). Every
  inserted head gets zero q rows, zero q bias and zero o_proj columns, so the
  model's output is unchanged.
* ``load_synthetic_tp``: the seeded synthetic checkpoint of
  ``minitp_b200.synthetic``, drawn tensor by tensor without touching disk.
"""

from __future__ import annotations

import json
import os
from collections.abc import Iterator

import torch

from minitp_b200.config import ModelConfig
from minitp_b200.distributed.context import ParallelContext
from minitp_b200.layer import TPQwen2ForCausalLM


def shard_len(size: int, rank: int, tp: int) -> tuple[int, int]:
    """(start, length) of rank's contiguous chunk (reference weight_loader.py:40-44)."""
    base, rem = divmod(size, tp)
    start = rank * base + min(rank, rem)
    return start, base + (1 if rank < rem else 0)


def kv_head_rows(num_kv_heads: int, head_dim: int, rank: int, tp: int) -> tuple[int, int]:
    """(row_start, row_count) of this rank's KV-head block (weight_loader.py:52-58)."""
    if num_kv_heads % tp == 0:
        heads = num_kv_heads // tp
        return rank * heads * head_dim, heads * head_dim
    group = tp // num_kv_heads
    return (rank // group) * head_dim, head_dim


def fused_qkv_local_sizes(cfg: ModelConfig, tp: int) -> tuple[int, int]:
    """(q_rows, kv_rows) per rank of the fused QKV parameter (weight_loader.py:66-70)."""
    q_heads = cfg.num_attention_heads // tp
    kv_heads = max(1, cfg.num_key_value_heads // tp)
    return q_heads * cfg.head_dim, kv_heads * cfg.head_dim


def local_q_heads(cfg: ModelConfig, rank: int, tp: int) -> list[int]:
    """Checkpoint head index of each local (possibly padded) Q head; -1 = zero head."""
    hq = cfg.num_attention_heads // tp
    return cfg.padded_head_map()[rank * hq : (rank + 1) * hq]


# ---------------------------------------------------------------------- #
# tensor sources
# ---------------------------------------------------------------------- #
class SafetensorsSource:
    """Reads HF-named tensors (or slices) from ``model.safetensors`` or a sharded index."""

    def __init__(self, model_dir: str) -> None:
        from safetensors import safe_open

        self._open = safe_open
        self._handles: dict = {}
        index = os.path.join(model_dir, "model.safetensors.index.json")
        if os.path.exists(index):
            with open(index) as f:
                wm = json.load(f)["weight_map"]
            self._map = {k: os.path.join(model_dir, v) for k, v in wm.items()}
            self._single = None
        else:
            self._map = {}
            self._single = os.path.join(model_dir, "model.safetensors")

    def _h(self, name: str):
        path = self._map.get(name, self._single)
        if path is None:
            raise KeyError(f"tensor {name!r} not in checkpoint index")
        if path not in self._handles:
            self._handles[path] = self._open(path, framework="pt", device="cpu")
        return self._handles[path]

    def has(self, name: str) -> bool:
        if self._single is not None:
            return name in self._h(name).keys()
        return name in self._map

    def get(self, name: str) -> torch.Tensor:
        return self._h(name).get_tensor(name)

    def rows(self, name: str, start: int, length: int) -> torch.Tensor:
        sl = self._h(name).get_slice(name)
        if len(sl.get_shape()) == 1:
            return self.get(name).narrow(0, start, length)
        return sl[start : start + length]

    def cols(self, name: str, start: int, length: int) -> torch.Tensor:
        sl = self._h(name).get_slice(name)
        return sl[:, start : start + length]

    def close(self) -> None:
        self._handles.clear()


def _iter_layer_slices(cfg: ModelConfig, rank: int, tp: int, get) -> Iterator[tuple[str, torch.Tensor]]:
    """Yield (state_dict key, local tensor) of this rank, reading via ``get(name, kind, a, b)``.

    ``kind`` is "full", "rows" or "cols"; slices are [a, a + b).
    """
    hd, h = cfg.head_dim, cfg.hidden_size
    q_heads = local_q_heads(cfg, rank, tp)
    inter_start, inter_len = shard_len(cfg.intermediate_size, rank, tp)
    kv_start, kv_len = kv_head_rows(cfg.num_key_value_heads, hd, rank, tp)
    vs, vl = shard_len(cfg.vocab_size, rank, tp)
    yield "model.embed_tokens.weight", get("model.embed_tokens.weight", "rows", vs, vl)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        a, m = p + "self_attn.", p + "mlp."
        yield p + "input_layernorm.weight", get(p + "input_layernorm.weight", "full", 0, 0)
        kw = get(a + "k_proj.weight", "rows", kv_start, kv_len)
        vw = get(a + "v_proj.weight", "rows", kv_start, kv_len)
        kb = get(a + "k_proj.bias", "rows", kv_start, kv_len)
        vb = get(a + "v_proj.bias", "rows", kv_start, kv_len)
        # padded heads: zeros on the device and in the dtype of the source tensors
        zeros = lambda *shape: torch.zeros(*shape, dtype=kw.dtype, device=kw.device)  # noqa: E731
        qw, qb = [], []
        for head in q_heads:
            if head < 0:
                qw.append(zeros(hd, h))
                qb.append(zeros(hd))
            else:
                qw.append(get(a + "q_proj.weight", "rows", head * hd, hd))
                qb.append(get(a + "q_proj.bias", "rows", head * hd, hd))
        yield a + "qkv_proj.weight", torch.cat([*qw, kw, vw], dim=0)
        yield a + "qkv_proj.bias", torch.cat([*qb, kb, vb], dim=0)
        ocols = []
        for head in q_heads:
            ocols.append(zeros(h, hd) if head < 0 else get(a + "o_proj.weight", "cols", head * hd, hd))
        yield a + "o_proj.weight", torch.cat(ocols, dim=1)
        yield p + "post_attention_layernorm.weight", get(p + "post_attention_layernorm.weight", "full", 0, 0)
        gate = get(m + "gate_proj.weight", "rows", inter_start, inter_len)
        up = get(m + "up_proj.weight", "rows", inter_start, inter_len)
        yield m + "gate_up_proj.weight", torch.cat([gate, up], dim=0)
        yield m + "down_proj.weight", get(m + "down_proj.weight", "cols", inter_start, inter_len)
    yield "model.norm.weight", get("model.norm.weight", "full", 0, 0)
    if not cfg.tie_word_embeddings:
        yield "lm_head.weight", get("lm_head.weight", "rows", vs, vl)


def _prepare_cfg(cfg: ModelConfig, tp: int, pad_heads: bool) -> ModelConfig:
    if cfg.is_padded:
        cfg.validate(tp)
        return cfg
    if pad_heads and cfg.needs_padding(tp):
        return cfg.padded_for(tp)
    cfg.validate(tp)
    return cfg


def _materialise(cfg, ctx, dtype, device, items) -> TPQwen2ForCausalLM:
    model = TPQwen2ForCausalLM(cfg, ctx, init_weights=False).to(dtype=dtype, device=device)
    sd = model.state_dict()
    seen = set()
    for key, t in items:
        dst = sd[key]
        if tuple(dst.shape) != tuple(t.shape):
            raise ValueError(f"{key}: checkpoint slice {tuple(t.shape)} != parameter {tuple(dst.shape)}")
        dst.copy_(t.to(dtype))
        seen.add(key)
    missing = [k for k in sd if k not in seen and not (k == "lm_head.weight" and cfg.tie_word_embeddings)]
    if missing:
        raise ValueError(f"checkpoint did not provide: {missing[:5]}")
    return model.eval()


def load_qwen2_tp(
    model_dir: str,
    cfg: ModelConfig,
    ctx: ParallelContext,
    dtype: torch.dtype = torch.float32,
    device: torch.device | None = None,
    loader: str = "selective",
    pad_heads: bool = False,
) -> TPQwen2ForCausalLM:
    """Build the TP model and load only this rank's shards (reference weight_loader.py:172-269)."""
    if loader not in ("selective", "legacy", "direct_gpu"):
        raise ValueError(f"unknown loader {loader!r}")
    tp, rank = ctx.tp_size, ctx.tp_rank
    cfg = _prepare_cfg(cfg, tp, pad_heads)
    target = device if device is not None else ctx.device
    src = SafetensorsSource(model_dir)

    def get(name, kind, a, b):
        if kind == "full":
            return src.get(name).float()
        if kind == "rows":
            return src.rows(name, a, b).float()
        return src.cols(name, a, b).float()

    try:
        return _materialise(cfg, ctx, dtype, target, _iter_layer_slices(cfg, rank, tp, get))
    finally:
        src.close()


def load_synthetic_tp(
    cfg: ModelConfig,
    ctx: ParallelContext,
    dtype: torch.dtype = torch.bfloat16,
    device: torch.device | None = None,
    seed: int = 0,
    gen_device: str = "cpu",
    pad_heads: bool = True,
) -> TPQwen2ForCausalLM:
    """The seeded synthetic checkpoint of ``minitp_b200.synthetic``, sharded for this rank.

    Every rank draws the whole sequence (the generator must advance through
    all tensors) but keeps only its slices, one tensor alive at a time.
    """
    from minitp_b200.synthetic import iter_checkpoint

    tp, rank = ctx.tp_size, ctx.tp_rank
    cfg = _prepare_cfg(cfg, tp, pad_heads)
    target = device if device is not None else ctx.device
    model = TPQwen2ForCausalLM(cfg, ctx, init_weights=False).to(dtype=dtype, device=target)
    sd = model.state_dict()
    it = iter_checkpoint(cfg, seed, gen_device)
    cache: dict[str, torch.Tensor] = {}

    # Consume the draw stream in order; a tensor drawn before it is needed
    # waits in `cache` until its state_dict entry is assembled.
    def get(name, kind, a, b):
        while name not in cache:
            n, t = next(it)
            cache[n] = t
        t = cache[name]
        if kind == "full":
            return t
        if kind == "rows":
            return t.narrow(0, a, b)
        return t.narrow(1, a, b)

    seen = set()
    for key, t in _iter_layer_slices(cfg, rank, tp, get):
        dst = sd[key]
        if tuple(dst.shape) != tuple(t.shape):
            raise ValueError(f"{key}: slice {tuple(t.shape)} != parameter {tuple(dst.shape)}")
        dst.copy_(t.to(device=dst.device, dtype=dtype))
        seen.add(key)
        # every source tensor of the embedding / of a layer is consumed by the
        # time its last entry is copied: keep at most one layer alive
        if key.endswith("down_proj.weight") or key == "model.embed_tokens.weight":
            cache.clear()
    missing = [k for k in sd if k not in seen and not (k == "lm_head.weight" and cfg.tie_word_embeddings)]
    if missing:
        raise ValueError(f"synthetic checkpoint did not provide: {missing[:5]}")
    return model.eval()
