"""Seeded synthetic Qwen2 checkpoints and prompts.

No real checkpoint is reachable from the GPU boxes, so every benchmark and
parity run uses random weights drawn by one fixed protocol, which the oracle
and the parity fixtures share:

* One ``torch.Generator`` seeded with ``seed`` draws every weight and bias in
  checkpoint order: ``model.embed_tokens.weight``; then per layer
  ``q_proj.{weight,bias}``, ``k_proj.{weight,bias}``, ``v_proj.{weight,bias}``,
  ``o_proj.weight``, ``gate_proj.weight``, ``up_proj.weight``,
  ``down_proj.weight``; then ``lm_head.weight`` when the head is untied.
* Each tensor is ``randn(shape, generator=g) * 0.02`` in fp32.
* RMSNorm gains (``input_layernorm``, ``post_attention_layernorm``,
  ``model.norm``) are ones and draw nothing.
* Prompt ids are ``randint(0, vocab, (B, P))`` from a fresh generator seeded
  with ``seed``.

``device="cuda"`` draws from a CUDA generator instead. It is much faster for the
7B shape, but its numbers differ from the CPU protocol. Use it only for
benchmarks; parity runs use the CPU protocol.
"""

from __future__ import annotations

from collections.abc import Iterator

import torch

from minitp_b200.config import ModelConfig


def checkpoint_order(cfg: ModelConfig) -> list[tuple[str, tuple[int, ...], str]]:
    """``(name, shape, kind)`` in draw order; kind is "randn" or "ones"."""
    h, inter = cfg.hidden_size, cfg.intermediate_size
    q = cfg.checkpoint_q_heads * cfg.head_dim
    kv = cfg.num_key_value_heads * cfg.head_dim
    out: list[tuple[str, tuple[int, ...], str]] = [
        ("model.embed_tokens.weight", (cfg.vocab_size, h), "randn")
    ]
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        out += [
            (p + "input_layernorm.weight", (h,), "ones"),
            (p + "self_attn.q_proj.weight", (q, h), "randn"),
            (p + "self_attn.q_proj.bias", (q,), "randn"),
            (p + "self_attn.k_proj.weight", (kv, h), "randn"),
            (p + "self_attn.k_proj.bias", (kv,), "randn"),
            (p + "self_attn.v_proj.weight", (kv, h), "randn"),
            (p + "self_attn.v_proj.bias", (kv,), "randn"),
            (p + "self_attn.o_proj.weight", (h, q), "randn"),
            (p + "post_attention_layernorm.weight", (h,), "ones"),
            (p + "mlp.gate_proj.weight", (inter, h), "randn"),
            (p + "mlp.up_proj.weight", (inter, h), "randn"),
            (p + "mlp.down_proj.weight", (h, inter), "randn"),
        ]
    out.append(("model.norm.weight", (h,), "ones"))
    if not cfg.tie_word_embeddings:
        out.append(("lm_head.weight", (cfg.vocab_size, h), "randn"))
    return out


def iter_checkpoint(
    cfg: ModelConfig, seed: int = 0, device: str | torch.device = "cpu", std: float = 0.02
) -> Iterator[tuple[str, torch.Tensor]]:
    """Yield ``(hf_name, fp32 tensor)`` in draw order (one tensor alive at a time)."""
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    for name, shape, kind in checkpoint_order(cfg):
        if kind == "ones":
            yield name, torch.ones(shape, dtype=torch.float32, device=device)
        else:
            t = torch.randn(shape, generator=g, dtype=torch.float32, device=device)
            t.mul_(std)
            yield name, t


def make_checkpoint(cfg: ModelConfig, seed: int = 0, device="cpu") -> dict[str, torch.Tensor]:
    """The whole checkpoint as a dict (small configs only)."""
    return dict(iter_checkpoint(cfg, seed, device))


def make_prompt(vocab_size: int, batch: int, prompt_len: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator()
    g.manual_seed(seed)
    return torch.randint(0, vocab_size, (batch, prompt_len), generator=g)


def save_checkpoint(cfg: ModelConfig, model_dir: str, seed: int = 0) -> None:
    """Write the synthetic checkpoint as ``model.safetensors`` (HF names)."""
    import os

    from safetensors.torch import save_file

    os.makedirs(model_dir, exist_ok=True)
    save_file(make_checkpoint(cfg, seed), os.path.join(model_dir, "model.safetensors"))
