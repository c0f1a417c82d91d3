"""Rotary position embedding tables (HF Qwen2 rotate_half convention).

Reference: minitp/rope.py:17-88. The fp32 ``[max_seq_len, head_dim]`` cos/sin
tables follow the reference's formula exactly:
``inv_freq = 1 / theta**(arange(0, hd, 2)/hd)``, ``freqs = pos * inv_freq``,
``emb = cat(freqs, freqs)``. They are computed on the CPU and copied to the
device, so the GPU kernels see the same bits as a CPU run of the reference.
The rotation itself runs inside the fused QKV kernel (``ops.qkv_rope``).
"""

from __future__ import annotations

import torch


def rope_tables(head_dim: int, theta: float, max_seq_len: int) -> tuple[torch.Tensor, torch.Tensor]:
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    pos = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


class RotaryEmbedding:
    """Precomputed rotary tables for absolute positions [0, max_seq_len)."""

    def __init__(self, head_dim: int, theta: float, max_seq_len: int, device: torch.device | None = None) -> None:
        cos, sin = rope_tables(head_dim, theta, max_seq_len)
        self.cos_cache = cos.to(device) if device is not None else cos
        self.sin_cache = sin.to(device) if device is not None else sin
        self.max_seq_len = max_seq_len
        self.head_dim = head_dim

    def cos_sin(self, positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Rows of the tables for ``positions`` (IndexError when out of range on CPU)."""
        return self.cos_cache[positions], self.sin_cache[positions]
