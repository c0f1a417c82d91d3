"""Per-rank contiguous KV cache (reference: minitp/kv_cache.py:8-63).

Layout per layer: ``k[l]``, ``v[l]`` = ``[batch, kv_heads_local, max_seq_len, head_dim]``
in the model dtype. ``seq_len`` is the host fill cursor; the kernels write
K/V in place at slots ``[seq_len, seq_len + T)`` and read ``[0, seq_len + T)``,
so unwritten slots are never read (``init="empty"`` is safe).
"""

from __future__ import annotations

import ctypes

import torch


class KVCache:
    def __init__(
        self,
        num_layers: int,
        batch_size: int,
        kv_heads_local: int,
        head_dim: int,
        max_seq_len: int,
        dtype: torch.dtype,
        device: torch.device,
        init: str = "empty",
    ) -> None:
        if init not in ("empty", "zeros"):
            raise ValueError(f"init must be 'empty' or 'zeros', got {init!r}")
        self.max_seq_len = max_seq_len
        self.seq_len = 0
        alloc = torch.empty if init == "empty" else torch.zeros
        self.k = [alloc(batch_size, kv_heads_local, max_seq_len, head_dim, dtype=dtype, device=device)
                  for _ in range(num_layers)]
        self.v = [alloc(batch_size, kv_heads_local, max_seq_len, head_dim, dtype=dtype, device=device)
                  for _ in range(num_layers)]
        self._ptrs = None

    def check_room(self, t: int) -> None:
        """Raise the reference's overflow error before writing ``t`` tokens."""
        end = self.seq_len + t
        if end > self.max_seq_len:
            raise ValueError(f"KV cache overflow: seq {self.seq_len}+{t} > max_seq_len={self.max_seq_len}")

    def update(self, layer_idx: int, k_new: torch.Tensor, v_new: torch.Tensor):
        """Append ``[B, H, T, D]`` at the cursor; returns the valid views (reference API)."""
        t = k_new.shape[2]
        self.check_room(t)
        end = self.seq_len + t
        self.k[layer_idx][:, :, self.seq_len:end] = k_new
        self.v[layer_idx][:, :, self.seq_len:end] = v_new
        return self.k[layer_idx][:, :, :end], self.v[layer_idx][:, :, :end]

    def advance(self, tokens: int) -> None:
        self.seq_len += tokens

    def poison(self, value: float = float("nan")) -> None:
        for buf in (*self.k, *self.v):
            buf.fill_(value)

    def pointer_arrays(self):
        """Host arrays of the per-layer K and V device pointers (for the C ABI)."""
        key = tuple(t.data_ptr() for t in (*self.k, *self.v))
        if self._ptrs is None or self._ptrs[0] != key:
            n = len(self.k)
            ka = (ctypes.c_void_p * n)(*[t.data_ptr() for t in self.k])
            va = (ctypes.c_void_p * n)(*[t.data_ptr() for t in self.v])
            self._ptrs = (key, ka, va)
        return self._ptrs[1], self._ptrs[2]
