"""Tensor-level wrappers of the C ABI (include/minitp_b200.h).

Each function validates device, dtype and layout, allocates its outputs with
torch (device memory plumbing) and enqueues the kernel on the current CUDA
stream. None of them has a CPU path: CPU tensors raise.
"""

from __future__ import annotations

import torch

from minitp_b200 import _lib


def _c(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


def _comm_handle(comm) -> int | None:
    return None if comm is None else comm.handle


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear(x, w, bias)`` on the weight-streaming GEMV (fp32 accumulate)."""
    _lib.require_cuda(x, w, bias)
    if x.dtype != w.dtype or (bias is not None and bias.dtype != w.dtype):
        raise _lib.MinitpB200Error(f"linear: dtype mismatch ({x.dtype}, {w.dtype})")
    n, k = w.shape
    if x.shape[-1] != k:
        raise _lib.MinitpB200Error(f"linear: x has {x.shape[-1]} features, weight expects {k}")
    x2 = _c(x).reshape(-1, k)
    m = x2.shape[0]
    y = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    if m == 0:
        return y
    w = _c(w)
    _lib.call("mtpb_linear", x2.data_ptr(), k, w.data_ptr(), _lib.ptr(None if bias is None else _c(bias)),
              y.data_ptr(), n, m, n, k, _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device))
    return y


def linear_swiglu(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` with ``gate, up = F.linear(x, w).chunk(2, -1)``."""
    _lib.require_cuda(x, w)
    n2, k = w.shape
    inter = n2 // 2
    x2 = _c(x).reshape(-1, k)
    m = x2.shape[0]
    y = torch.empty(*x.shape[:-1], inter, dtype=x.dtype, device=x.device)
    if m == 0:
        return y
    _lib.call("mtpb_linear_swiglu", x2.data_ptr(), k, _c(w).data_ptr(), y.data_ptr(), inter, m, inter, k,
              _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device))
    return y


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    _lib.require_cuda(x, w)
    h = x.shape[-1]
    x2 = _c(x).reshape(-1, h)
    y = torch.empty_like(x2)
    if x2.shape[0]:
        _lib.call("mtpb_rmsnorm", x2.data_ptr(), _c(w).data_ptr(), y.data_ptr(), x2.shape[0], h, float(eps),
                  _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device))
    return y.view(x.shape)


def allreduce_(t: torch.Tensor, comm) -> torch.Tensor:
    """In-place SUM over the communicator's ranks (one-shot NVLink push)."""
    _lib.require_cuda(t)
    if not t.is_contiguous():
        raise _lib.MinitpB200Error("allreduce_: tensor must be contiguous")
    h = t.shape[-1]
    _lib.call("mtpb_allreduce", _comm_handle(comm), t.data_ptr(), t.numel() // h, h, _lib.dtype_code(t.dtype),
              _lib.stream_ptr(t.device))
    return t


def allreduce_residual_rmsnorm(
    partial: torch.Tensor,
    residual: torch.Tensor | None,
    gain: torch.Tensor | None,
    eps: float,
    comm,
    bias: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """(residual + T(sum_r partial_r) [+ bias], RMSNorm of that) in one kernel."""
    _lib.require_cuda(partial, residual, gain, bias)
    h = partial.shape[-1]
    p = _c(partial)
    rows = p.numel() // h
    out_res = torch.empty_like(p)
    out_norm = torch.empty_like(p) if gain is not None else None
    if rows:
        _lib.call(
            "mtpb_allreduce_residual_rmsnorm", _comm_handle(comm), p.data_ptr(),
            _lib.ptr(None if residual is None else _c(residual)), _lib.ptr(None if gain is None else _c(gain)),
            _lib.ptr(None if bias is None else _c(bias)), out_res.data_ptr(), _lib.ptr(out_norm),
            rows, h, float(eps), _lib.dtype_code(p.dtype), _lib.stream_ptr(p.device),
        )
    return out_res, out_norm


def embedding(ids: torch.Tensor, table: torch.Tensor, vstart: int, vend: int, vocab: int, comm) -> torch.Tensor:
    """Masked local lookup of ``ids`` in the shard [vstart, vend), summed over ranks."""
    _lib.require_cuda(ids, table)
    ids2 = _c(ids.to(torch.int64)).reshape(-1)
    h = table.shape[1]
    out = torch.empty(*ids.shape, h, dtype=table.dtype, device=table.device)
    if ids2.numel():
        _lib.call("mtpb_embedding", _comm_handle(comm), ids2.data_ptr(), _c(table).data_ptr(), out.data_ptr(),
                  ids2.numel(), h, vstart, vend, vocab, _lib.dtype_code(table.dtype), _lib.stream_ptr(table.device))
    return out


def argmax(local_logits: torch.Tensor, vstart: int, comm) -> torch.Tensor:
    """Greedy ids over vocab-sharded logits ``[..., V_local]`` -> ``[..., 1]`` int64."""
    _lib.require_cuda(local_logits)
    v = local_logits.shape[-1]
    x = local_logits.reshape(-1, v)
    if x.stride(-1) != 1:
        x = x.contiguous()
    m = x.shape[0]
    out = torch.empty(m, dtype=torch.int64, device=x.device)
    scratch = torch.empty(64 * 64, dtype=torch.int64, device=x.device)
    for s in range(0, m, 64):
        n = min(64, m - s)
        _lib.call("mtpb_argmax", _comm_handle(comm), x[s].data_ptr(), n, v, x.stride(0), vstart,
                  out[s].data_ptr(), scratch.data_ptr(), _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device))
    return out.view(*local_logits.shape[:-1], 1)


def qkv_rope(
    x: torch.Tensor,  # [B, T, H]
    w: torch.Tensor,
    bias: torch.Tensor | None,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    hq: int,
    hkv: int,
    cache_len: int,
    rope_pos: torch.Tensor | None,
    cos: torch.Tensor,
    sin: torch.Tensor,
    comm=None,
) -> torch.Tensor:
    """Fused QKV GEMV + bias + RoPE; writes K/V at slots [cache_len, cache_len + T)."""
    _lib.require_cuda(x, w, k_cache, v_cache)
    b, t, h = x.shape
    hd = k_cache.shape[-1]
    cap = k_cache.shape[2]
    q = torch.empty(b, t, hq * hd, dtype=x.dtype, device=x.device)
    xc = _c(x)
    rp = None if rope_pos is None else _c(rope_pos.to(torch.int64))
    _lib.call(
        "mtpb_qkv_rope", xc.data_ptr(), h, _c(w).data_ptr(), _lib.ptr(None if bias is None else _c(bias)),
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), b, t, hq, hkv, hd, h, cap, cache_len,
        _lib.ptr(rp), cos.data_ptr(), sin.data_ptr(), cos.shape[0], _lib.dtype_code(x.dtype), _comm_handle(comm),
        _lib.stream_ptr(x.device),
    )
    return q


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, hq: int, hkv: int,
              cache_len: int, comm=None) -> torch.Tensor:
    """q [B, T, hq*hd] against cache slots [0, cache_len + t] -> [B, T, hq*hd]."""
    _lib.require_cuda(q, k_cache, v_cache)
    b, t, _ = q.shape
    hd = k_cache.shape[-1]
    out = torch.empty_like(q)
    _lib.call("mtpb_attention", _c(q).data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), b, t, hq,
              hkv, hd, k_cache.shape[2], cache_len, _lib.dtype_code(q.dtype), _comm_handle(comm),
              _lib.stream_ptr(q.device))
    return out
