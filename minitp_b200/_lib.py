"""ctypes binding of libminitp_b200.so (C ABI declared in include/minitp_b200.h).

This module is the only place that loads the native library. There is no
fallback: if the library is missing or the tensors are not on a CUDA device,
calls raise.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int, c_int64, c_uint32, c_uint64, c_void_p

import torch

from minitp_b200.build import LIB_PATH

MTPB_F32 = 0
MTPB_BF16 = 1
ERR_INVALID, ERR_CUDA, ERR_TIMEOUT, ERR_DEVICE = -1, -2, -3, -4

STATUS_TIMEOUT = 1
STATUS_BAD_POSITION = 2
STATUS_BAD_TOKEN = 4


class ModelDesc(ctypes.Structure):
    _fields_ = [
        ("dtype", c_int),
        ("hidden", c_int),
        ("inter_local", c_int),
        ("n_layers", c_int),
        ("hq_local", c_int),
        ("hkv_local", c_int),
        ("head_dim", c_int),
        ("vocab_start", c_int64),
        ("vocab_end", c_int64),
        ("vocab_size", c_int64),
        ("eps", c_float),
        ("embed", c_void_p),
        ("lm_head", c_void_p),
        ("final_norm", c_void_p),
        ("cos_tab", c_void_p),
        ("sin_tab", c_void_p),
        ("rope_len", c_int),
    ]


class LayerDesc(ctypes.Structure):
    _fields_ = [
        ("ln1", c_void_p),
        ("qkv_w", c_void_p),
        ("qkv_b", c_void_p),
        ("o_w", c_void_p),
        ("ln2", c_void_p),
        ("gu_w", c_void_p),
        ("down_w", c_void_p),
    ]


# name -> (restype, argtypes), in the order of include/minitp_b200.h
SIGNATURES: dict[str, tuple] = {
    "mtpb_last_error": (ctypes.c_char_p, []),
    "mtpb_version": (c_int, []),
    "mtpb_set_pdl": (c_int, [c_int]),
    "mtpb_set_prefetch_cap": (c_int, [c_uint32]),
    "mtpb_set_gemv_ctas_per_sm": (c_int, [c_int]),
    "mtpb_set_tc_min_rows": (c_int, [c_int]),
    "mtpb_set_tc_min_rows_decode": (c_int, [c_int]),
    "mtpb_set_tc_pair": (c_int, [c_int]),
    "mtpb_set_tc_split": (c_int, [c_int]),
    "mtpb_set_allreduce_two_shot": (c_int, [c_int64, c_int]),
    "mtpb_allreduce_two_shot_cols": (c_int, [c_int64, c_int, c_int, c_int]),
    "mtpb_comm_create": (c_int, [c_int, c_int, c_uint64, POINTER(c_void_p)]),
    "mtpb_comm_ipc_handle": (c_int, [c_void_p, c_void_p]),
    "mtpb_comm_open": (c_int, [c_void_p, c_void_p]),
    "mtpb_comm_destroy": (c_int, [c_void_p]),
    "mtpb_comm_set_timeout": (c_int, [c_void_p, c_uint64]),
    "mtpb_comm_status": (c_int, [c_void_p, POINTER(c_uint32)]),
    "mtpb_comm_clear_status": (c_int, [c_void_p]),
    "mtpb_comm_pos_ptr": (c_void_p, [c_void_p]),
    "mtpb_comm_set_pos": (c_int, [c_void_p, c_int, c_void_p]),
    "mtpb_comm_slot_bytes": (c_uint64, [c_void_p]),
    "mtpb_comm_pingpong": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "mtpb_linear": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                            c_void_p]),
    "mtpb_linear_swiglu": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                   c_void_p]),
    "mtpb_qkv_rope": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                              c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int,
                              c_int, c_void_p, c_void_p]),
    "mtpb_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                               c_int, c_int, c_void_p, c_void_p]),
    "mtpb_attention_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                       c_int, c_int, c_int, c_void_p, c_void_p]),
    "mtpb_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_int, c_void_p]),
    "mtpb_allreduce": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "mtpb_allreduce_residual_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                                c_void_p, c_int, c_int, c_float, c_int, c_void_p]),
    "mtpb_embedding": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int64, c_int64, c_int64,
                               c_int, c_void_p]),
    "mtpb_argmax": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int64, c_int64, c_void_p, c_void_p, c_int,
                            c_void_p]),
    "mtpb_model_create": (c_int, [POINTER(ModelDesc), c_void_p, POINTER(c_void_p)]),
    "mtpb_model_set_layer": (c_int, [c_void_p, c_int, POINTER(LayerDesc)]),
    "mtpb_model_reserve": (c_int, [c_void_p, c_int, c_int]),
    "mtpb_model_destroy": (c_int, [c_void_p]),
    "mtpb_model_forward": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int,
                                   c_void_p, c_int, c_void_p]),
    "mtpb_model_decode_step": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int,
                                       c_void_p, c_void_p]),
    "mtpb_model_decode_kernels": (c_int, [c_void_p, c_int, c_int, POINTER(c_int)]),
    "mtpb_set_decode_impl": (c_int, [c_int]),
    "mtpb_set_decode_trace": (c_int, [c_void_p]),
    "mtpb_set_decode_ring": (c_int, [c_int, c_int, c_int]),
    "mtpb_set_decode_spin": (c_int, [c_int]),
    "mtpb_settings_epoch": (c_uint64, []),
}

_lib: ctypes.CDLL | None = None


class MinitpB200Error(RuntimeError):
    """A failure reported by the native library."""


class PeerTimeoutError(MinitpB200Error):
    """A bounded wait on a peer rank ran out (the peer never joined the step)."""


def load() -> ctypes.CDLL:
    """Load the library (once) and declare every exported function."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MinitpB200Error(
                f"{LIB_PATH} is missing: build it with `python -m minitp_b200.build` "
                "(minitp_b200 has no CPU or library fallback)"
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int) -> None:
    if rc == 0:
        return
    msg = load().mtpb_last_error().decode(errors="replace")
    if rc == ERR_TIMEOUT:
        raise PeerTimeoutError(msg)
    raise MinitpB200Error(f"minitp_b200 error {rc}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return MTPB_BF16
    if dtype == torch.float32:
        return MTPB_F32
    raise MinitpB200Error(f"unsupported dtype {dtype}: minitp_b200 kernels run fp32 or bf16")


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise MinitpB200Error(
                "minitp_b200 kernels run on CUDA devices only (got a tensor on "
                f"{t.device}); there is no CPU fallback"
            )


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def status_error(status: int) -> str:
    parts = []
    if status & STATUS_TIMEOUT:
        parts.append("a bounded wait on a peer rank timed out")
    if status & STATUS_BAD_POSITION:
        parts.append("a position outside the KV cache or the RoPE table")
    if status & STATUS_BAD_TOKEN:
        parts.append("a token id outside the vocabulary")
    return "; ".join(parts) or f"status {status:#x}"
