"""The C ABI: the library builds, loads on a CPU-only host and exports every declared symbol.

No compute call is made here (no GPU).
"""

import os
import re

from minitp_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "minitp_b200.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mtpb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "mtpb_model_decode_step" in names and "mtpb_allreduce_residual_rmsnorm" in names
    assert len(names) >= 25


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_version_and_error_string(lib):
    assert lib.mtpb_version() >= 1
    assert isinstance(lib.mtpb_last_error(), bytes)


def test_invalid_comm_arguments_fail_cleanly(lib):
    import ctypes

    h = ctypes.c_void_p()
    assert lib.mtpb_comm_create(3, 2, 1 << 20, ctypes.byref(h)) == _lib.ERR_INVALID
    assert b"rank" in lib.mtpb_last_error()
    assert lib.mtpb_comm_create(0, 9, 1 << 20, ctypes.byref(h)) == _lib.ERR_INVALID


def test_cpu_tensors_raise_no_fallback(lib):
    import pytest
    import torch

    from minitp_b200 import ops

    with pytest.raises(_lib.MinitpB200Error, match="CUDA"):
        ops.linear(torch.zeros(1, 16), torch.zeros(8, 16))


def test_two_shot_slice_rule(lib):
    """Which AllReduce form a model site gets: one-shot by default; with the switch on, the two-shot
    column slice of ceil(H / tp) rounded up to whole 16-byte vectors, only from the set size and
    rank count on (host logic; no GPU needed)."""
    bf16 = _lib.MTPB_BF16
    assert lib.mtpb_allreduce_two_shot_cols(1 << 24, 3584, 8, bf16) == 0  # off by default
    try:
        assert lib.mtpb_set_allreduce_two_shot(1 << 20, 4) == 0
        assert lib.mtpb_allreduce_two_shot_cols(1 << 20, 3584, 8, bf16) == 448
        assert lib.mtpb_allreduce_two_shot_cols(1 << 20, 896, 4, bf16) == 224
        assert lib.mtpb_allreduce_two_shot_cols(1 << 20, 896, 8, _lib.MTPB_F32) == 112
        assert lib.mtpb_allreduce_two_shot_cols((1 << 20) - 1, 3584, 8, bf16) == 0  # below the size
        assert lib.mtpb_allreduce_two_shot_cols(1 << 20, 3584, 2, bf16) == 0  # below the rank count
        assert lib.mtpb_allreduce_two_shot_cols(1 << 20, 900, 4, bf16) == 0  # rows of partial vectors
        assert lib.mtpb_set_allreduce_two_shot(1 << 20, 2) == 0
        assert lib.mtpb_allreduce_two_shot_cols(1 << 20, 896, 3, bf16) == 304  # 298.7 -> 38 vectors of 8
        assert lib.mtpb_set_allreduce_two_shot(0, 1) == _lib.ERR_INVALID
    finally:
        lib.mtpb_set_allreduce_two_shot(-1, 4)
