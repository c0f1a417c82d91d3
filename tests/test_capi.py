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
