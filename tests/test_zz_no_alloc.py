"""mtpb_attention_noalloc: split-KV attention without any device allocation.

Callers whose device memory is owned by their own allocator or budget, or
whose serving loop cannot take the device-wide synchronisation of
cudaMalloc/cudaFree, use this entry point; it keeps its split-KV scratch in
a fixed array compiled into the library. These tests call it through the C
ABI and compare it with mtpb_attention (which allocates its scratch) on the
same inputs, twice in a row per shape, so results cannot depend on what an
earlier call left in the shared array. The file name makes pytest collect it
last.
"""

import pytest
import torch

from minitp_b200 import _lib

DT = {"fp32": torch.float32, "bf16": torch.bfloat16}
TOL = {"fp32": dict(atol=2e-5, rtol=1e-4), "bf16": dict(atol=2e-2, rtol=2e-2)}

# (dtype, B, T, hq, hkv, hd, cap, cache_len): decode shapes that split the
# cache (scratch in use), a chunked-prefill shape, and a 7B-like head shape.
SHAPES = [
    ("bf16", 1, 1, 14, 2, 64, 4096, 3000),
    ("fp32", 2, 1, 7, 1, 128, 2048, 1500),
    ("bf16", 4, 1, 28, 4, 128, 1024, 700),
    ("fp32", 1, 3, 4, 2, 16, 512, 200),
]


def _inputs(dtype, B, T, hq, hkv, hd, cap, seed):
    g = torch.Generator().manual_seed(seed)
    dt = DT[dtype]
    q = torch.randn(B, T, hq * hd, generator=g).to(dt).cuda()
    kc = torch.randn(B, hkv, cap, hd, generator=g).to(dt).cuda()
    vc = torch.randn(B, hkv, cap, hd, generator=g).to(dt).cuda()
    return q, kc, vc


def _allocating(q, kc, vc, B, T, hq, hkv, hd, cap, cache_len):
    out = torch.empty_like(q)
    _lib.call("mtpb_attention", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), B, T, hq, hkv, hd,
              cap, cache_len, _lib.dtype_code(q.dtype), None, _lib.stream_ptr())
    return out


def _noalloc(q, kc, vc, B, T, hq, hkv, hd, cap, cache_len):
    out = torch.empty_like(q)
    _lib.call("mtpb_attention_noalloc", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), B, T, hq,
              hkv, hd, cap, cache_len, _lib.dtype_code(q.dtype), _lib.stream_ptr())
    return out


@pytest.mark.gpu
def test_noalloc_attention_matches_allocating_entry_point(lib):
    for i, (dtype, B, T, hq, hkv, hd, cap, cache_len) in enumerate(SHAPES):
        q, kc, vc = _inputs(dtype, B, T, hq, hkv, hd, cap, seed=100 + i)
        want = _allocating(q, kc, vc, B, T, hq, hkv, hd, cap, cache_len)
        for _ in range(2):
            got = _noalloc(q, kc, vc, B, T, hq, hkv, hd, cap, cache_len)
            torch.cuda.synchronize()
            torch.testing.assert_close(got.float().cpu(), want.float().cpu(), **TOL[dtype])


@pytest.mark.gpu
def test_noalloc_attention_rejects_scratch_beyond_its_array(lib):
    # 8 rows x 64 query heads of 128 dims over 32 cache splits need 8 MiB of
    # partials, twice the fixed array: refused on the host before any launch.
    B, T, hq, hkv, hd, cap = 8, 1, 64, 1, 128, 8192
    q, kc, vc = _inputs("fp32", B, T, hq, hkv, hd, cap, seed=7)
    with pytest.raises(_lib.MinitpB200Error, match="bytes of scratch"):
        _noalloc(q, kc, vc, B, T, hq, hkv, hd, cap, 100)
