"""mtpb_attention_noalloc: split-KV attention without any device allocation.

Callers whose device memory is owned by their own allocator or budget, or
whose serving loop cannot take the device-wide synchronisation of
cudaMalloc/cudaFree, use this entry point; it keeps its split-KV scratch in
a fixed array compiled into the library. These tests call it through the C
ABI, twice in a row per shape, so results cannot depend on what an earlier
call left in the shared array:

* against mtpb_attention (which allocates its scratch): the same kernel with
  the same split count, so the outputs must be bit-identical;
* against the CPU oracle of the reference's attention (minitp/attention.py:
  71-106) at the fp32 / bf16 tolerances of the other attention tests;
* the caller's status word stays clear on valid calls.

The file name makes pytest collect it last.
"""

import pytest
import torch

from minitp_b200 import _lib
from oracle import model as om

DT = {"fp32": torch.float32, "bf16": torch.bfloat16}
TOL = {"fp32": dict(atol=2e-5, rtol=1e-4), "bf16": dict(atol=2e-2, rtol=2e-2)}

# (dtype, B, T, hq, hkv, hd, cap, cache_len): decode shapes that split the
# cache (scratch in use), a chunked-prefill shape, and 7B-like head shapes.
SHAPES = [
    ("bf16", 1, 1, 14, 2, 64, 4096, 3000),
    ("fp32", 2, 1, 7, 1, 128, 2048, 1500),
    ("bf16", 4, 1, 28, 4, 128, 1024, 700),
    ("bf16", 1, 1, 7, 1, 128, 1280, 1279),
    ("fp32", 1, 3, 4, 2, 16, 512, 200),
]


def _inputs(dtype, B, T, hq, hkv, hd, cap, seed):
    g = torch.Generator().manual_seed(seed)
    dt = DT[dtype]
    q = torch.randn(B, T, hq * hd, generator=g).to(dt)
    kc = torch.randn(B, hkv, cap, hd, generator=g).to(dt)
    vc = torch.randn(B, hkv, cap, hd, generator=g).to(dt)
    return q, kc, vc


def _allocating(q, kc, vc, B, T, hq, hkv, hd, cap, cache_len):
    out = torch.empty_like(q)
    _lib.call("mtpb_attention", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), B, T, hq, hkv, hd,
              cap, cache_len, _lib.dtype_code(q.dtype), None, _lib.stream_ptr())
    return out


def _noalloc(q, kc, vc, B, T, hq, hkv, hd, cap, cache_len, status=None):
    out = torch.empty_like(q)
    _lib.call("mtpb_attention_noalloc", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), B, T, hq,
              hkv, hd, cap, cache_len, _lib.dtype_code(q.dtype), status.data_ptr() if status is not None else None,
              _lib.stream_ptr())
    return out


def _oracle(q, kc, vc, B, T, hq, hkv, hd, cache_len):
    qo = q.reshape(B, T, hq, hd).transpose(1, 2)
    end = cache_len + T
    ref = om.attention(qo, kc[:, :, :end], vc[:, :, :end], cache_len)
    return ref.transpose(1, 2).reshape(B, T, hq * hd)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{s[0]}_b{s[1]}_t{s[2]}_hq{s[3]}_hd{s[5]}_L{s[7]}" for s in SHAPES])
def test_noalloc_attention_matches_allocating_entry_point_and_oracle(lib, shape):
    dtype, B, T, hq, hkv, hd, cap, cache_len = shape
    q, kc, vc = _inputs(dtype, B, T, hq, hkv, hd, cap, seed=100 + SHAPES.index(shape))
    qg, kg, vg = q.cuda(), kc.cuda(), vc.cuda()
    want = _allocating(qg, kg, vg, B, T, hq, hkv, hd, cap, cache_len)
    ref = _oracle(q, kc, vc, B, T, hq, hkv, hd, cache_len)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(2):
        got = _noalloc(qg, kg, vg, B, T, hq, hkv, hd, cap, cache_len, status)
        torch.cuda.synchronize()
        assert torch.equal(got, want)  # same kernel, same splits: bit-identical
        torch.testing.assert_close(got.float().cpu(), ref.float(), **TOL[dtype])
    assert int(status.item()) == 0


@pytest.mark.gpu
def test_noalloc_attention_without_status_word(lib):
    dtype, B, T, hq, hkv, hd, cap, cache_len = SHAPES[0]
    q, kc, vc = _inputs(dtype, B, T, hq, hkv, hd, cap, seed=11)
    qg, kg, vg = q.cuda(), kc.cuda(), vc.cuda()
    want = _allocating(qg, kg, vg, B, T, hq, hkv, hd, cap, cache_len)
    for _ in range(2):
        got = _noalloc(qg, kg, vg, B, T, hq, hkv, hd, cap, cache_len)
        torch.cuda.synchronize()
        assert torch.equal(got, want)


@pytest.mark.gpu
def test_noalloc_attention_rejects_scratch_beyond_its_array(lib):
    # 8 rows x 64 query heads of 128 dims over 32 cache splits need 8 MiB of
    # partials, twice the fixed array: refused on the host before any launch.
    B, T, hq, hkv, hd, cap = 8, 1, 64, 1, 128, 8192
    q, kc, vc = _inputs("fp32", B, T, hq, hkv, hd, cap, seed=7)
    with pytest.raises(_lib.MinitpB200Error, match="bytes of scratch"):
        _noalloc(q.cuda(), kc.cuda(), vc.cuda(), B, T, hq, hkv, hd, cap, 100)
