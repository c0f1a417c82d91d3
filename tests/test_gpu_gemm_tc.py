"""Tensor-core (tcgen05) GEMM of the bf16 prefill projections.

bf16 projections with at least 64 rows run on the tensor-core kernel
(gemm_tc.cuh); these tests pin its output against a float64 reference of the
same bf16 inputs, with the store, SwiGLU and fused QKV + RoPE + KV-append
epilogues, full and partial tiles, K that is not a multiple of the 64-element
K block, both tile widths of the single-CTA kernel (128 and 256 accumulator
columns), the CTA-pair kernel (256 x 256 tiles, cta_group::2: projections of
>= 256 rows with at least one tile per co-resident pair), and persistent CTAs
that take several tiles each (both tensor-memory accumulators in turn), and
split K for projections with few output tiles.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import model as om

pytestmark = pytest.mark.gpu


def _ref_linear(x, w, b=None):
    y = x.double() @ w.double().t()
    return y if b is None else y + b.double()


@pytest.mark.parametrize("M,N,K", [(64, 128, 64), (128, 1152, 896), (200, 300, 896), (128, 896, 4864),
                                   (256, 640, 1000), (130, 4096, 896),
                                   (2048, 9728, 896), (1152, 2304, 512), (300, 20000, 128),
                                   (200, 40000, 64)])
def test_tc_linear(lib, M, N, K):
    from minitp_b200 import ops

    g = torch.Generator().manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16)
    y = ops.linear(x.cuda(), w.cuda(), b.cuda()).cpu()
    ref = _ref_linear(x, w, b)
    # fp32 accumulation in tensor memory, one rounding to bf16
    torch.testing.assert_close(y.double(), ref.to(torch.bfloat16).double(), atol=1e-3, rtol=2 ** -7)
    # the GEMV kernel on the same inputs agrees to the same tolerance
    lib.mtpb_set_tc_min_rows(1 << 30)
    try:
        y2 = ops.linear(x.cuda(), w.cuda(), b.cuda()).cpu()
    finally:
        lib.mtpb_set_tc_min_rows(64)
    torch.testing.assert_close(y.float(), y2.float(), atol=1e-3, rtol=2 ** -7)


@pytest.mark.parametrize("M,N,K", [(16, 1152, 3584), (32, 3584, 4736), (48, 896, 896)])
def test_tc_linear_few_rows(lib, M, N, K):
    """Projections of 16-63 rows (a kernel-chain decode step at batch >= 16) on the tensor cores."""
    from minitp_b200 import ops

    g = torch.Generator().manual_seed(M * 5 + N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    lib.mtpb_set_tc_min_rows(16)
    try:
        y = ops.linear(x.cuda(), w.cuda()).cpu()
        s = ops.linear_swiglu(x.cuda(), w.cuda()).cpu()
    finally:
        lib.mtpb_set_tc_min_rows(64)
    ref = _ref_linear(x, w)
    torch.testing.assert_close(y.double(), ref.to(torch.bfloat16).double(), atol=1e-3, rtol=2 ** -7)
    gate, up = torch.chunk(ref.to(torch.bfloat16), 2, dim=-1)
    sref = F.silu(gate.float()).to(torch.bfloat16).float() * up.float()
    torch.testing.assert_close(s.float(), sref.to(torch.bfloat16).float(), atol=1e-3, rtol=2 ** -6)


@pytest.mark.parametrize("epi,M,N,K", [("store", 8, 768, 3584), ("store", 32, 896, 4864), ("swiglu", 8, 4736, 3584),
                                       ("store", 48, 1152, 896), ("store", 8, 3584, 512), ("swiglu", 64, 2000, 200)])
def test_tc_split_k(lib, epi, M, N, K):
    """Split K (output tiles filling at most half of the SMs): the float64 reference, the unsplit kernel
    within the same tolerance, and bit-identical results on repeated calls (partials summed in range order)."""
    from minitp_b200 import ops

    g = torch.Generator().manual_seed(M * 3 + N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).cuda()
    fn = ops.linear_swiglu if epi == "swiglu" else ops.linear
    lib.mtpb_set_tc_min_rows(1)
    try:
        y1 = fn(x, w).cpu()
        y2 = fn(x, w).cpu()
        prev = lib.mtpb_set_tc_split(1)
        try:
            y0 = fn(x, w).cpu()
        finally:
            lib.mtpb_set_tc_split(prev)
    finally:
        lib.mtpb_set_tc_min_rows(64)
    assert torch.equal(y1, y2)
    ref = _ref_linear(x.cpu(), w.cpu()).to(torch.bfloat16)
    if epi == "swiglu":
        gate, up = torch.chunk(ref, 2, dim=-1)
        ref = (F.silu(gate.float()).to(torch.bfloat16).float() * up.float()).to(torch.bfloat16)
    tol = dict(atol=1e-3, rtol=2 ** -6)
    torch.testing.assert_close(y1.float(), ref.float(), **tol)
    torch.testing.assert_close(y1.float(), y0.float(), **tol)


@pytest.mark.parametrize("M,I,K", [(128, 2432, 896), (96, 200, 256), (1024, 4864, 896),
                                   (1000, 2500, 192)])
def test_tc_swiglu(lib, M, I, K):
    from minitp_b200 import ops

    g = torch.Generator().manual_seed(M + I + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * I, K, generator=g) * 0.02).to(torch.bfloat16)
    y = ops.linear_swiglu(x.cuda(), w.cuda()).cpu()
    gate, up = torch.chunk(_ref_linear(x, w).to(torch.bfloat16), 2, dim=-1)
    ref = F.silu(gate.float()).to(torch.bfloat16).float() * up.float()
    torch.testing.assert_close(y.float(), ref.to(torch.bfloat16).float(), atol=1e-3, rtol=2 ** -6)


@pytest.mark.parametrize("hq,hkv,hd,T,H", [(14, 2, 64, 128, 896), (7, 1, 64, 100, 896), (7, 1, 128, 64, 896),
                                          (28, 4, 128, 2048, 256), (8, 2, 32, 300, 256)])
def test_tc_qkv_rope(lib, hq, hkv, hd, T, H):
    """Prefill QKV projection + bias + RoPE + KV append through the tensor-core path."""
    from minitp_b200 import ops
    from minitp_b200.rope import rope_tables

    torch.manual_seed(hq * 10 + hd + T)
    B, cap = 1, max(512, T + 64)
    x = torch.randn(B, T, H).to(torch.bfloat16)
    w = (torch.randn((hq + 2 * hkv) * hd, H) * 0.05).to(torch.bfloat16)
    b = (torch.randn((hq + 2 * hkv) * hd) * 0.05).to(torch.bfloat16)
    kc = torch.zeros(B, hkv, cap, hd).to(torch.bfloat16)
    vc = torch.zeros(B, hkv, cap, hd).to(torch.bfloat16)
    cos, sin = rope_tables(hd, 1e6, 4096)
    kcg, vcg = kc.cuda(), vc.cuda()
    q = ops.qkv_rope(x.cuda(), w.cuda(), b.cuda(), kcg, vcg, hq, hkv, 0, None, cos.cuda(), sin.cuda()).cpu()
    y = (x.double() @ w.double().t() + b.double()).to(torch.bfloat16)
    qo, ko, vo = torch.split(y, [hq * hd, hkv * hd, hkv * hd], dim=-1)
    qo = qo.reshape(B, T, hq, hd).transpose(1, 2)
    ko = ko.reshape(B, T, hkv, hd).transpose(1, 2)
    vo = vo.reshape(B, T, hkv, hd).transpose(1, 2)
    pos = torch.arange(T)
    qo, ko = om.apply_rope(qo, cos[pos], sin[pos]), om.apply_rope(ko, cos[pos], sin[pos])
    tol = dict(atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(q.reshape(B, T, hq, hd).transpose(1, 2).float(), qo.float(), **tol)
    torch.testing.assert_close(kcg.cpu()[:, :, :T].float(), ko.float(), **tol)
    torch.testing.assert_close(vcg.cpu()[:, :, :T].float(), vo.float(), **tol)
    assert torch.equal(kcg.cpu()[:, :, T:], kc[:, :, T:])


@pytest.mark.parametrize("epi,M,N,K", [("store", 2048, 9728, 896), ("swiglu", 1024, 9728, 896),
                                       ("store", 768, 20480, 320), ("swiglu", 300, 20000, 128)])
def test_tc_pair_matches_single_cta(lib, epi, M, N, K):
    """The CTA-pair kernel and the single-CTA kernel agree on the same inputs."""
    from minitp_b200 import ops

    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).cuda()
    fn = ops.linear_swiglu if epi == "swiglu" else ops.linear
    y_pair = fn(x, w).cpu()
    prev = lib.mtpb_set_tc_pair(0)
    try:
        y_single = fn(x, w).cpu()
    finally:
        lib.mtpb_set_tc_pair(prev)
    torch.testing.assert_close(y_pair.float(), y_single.float(), atol=1e-3, rtol=2 ** -7)
