"""Operator parity on the GPU: each minitp_b200 kernel against a CPU reference.

Floating-point kernels are compared with a torch fp32 computation or the
CPU oracle (the reference algorithm). The tolerance is written beside each
check. Integer and id outputs (argmax, embedding) must be bit-exact.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import model as om
from oracle.argmax import distributed_argmax

pytestmark = pytest.mark.gpu

DT = {"fp32": torch.float32, "bf16": torch.bfloat16}


def _ref_linear(x, w, b=None):
    y = x.double() @ w.double().T
    if b is not None:
        y = y + b.double()
    return y


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("M,N,K", [(1, 576, 896), (1, 896, 448), (1, 896, 2432), (3, 4864, 896),
                                   (8, 1000, 64), (17, 128, 64), (1, 75968, 896), (5, 96, 32)])
def test_linear(lib, dtype, M, N, K):
    from minitp_b200 import ops

    g = torch.Generator().manual_seed(M * 1000 + N + K)
    x = torch.randn(M, K, generator=g).to(DT[dtype])
    w = (torch.randn(N, K, generator=g) * 0.02).to(DT[dtype])
    b = (torch.randn(N, generator=g) * 0.02).to(DT[dtype])
    y = ops.linear(x.cuda(), w.cuda(), b.cuda()).cpu()
    ref = _ref_linear(x, w, b)
    if dtype == "fp32":
        # fp32 accumulation order differs from the float64 reference
        torch.testing.assert_close(y.double(), ref, atol=2e-5, rtol=1e-4)
    else:
        # one rounding of an fp32 accumulation to bf16: within 1 bf16 ulp (2^-8 relative)
        torch.testing.assert_close(y.double(), ref.to(torch.bfloat16).double(), atol=1e-3, rtol=2 ** -7)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_swiglu(lib, dtype):
    from minitp_b200 import ops

    g = torch.Generator().manual_seed(5)
    M, I, K = 3, 2432, 896
    x = torch.randn(M, K, generator=g).to(DT[dtype])
    w = (torch.randn(2 * I, K, generator=g) * 0.02).to(DT[dtype])
    y = ops.linear_swiglu(x.cuda(), w.cuda()).cpu()
    gate, up = torch.chunk(_ref_linear(x, w).to(DT[dtype]), 2, dim=-1)  # rounded like F.linear
    ref = F.silu(gate.float()).to(DT[dtype]).float() * up.float()
    tol = dict(atol=1e-5, rtol=1e-4) if dtype == "fp32" else dict(atol=1e-3, rtol=2 ** -6)
    torch.testing.assert_close(y.float(), ref.to(DT[dtype]).float(), **tol)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("H", [64, 896, 3584])
def test_rmsnorm(lib, dtype, H):
    from minitp_b200 import ops

    g = torch.Generator().manual_seed(H)
    x = torch.randn(5, H, generator=g).to(DT[dtype])
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(DT[dtype])
    y = ops.rmsnorm(x.cuda(), w.cuda(), 1e-6).cpu()
    ref = om.rmsnorm(x, w, 1e-6)
    tol = dict(atol=1e-6, rtol=1e-5) if dtype == "fp32" else dict(atol=0, rtol=2 ** -7)
    torch.testing.assert_close(y.float(), ref.float(), **tol)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("hq,hkv,hd", [(7, 1, 64), (14, 2, 64), (4, 2, 16), (7, 1, 128), (4, 1, 128)])
@pytest.mark.parametrize("T,cache_len", [(1, 0), (1, 37), (1, 300), (9, 0), (5, 11), (16, 0), (100, 0), (257, 20),
                                         (40, 130)])
def test_qkv_rope_attention(lib, dtype, hq, hkv, hd, T, cache_len):
    """Fused QKV + RoPE + KV append, then split-KV GQA attention, vs the oracle."""
    from minitp_b200 import ops
    from minitp_b200.rope import rope_tables

    torch.manual_seed(hq * 100 + hd + T + cache_len)
    B, H, cap = 2, 128, 512
    dt = DT[dtype]
    x = torch.randn(B, T, H).to(dt)
    w = (torch.randn((hq + 2 * hkv) * hd, H) * 0.05).to(dt)
    b = (torch.randn((hq + 2 * hkv) * hd) * 0.05).to(dt)
    kc = torch.randn(B, hkv, cap, hd).to(dt)
    vc = torch.randn(B, hkv, cap, hd).to(dt)
    cos, sin = rope_tables(hd, 1e6, 4096)
    q = ops.qkv_rope(x.cuda(), w.cuda(), b.cuda(), kcg := kc.cuda(), vcg := vc.cuda(), hq, hkv, cache_len,
                     None, cos.cuda(), sin.cuda())
    out = ops.attention(q, kcg, vcg, hq, hkv, cache_len).cpu()
    # oracle
    y = F.linear(x, w, b)
    qo, ko, vo = torch.split(y, [hq * hd, hkv * hd, hkv * hd], dim=-1)
    qo = qo.reshape(B, T, hq, hd).transpose(1, 2)
    ko = ko.reshape(B, T, hkv, hd).transpose(1, 2)
    vo = vo.reshape(B, T, hkv, hd).transpose(1, 2)
    pos = torch.arange(cache_len, cache_len + T)
    qo, ko = om.apply_rope(qo, cos[pos], sin[pos]), om.apply_rope(ko, cos[pos], sin[pos])
    kref, vref = kc.clone(), vc.clone()
    kref[:, :, cache_len:cache_len + T] = ko
    vref[:, :, cache_len:cache_len + T] = vo
    end = cache_len + T
    ref = om.attention(qo, kref[:, :, :end], vref[:, :, :end], cache_len).transpose(1, 2).reshape(B, T, hq * hd)
    tol = dict(atol=2e-5, rtol=1e-4) if dtype == "fp32" else dict(atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(kcg.cpu()[:, :, :end].float(), kref[:, :, :end].float(), **tol)
    torch.testing.assert_close(vcg.cpu()[:, :, :end].float(), vref[:, :, :end].float(), **tol)
    torch.testing.assert_close(out.float(), ref.float(), **tol)
    # slots beyond the written range are untouched
    assert torch.equal(kcg.cpu()[:, :, end:], kc[:, :, end:])


def test_rope_matches_reference_golden(lib):
    """RoPE through the fused kernel (identity projection) vs the reference RotaryEmbedding.apply."""
    from tests.conftest import golden
    from minitp_b200 import ops
    from minitp_b200.rope import rope_tables

    gd = golden("rope.npz")
    for hd in (16, 64, 128):
        cos, sin = rope_tables(hd, 1e6, 4096)
        assert np.array_equal(cos[[0, 1, 95, 1000, 4095]].numpy(), gd[f"cos_hd{hd}"])
        g = torch.Generator().manual_seed(hd)
        q = torch.randn(2, 4, 5, hd, generator=g)
        k = torch.randn(2, 1, 5, hd, generator=g)
        pos = torch.tensor([0, 1, 95, 1000, 4095])
        for dt in ("fp32", "bf16"):
            # feed q/k heads as rows of the identity: y = x @ I^T = x
            for t in range(5):
                hq, hkv = 4, 1
                x = torch.cat([q[:, :, t].reshape(2, -1), k[:, :, t].reshape(2, -1),
                               torch.zeros(2, hd)], dim=-1).to(DT[dt])  # [B, (hq+2hkv)*hd]
                n = (hq + 2 * hkv) * hd
                w = torch.eye(n, dtype=DT[dt])
                kc = torch.zeros(2, hkv, 4096, hd, dtype=DT[dt], device="cuda")
                vc = torch.zeros_like(kc)
                rp = pos[t:t + 1].cuda()
                qo = ops.qkv_rope(x[:, None].cuda(), w.cuda(), None, kc, vc, hq, hkv, int(pos[t]), rp,
                                  cos.cuda(), sin.cuda()).cpu()
                want_q = torch.from_numpy(gd[f"q_hd{hd}_{dt}"])[:, :, t].reshape(2, -1)
                want_k = torch.from_numpy(gd[f"k_hd{hd}_{dt}"])[:, 0, t]
                assert torch.equal(qo[:, 0].float(), want_q), (hd, dt, t)
                assert torch.equal(kc[:, 0, int(pos[t])].cpu().float(), want_k), (hd, dt, t)


@pytest.mark.parametrize("vocab,batch", [(151936, 1), (151936, 8), (151937, 64)])
def test_embedding_tp1_exact(lib, vocab, batch):
    from minitp_b200 import ops
    from minitp_b200.synthetic_cases import embedding_case

    table, ids = embedding_case(vocab, 896, batch, seed=vocab * 7 + batch)
    out = ops.embedding(ids.cuda(), table.cuda(), 0, vocab, vocab, None).cpu()
    assert torch.equal(out, F.embedding(ids, table))


def test_argmax_tp1_semantics(lib):
    """TP=1 greedy ids follow torch.argmax: first max, NaN wins (reference embedding.py:146-147)."""
    from minitp_b200 import ops
    from minitp_b200.synthetic_cases import argmax_logits

    for vocab, batch in [(151936, 1), (151937, 8), (151936, 64)]:
        x = argmax_logits(vocab, batch, seed=vocab + batch)
        got = ops.argmax(x.cuda(), 0, None).cpu().squeeze(-1)
        assert torch.equal(got, x.argmax(-1)), (vocab, batch)
    x = torch.zeros(3, 1000)
    x[0, 5] = x[0, 2] = 2.0  # tie -> 2
    x[1, 7] = float("nan")
    x[1, 9] = float("nan")  # first NaN wins at tp=1
    x[2] = -1.0
    x[2, 999] = -0.0  # -0.0 normalised: equals +0.0, the max
    got = ops.argmax(x.cuda(), 0, None).cpu().squeeze(-1)
    assert got.tolist() == [2, 7, 999]
    assert got.tolist() == distributed_argmax(x.numpy(), 1).tolist()
    for b in (torch.bfloat16,):
        xb = torch.randn(4, 5000).to(b)
        assert torch.equal(ops.argmax(xb.cuda(), 0, None).cpu().squeeze(-1), xb.float().argmax(-1))


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("rows", [1, 8, 64, 2048])
def test_allreduce_residual_rmsnorm_world1(lib, dtype, rows):
    from minitp_b200 import ops

    g = torch.Generator().manual_seed(rows)
    dt = DT[dtype]
    p = torch.randn(rows, 896, generator=g).to(dt)
    r = torch.randn(rows, 896, generator=g).to(dt)
    gain = (1 + 0.1 * torch.randn(896, generator=g)).to(dt)
    res, nrm = ops.allreduce_residual_rmsnorm(p.cuda(), r.cuda(), gain.cuda(), 1e-6, None)
    want_res, want_nrm = om.allreduce_residual_rmsnorm([p], r, gain, 1e-6)
    assert torch.equal(res.cpu(), want_res)  # one rounding of an exact sum
    tol = dict(atol=1e-6, rtol=1e-5) if dtype == "fp32" else dict(atol=0, rtol=2 ** -7)
    torch.testing.assert_close(nrm.cpu().float(), want_nrm.float(), **tol)


def test_row_parallel_bias_added_once(lib):
    """Reference tests/test_column_row_parallel.py:72-80: zero weight, bias 1 -> exactly 1."""
    from minitp_b200.distributed.context import context_for
    from minitp_b200.parallel.linear import RowParallelLinear

    layer = RowParallelLinear(12, 8, context_for(1, "cuda"), bias=True, input_is_parallel=False).cuda()
    with torch.no_grad():
        layer.weight.zero_()
        layer.bias.fill_(1.0)
    assert layer(torch.zeros(2, 12, device="cuda")).max().item() == 1.0
