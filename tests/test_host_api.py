"""Host-side API of minitp_b200: config validation, shard math, padding, loaders, module layout.

Known-answer values are the reference's hand-computed ones
(tests/test_shard_oracle.py:15-75, tests/test_column_row_parallel.py:143-154,
tests/test_fused_projections.py:59-76).
"""

import numpy as np
import pytest
import torch

from minitp_b200 import config as mcfg
from minitp_b200.config import ModelConfig
from minitp_b200.distributed.context import ParallelContext
from minitp_b200.parallel.linear import ColumnParallelLinear, RowParallelLinear, shard_range
from minitp_b200.weight_loader import fused_qkv_local_sizes, kv_head_rows, shard_len


def _ctx(tp, rank=0):
    return ParallelContext(rank, rank, tp, rank, tp, torch.device("cpu"), None)


def test_shard_range_known_answers():
    assert shard_range(12, 0, 2) == (0, 6)
    assert shard_range(12, 1, 2) == (6, 12)
    assert shard_range(9, 0, 2) == (0, 5)
    assert shard_range(9, 1, 2) == (5, 9)
    assert shard_range(10, 0, 3) == (0, 4)
    assert shard_range(10, 1, 3) == (4, 7)
    assert shard_range(10, 2, 3) == (7, 10)
    assert shard_len(151937, 0, 2) == (0, 75969)
    assert shard_len(151937, 1, 2) == (75969, 75968)


def test_kv_head_rows_and_fused_sizes():
    assert kv_head_rows(2, 2, 0, 2) == (0, 2)
    assert kv_head_rows(2, 2, 1, 2) == (2, 2)
    assert kv_head_rows(1, 2, 0, 2) == (0, 2) and kv_head_rows(1, 2, 1, 2) == (0, 2)
    assert kv_head_rows(4, 128, 5, 8) == (256, 128)  # 7B TP8: rank 5 owns head 2
    cfg = ModelConfig(896, 4864, 2, 14, 2, 64, 1000, 1e-6, 1e6, 128)
    assert fused_qkv_local_sizes(cfg, 1) == (896, 128)
    assert fused_qkv_local_sizes(cfg, 2) == (448, 64)
    cfg2 = ModelConfig(64, 128, 1, 8, 1, 16, 100, 1e-6, 1e4, 64)
    assert fused_qkv_local_sizes(cfg2, 2) == (64, 16)


def test_validate_matches_reference_errors():
    with pytest.raises(ValueError, match="num_attention_heads=28 not divisible by tp_size=8"):
        mcfg.qwen25_7b().validate(8)
    with pytest.raises(ValueError, match="divisible"):
        mcfg.qwen25_05b().validate(4)
    mcfg.qwen25_05b().validate(2)
    mcfg.qwen25_7b().validate(4)


@pytest.mark.parametrize("factory,tp,q_pad,q_local", [
    (mcfg.qwen25_7b, 8, 32, 4), (mcfg.qwen25_05b, 4, 16, 4), (mcfg.qwen25_05b, 8, 16, 2),
    (mcfg.qwen25_7b, 4, 28, 7), (mcfg.qwen25_05b, 2, 14, 7),
])
def test_q_head_padding(factory, tp, q_pad, q_local):
    cfg = factory().padded_for(tp)
    assert cfg.num_attention_heads == q_pad
    assert cfg.local_heads(tp)[0] == q_local
    hmap = cfg.padded_head_map()
    real = [h for h in hmap if h >= 0]
    assert sorted(real) == list(range(factory().num_attention_heads))  # every real head kept once
    # each rank's q heads belong to its KV head's group (GQA structure preserved)
    g_real = factory().num_attention_heads // cfg.num_key_value_heads
    for r in range(tp):
        kv0, kvn = kv_head_rows(cfg.num_key_value_heads, 1, r, tp)
        heads = [h for h in hmap[r * q_local:(r + 1) * q_local] if h >= 0]
        assert all(kv0 <= h // g_real < kv0 + kvn for h in heads)


def test_divisibility_errors_of_layers():
    ctx = _ctx(2)
    with pytest.raises(ValueError, match="divisible"):
        ColumnParallelLinear(8, 15, ctx)
    with pytest.raises(ValueError, match="divisible"):
        RowParallelLinear(15, 8, ctx)


def test_state_dict_keys_match_reference_layout():
    from minitp_b200.layer import TPQwen2ForCausalLM

    cfg = mcfg.baseline_tiny()
    m = TPQwen2ForCausalLM(cfg, _ctx(1), init_weights=False)
    keys = set(m.state_dict())
    assert "model.layers.0.self_attn.qkv_proj.weight" in keys
    assert "model.layers.1.mlp.gate_up_proj.weight" in keys
    assert "model.embed_tokens.weight" in keys and "model.norm.weight" in keys
    assert m.lm_head.weight is m.model.embed_tokens.weight  # tied
    assert tuple(m.model.layers[0].self_attn.qkv_proj.weight.shape) == (128, 64)


def test_kv_cache_api():
    from minitp_b200.kv_cache import KVCache

    with pytest.raises(ValueError, match="init"):
        KVCache(1, 1, 1, 8, 4, torch.float32, torch.device("cpu"), init="bogus")
    kv = KVCache(2, 1, 1, 8, 4, torch.float32, torch.device("cpu"), init="zeros")
    k, v = kv.update(0, torch.ones(1, 1, 3, 8), torch.ones(1, 1, 3, 8))
    assert k.shape == (1, 1, 3, 8)
    kv.advance(3)
    with pytest.raises(ValueError, match="overflow"):
        kv.update(0, torch.ones(1, 1, 2, 8), torch.ones(1, 1, 2, 8))


def test_argmax_encoding_guards():
    from minitp_b200.parallel.embedding import VocabParallelLMHead

    head = VocabParallelLMHead(4, 21_000_000, _ctx(2), init_weights=False)
    logits = torch.zeros(1, 10)
    with pytest.raises(ValueError, match=r"2\*\*24"):
        head.distributed_argmax(logits, encoding="fp32")
    with pytest.raises(ValueError, match="unknown argmax encoding"):
        head.distributed_argmax(logits, encoding="bogus")


def test_loader_unknown_and_padding(tmp_path):
    from minitp_b200.synthetic import save_checkpoint
    from minitp_b200.weight_loader import load_qwen2_tp, load_synthetic_tp

    cfg = ModelConfig(64, 128, 1, 6, 2, 8, 50, 1e-6, 1e6, 64, True)  # 6 q heads: tp=4 needs padding
    with pytest.raises(ValueError, match="unknown loader"):
        load_qwen2_tp(str(tmp_path), cfg, _ctx(1), loader="bogus")
    save_checkpoint(cfg, str(tmp_path))
    full = load_qwen2_tp(str(tmp_path), cfg, _ctx(1))
    fw = full.model.layers[0].self_attn
    for r in range(4):
        m = load_qwen2_tp(str(tmp_path), cfg, _ctx(4, r), pad_heads=True)
        s = load_synthetic_tp(cfg, _ctx(4, r), dtype=torch.float32, device=torch.device("cpu"))
        for (k, a), (k2, b) in zip(m.state_dict().items(), s.state_dict().items()):
            assert k == k2 and torch.equal(a, b), k
        a = m.model.layers[0].self_attn
        assert a.q_heads_local == 2  # 6 heads/2 kv -> 3 per group -> padded to 4 -> 8 heads, 2 per rank
        hmap = m.cfg.padded_head_map()[r * 2:(r + 1) * 2]
        for j, head in enumerate(hmap):
            rows = a.qkv_proj.weight[j * 8:(j + 1) * 8]
            cols = a.o_proj.weight[:, j * 8:(j + 1) * 8]
            if head < 0:
                assert not rows.any() and not cols.any()
            else:
                assert torch.equal(rows, fw.qkv_proj.weight[head * 8:(head + 1) * 8])
                assert torch.equal(cols, fw.o_proj.weight[:, head * 8:(head + 1) * 8])


def test_synthetic_protocol_matches_fixture_prompt():
    from tests.conftest import golden
    from minitp_b200.synthetic import make_prompt

    g = golden("model_q05b_tp1_fp32.npz")
    assert np.array_equal(make_prompt(151936, 1, 128).numpy(), g["prompt"])


def test_launch_count_formula():
    from bench import launches_per_generation, prefill_launch_count

    # prefill: embed + 5 per layer + consume passes (2 per layer + final) + LM head
    assert prefill_launch_count(2, 1, True) == 1 + 10 + 4 + 1 + 1
    assert prefill_launch_count(2, 1, False) == 1 + 10 + 1
    assert prefill_launch_count(2, 3, True) == 3 * (1 + 10 + 4) + 1 + 1
    # then argmax (2), the position seed (1) and the decode steps
    assert launches_per_generation(17, 2, 1 + 10 + 2) == 17 + 2 + 1 + (1 + 10 + 2)
    # one decode megakernel launch per step
    assert launches_per_generation(17, 5, 1) == 17 + 2 + 1 + 4


def test_padded_heads_follow_the_source_tensors():
    """Zero rows of padded Q heads take the device and dtype of the checkpoint tensors
    (weights drawn on a GPU must not meet CPU zeros)."""
    from minitp_b200.weight_loader import _iter_layer_slices

    cfg = ModelConfig(64, 128, 1, 6, 2, 8, 50, 1e-6, 1e6, 64, True).padded_for(4)

    def get(name, kind, a, b):  # stand-in source: bf16 tensors of the right shapes
        shapes = {"model.embed_tokens.weight": (50, 64), "k_proj.weight": (16, 64), "v_proj.weight": (16, 64),
                  "k_proj.bias": (16,), "v_proj.bias": (16,), "q_proj.weight": (48, 64), "q_proj.bias": (48,),
                  "o_proj.weight": (64, 48), "gate_proj.weight": (128, 64), "up_proj.weight": (128, 64),
                  "down_proj.weight": (64, 128)}
        key = next((k for k in shapes if name.endswith(k)), None)
        full = torch.ones(shapes[key] if key else (64,), dtype=torch.bfloat16)
        if kind == "rows":
            return full[a:a + b]
        if kind == "cols":
            return full[:, a:a + b]
        return full

    padded = 0
    for r in range(4):
        for key, t in _iter_layer_slices(cfg, r, 4, get):
            assert t.dtype == torch.bfloat16, key
            if key.endswith("qkv_proj.weight"):
                padded += int((t == 0).all(dim=1).sum())
    assert padded > 0  # some rank holds zero (padded) head rows
