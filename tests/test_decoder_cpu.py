"""CPU oracle tests of the autograd decoder (reference numerics and config rules)."""
import json
import math

import pytest
import torch

from predicitivecoding_b200.models.config import DecoderLmConfig
from predicitivecoding_b200.models.decoder_lm import (DecoderLM, apply_rope, cross_entropy_masked, gelu_tanh,
                                                      mtp_targets, rms_norm, rope_tables)


def test_validate_rules():
    with pytest.raises(ValueError):
        DecoderLmConfig(10, 30, 1, 4, 8, 8).validate()  # dim % heads
    with pytest.raises(ValueError):
        DecoderLmConfig(10, 32, 2, 4, 8, 8, block_pattern="AX").validate()
    with pytest.raises(ValueError):
        DecoderLmConfig(10, 32, 2, 4, 8, 8, num_experts=2, moe_top_k=3).validate()
    with pytest.raises(ValueError):
        DecoderLmConfig(10, 32, 2, 4, 8, 8, use_rope=True, block_pattern="AT").validate()
    DecoderLmConfig.base(32000).validate()


def test_presets_and_parameter_formula():
    small = DecoderLmConfig.small(16384)
    assert (small.dim, small.num_blocks, small.num_heads, small.ff_dim) == (384, 8, 6, 1536)
    # the reference states 26.8M parameters for Small @ 16k (=16384) vocab and 135.3M for Base @ 32k
    # (DecoderLM.cs:96-100)
    assert abs(small.dense_parameter_formula() / 1e6 - 26.8) < 0.05
    assert abs(DecoderLmConfig.base(32768).dense_parameter_formula() / 1e6 - 135.3) < 0.1
    cfg = DecoderLmConfig(64, 32, 2, 2, 48, 16, use_rms_norm=True, use_rope=True)
    assert DecoderLM(cfg).parameter_count == cfg.dense_parameter_formula()


def test_config_json_roundtrip_pascal_case():
    cfg = DecoderLmConfig.small(16000)
    d = json.loads(cfg.to_json())
    assert d["Vocab"] == 16000 and d["UseRope"] is True and "Ffn" not in d
    assert DecoderLmConfig.from_json(cfg.to_json()) == cfg


def test_gelu_constants():
    x = torch.tensor([0.5, -1.0, 2.0])
    ref = [0.5 * v * (1 + math.tanh(0.7978845608 * (v + 0.044715 * v ** 3))) for v in x.tolist()]
    assert torch.allclose(gelu_tanh(x), torch.tensor(ref), atol=1e-6)


def test_rope_matches_reference_formula():
    S, hd = 5, 8
    x = torch.randn(S, hd)
    cos, sin = rope_tables(S, hd, base_pos=3)
    out = apply_rope(x, cos, sin)
    for r in range(S):
        for i in range(hd // 2):
            ang = (3 + r) * (1.0 / 10000 ** (2 * i / hd))
            x0, x1 = x[r, 2 * i].item(), x[r, 2 * i + 1].item()
            assert abs(out[r, 2 * i].item() - (x0 * math.cos(ang) - x1 * math.sin(ang))) < 1e-5
            assert abs(out[r, 2 * i + 1].item() - (x0 * math.sin(ang) + x1 * math.cos(ang))) < 1e-5


def test_rmsnorm_formula():
    x = torch.randn(3, 7)
    g = torch.rand(7)
    inv = 1 / torch.sqrt((x * x).sum(-1, keepdim=True) / 7 + 1e-5)
    assert torch.allclose(rms_norm(x, g, 1e-5), x * inv * g, atol=1e-6)


def test_masked_cross_entropy_mean_over_counted_rows():
    logits = torch.randn(4, 6)
    t = torch.tensor([1, -1, 3, -1])
    ref = (torch.nn.functional.cross_entropy(logits[[0, 2]], t[[0, 2]]))
    assert torch.allclose(cross_entropy_masked(logits, t, -1), ref)
    assert float(cross_entropy_masked(logits, torch.full((4,), -1), -1)) == 0.0


def test_mtp_targets_shift():
    t = torch.tensor([1, 2, 3, 4])
    assert mtp_targets(t, 2, -1).tolist() == [2, 3, 4, -1]


def test_every_mechanism_trains_a_step():
    cfg = DecoderLmConfig(64, 32, 2, 2, 64, 16, num_experts=3, moe_top_k=2, mtp_weight=0.3, use_plan=True,
                          num_loops=2)
    m = DecoderLM(cfg, seed=1)
    opt = torch.optim.AdamW(m.parameters(), lr=1e-2)
    t = torch.randint(0, 64, (4, 17), generator=torch.Generator().manual_seed(0))
    losses = []
    for _ in range(15):
        opt.zero_grad()
        loss = m.loss(t[:, :-1], t[:, 1:], training=True)
        loss.backward()
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < losses[0]
    # temporal 'T' blocks with LayerNorm + sinusoidal positions
    cfg_t = DecoderLmConfig(64, 32, 2, 2, 64, 16, block_pattern="AT")
    mt = DecoderLM(cfg_t)
    assert torch.isfinite(mt.loss(t[:, :-1], t[:, 1:]))


def test_reference_parameter_order_counts():
    cfg = DecoderLmConfig(64, 32, 2, 2, 48, 16)  # LayerNorm, GELU, 2 heads
    m = DecoderLM(cfg)
    ps = m.reference_parameters()
    # wemb + per block (g,b, 4 per head * 2 heads, g,b, w1,b1,w2,b2) + lnF g,b + wout
    assert len(ps) == 1 + 2 * (2 + 8 + 2 + 4) + 2 + 1
    assert ps[0].shape == (64, 32) and ps[-1].shape == (32, 64)
    assert ps[3].shape == (32, 16)  # block0 wq[0] [dim, head_dim]


def test_settle_plan_reduces_loss():
    cfg = DecoderLmConfig(32, 16, 1, 2, 32, 16, use_plan=True)
    m = DecoderLM(cfg, seed=2)
    trace = m.settle_plan(torch.randint(0, 32, (12,)), steps=5, lr=1.0)
    assert trace[-1] <= trace[0]
