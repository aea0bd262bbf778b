"""The 16-column gate/up interleave that the fused SwiGLU decode projection reads (pure tensor layout)."""
import pytest
import torch

from predicitivecoding_b200 import ops


def test_interleave16_alternates_blocks_of_sixteen():
    K, F = 3, 48
    gate = torch.arange(K * F, dtype=torch.float32).view(K, F)
    up = -gate - 1
    w = ops.interleave16(gate, up)
    assert w.shape == (K, 2 * F)
    for blk in range(F // 16):
        assert torch.equal(w[:, 32 * blk:32 * blk + 16], gate[:, 16 * blk:16 * blk + 16])
        assert torch.equal(w[:, 32 * blk + 16:32 * blk + 32], up[:, 16 * blk:16 * blk + 16])


def test_interleave16_product_matches_separate_gate_and_up():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(5, 8, generator=g)
    gate, up = torch.randn(8, 32, generator=g), torch.randn(8, 32, generator=g)
    y = x @ ops.interleave16(gate, up)
    # feature f: gate column (f // 16) * 32 + f % 16, up column 16 further
    f = torch.arange(32)
    gi = (f // 16) * 32 + f % 16
    assert torch.allclose(y[:, gi], x @ gate, atol=1e-5)
    assert torch.allclose(y[:, gi + 16], x @ up, atol=1e-5)


def test_interleave16_rejects_widths_not_multiple_of_16():
    with pytest.raises(ValueError):
        ops.interleave16(torch.zeros(2, 24), torch.zeros(2, 24))
