"""Mixture-of-experts: the layout the device kernels read against the autograd DecoderLM's MoE FFN
(DecoderLM.cs:556-615 semantics), and the shape rules of the device path."""
import torch

from predicitivecoding_b200.models.config import DecoderLmConfig
from predicitivecoding_b200.models.decoder_lm import DecoderLM
from predicitivecoding_b200.ops import moe
from predicitivecoding_b200.engine import fused_trainer


def moe_cfg(**kw):
    base = dict(vocab=64, dim=256, num_blocks=1, num_heads=4, ff_dim=512, max_seq=128, use_rms_norm=True,
                use_rope=True, num_experts=4, moe_top_k=2)
    base.update(kw)
    return DecoderLmConfig(**base)


def kernel_layout(blk, cfg):
    """DecoderLM block weights -> router [E, D], w1 [E*F, D], b1 [E*F], w2 [E*D, F], b2 [E*D]."""
    E = cfg.num_experts
    router = blk.router.detach().T.contiguous()
    w1 = torch.cat([blk.ew1[e].detach().T for e in range(E)], 0)
    b1 = torch.cat([blk.eb1[e].detach() for e in range(E)], 0)
    w2 = torch.cat([blk.ew2[e].detach().T for e in range(E)], 0)
    b2 = torch.cat([blk.eb2[e].detach() for e in range(E)], 0)
    return router, w1, b1, w2, b2


def test_capacity_and_supported():
    assert moe.capacity(256, 2, 4) % moe.SEG == 0
    assert moe.capacity(256, 2, 4) >= 256 * 2 + 4 * 255
    assert moe.supported(256, 512, 4, 2)
    assert not moe.supported(200, 512, 4, 2)       # tiles would straddle experts
    assert not moe.supported(256, 512, 4, 5)       # top-k above E
    assert not moe.supported(256, 512, 65, 2)
    assert fused_trainer.supports(moe_cfg())
    assert not fused_trainer.supports(moe_cfg(dim=192, num_heads=3))


def test_reference_matches_decoder_lm_moe_ffn():
    cfg = moe_cfg()
    model = DecoderLM(cfg, seed=5)
    blk = model.blocks[0]
    with torch.no_grad():
        for e in range(cfg.num_experts):
            blk.eb1[e].normal_(0, 0.1)
            blk.eb2[e].normal_(0, 0.1)
    x = torch.randn(2, 16, cfg.dim)
    aux = []
    want = blk.moe_ffn(x, aux)
    router, w1, b1, w2, b2 = kernel_layout(blk, cfg)
    got, bal, topi = moe.reference(x.view(-1, cfg.dim), router, w1, b1, w2, b2, cfg.moe_top_k)
    assert torch.allclose(got.view_as(want), want, atol=1e-5, rtol=1e-4)
    assert abs(float(bal.detach()) - float(aux[0].detach())) < 1e-5
    assert topi.shape == (32, 2)


def test_reference_gradients_flow_to_router_through_gates_and_balance():
    cfg = moe_cfg()
    blk = DecoderLM(cfg, seed=1).blocks[0]
    router, w1, b1, w2, b2 = [t.clone().requires_grad_(True) for t in kernel_layout(blk, cfg)]
    x = torch.randn(24, cfg.dim)
    y, bal, _ = moe.reference(x, router, w1, b1, w2, b2, 2)
    (y.square().mean() + 0.01 * bal).backward()
    assert router.grad is not None and float(router.grad.abs().sum()) > 0
    # only routed experts get weight gradients; every expert's block has the right shape
    assert w1.grad.shape == w1.shape and w2.grad.shape == w2.shape
