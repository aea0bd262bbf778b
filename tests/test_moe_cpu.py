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


# ---- DecoderLM MoE semantics (the properties PredictiveCoding.UnitTests/LlmMoeTests.cs and
# LlmMoeSparseTests.cs check on the reference)
from predicitivecoding_b200.llm.eval import ActivationProbe


def tiny_moe(**kw):
    base = dict(vocab=13, dim=16, num_blocks=2, num_heads=2, ff_dim=32, max_seq=8, use_rms_norm=True,
                use_rope=True, num_experts=4, moe_top_k=1)
    base.update(kw)
    return DecoderLmConfig(**base)


def test_invalid_moe_configs_raise():
    import pytest
    for kw in (dict(num_experts=4, moe_top_k=0), dict(num_experts=4, moe_top_k=5), dict(num_experts=-1)):
        with pytest.raises(ValueError):
            tiny_moe(**kw).validate()


def test_dense_model_counts_every_parameter_as_active():
    m = DecoderLM(tiny_moe(num_experts=0), seed=1)
    assert m.active_parameter_count_per_token == m.parameter_count


def test_active_parameters_count_only_the_routed_experts():
    cfg = tiny_moe(num_experts=4, moe_top_k=1)
    m = DecoderLM(cfg, seed=1)
    per_expert = cfg.dim * cfg.ff_dim + cfg.ff_dim + cfg.ff_dim * cfg.dim + cfg.dim
    assert m.active_parameter_count_per_token == m.parameter_count - cfg.num_blocks * 3 * per_expert
    every = DecoderLM(tiny_moe(num_experts=4, moe_top_k=4), seed=1)
    assert every.active_parameter_count_per_token == every.parameter_count


def test_uniform_router_balance_loss_is_one_per_block():
    cfg = tiny_moe(moe_balance_weight=0.5, num_experts=4, moe_top_k=2)
    m = DecoderLM(cfg, seed=2)
    with torch.no_grad():
        for blk in m.blocks:
            blk.router.zero_()                  # uniform gates: every expert 1/E
    tok = torch.tensor([[1, 2, 3, 4, 5, 6, 7, 8]])
    tgt = torch.tensor([[2, 3, 4, 5, 6, 7, 8, 9]])
    with_balance = float(m.loss(tok, tgt))
    aux = []
    main, _ = m.heads(tok, False, None, aux)
    without = float(torch.nn.functional.cross_entropy(main.reshape(-1, cfg.vocab), tgt.reshape(-1)))
    # E * sum_e (1/E) * frac_e = sum_e frac_e = 1 per block, whatever the (tie-broken) routing
    assert abs(with_balance - without - 0.5 * cfg.num_blocks) < 1e-4


def test_only_routed_rows_run_through_experts():
    for k in (1, 2, 4):
        cfg = tiny_moe(num_experts=4, moe_top_k=k, num_blocks=1)
        m = DecoderLM(cfg, seed=3)
        probe = ActivationProbe()
        tok = torch.tensor([[1, 2, 3, 4]])
        m.hidden(tok, probe=probe)
        assert probe.moe_rows_computed == 4 * k      # rows * k, not rows * E


def test_moe_ffn_gradients_match_finite_differences():
    cfg = tiny_moe(num_experts=3, moe_top_k=2, num_blocks=1)
    blk = DecoderLM(cfg, seed=4).blocks[0].double()
    x = torch.randn(1, 5, cfg.dim, dtype=torch.float64, requires_grad=True)

    def f(inp):
        aux = []
        y = blk.moe_ffn(inp, aux)
        return (y * torch.linspace(-1, 1, y.numel(), dtype=torch.float64).view_as(y)).sum() + 0.3 * aux[0]

    # the routing is piecewise constant: small steps keep every row on its experts
    assert torch.autograd.gradcheck(f, (x,), eps=1e-6, atol=1e-5, rtol=1e-4)
    params = [blk.router, blk.ew1[0], blk.eb2[1]]
    out = f(x)
    grads = torch.autograd.grad(out, params)
    for p, g in zip(params, grads):
        idx = (0,) * p.dim()
        with torch.no_grad():
            old = p[idx].item()
            p[idx] = old + 1e-6
            up = float(f(x))
            p[idx] = old - 1e-6
            dn = float(f(x))
            p[idx] = old
        assert abs((up - dn) / 2e-6 - float(g[idx])) < 1e-5 * max(1.0, abs(float(g[idx])))


def test_moe_model_learns_a_fixed_sequence():
    cfg = tiny_moe(num_experts=4, moe_top_k=2, num_blocks=1, moe_balance_weight=0.01)
    torch.manual_seed(0)
    m = DecoderLM(cfg, seed=5)
    opt = torch.optim.Adam(m.parameters(), lr=1e-2)
    tok = torch.tensor([[1, 2, 3, 4, 5, 6, 7, 8]])
    tgt = torch.tensor([[2, 3, 4, 5, 6, 7, 8, 9]])
    first = None
    for _ in range(60):
        loss = m.loss(tok, tgt, training=True)
        first = float(loss) if first is None else first
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert float(loss) < 0.5 * first
