"""DecoderLM mechanisms, property by property (the checks of PredictiveCoding.UnitTests' LlmLoopedTests,
LlmMtpTests, LlmPlanTests and LlmHybridTests, restated for this model)."""
import pytest
import torch

from predicitivecoding_b200.llm.eval import ActivationProbe
from predicitivecoding_b200.models.config import DecoderLmConfig
from predicitivecoding_b200.models.decoder_lm import DecoderLM, mtp_targets, recurrent_scan


def cfg(**kw):
    base = dict(vocab=17, dim=16, num_blocks=2, num_heads=2, ff_dim=32, max_seq=12, use_rms_norm=True,
                use_rope=True)
    base.update(kw)
    return DecoderLmConfig(**base)


TOK = torch.tensor([[1, 2, 3, 4, 5, 6, 7, 8]])
TGT = torch.tensor([[2, 3, 4, 5, 6, 7, 8, 9]])


def train(m, steps=60, lr=1e-2):
    opt = torch.optim.Adam(m.parameters(), lr=lr)
    losses = []
    for _ in range(steps):
        loss = m.loss(TOK, TGT, training=True)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    return losses


# ---------------------------------------------------------------- looped blocks
def test_one_loop_is_the_default_with_no_extra_parameters():
    a, b = DecoderLM(cfg(), seed=1), DecoderLM(cfg(num_loops=1), seed=1)
    assert a.parameter_count == b.parameter_count and a.loop_bias is None
    assert torch.equal(a(TOK), b(TOK))


def test_invalid_loop_configs_raise():
    with pytest.raises(ValueError):
        cfg(num_loops=0).validate()
    with pytest.raises(ValueError):
        cfg(loop_exit_tau=-0.1).validate()


def test_tied_loop_gradient_is_the_sum_over_passes():
    """Two passes through the same blocks: a block weight's gradient equals the sum of the gradients of
    two untied copies, one per pass."""
    m = DecoderLM(cfg(num_loops=2), seed=2).double()
    blk = m.blocks[0]
    g_tied = torch.autograd.grad(m.loss(TOK, TGT), [blk.wq])[0]
    w = blk.wq.detach().clone()
    w1, w2 = w.clone().requires_grad_(True), w.clone().requires_grad_(True)
    del blk._parameters["wq"]
    calls = []

    def untie(module, args):
        module.wq = w1 if not calls else w2
        calls.append(1)

    handle = blk.register_forward_pre_hook(untie)
    g1, g2 = torch.autograd.grad(m.loss(TOK, TGT), [w1, w2])
    handle.remove()
    assert len(calls) == 2
    assert torch.allclose(g_tied, g1 + g2, atol=1e-10, rtol=1e-8)


def test_looped_model_learns():
    losses = train(DecoderLM(cfg(num_loops=2), seed=3))
    assert losses[-1] < 0.5 * losses[0]


def test_early_exit_threshold_zero_runs_every_pass():
    m = DecoderLM(cfg(num_loops=3, loop_exit_tau=0.0), seed=4)
    probe = ActivationProbe()
    m.hidden(TOK, probe=probe)
    assert probe.loops_used == 3
    m2 = DecoderLM(cfg(num_loops=3, loop_exit_tau=1e6), seed=4)   # any change counts as converged
    probe2 = ActivationProbe()
    m2.hidden(TOK, probe=probe2)
    assert probe2.loops_used == 2                                    # needs two passes to compare


# ---------------------------------------------------------------- multi-token prediction
def test_mtp_off_matches_the_plain_model():
    a, b = DecoderLM(cfg(), seed=5), DecoderLM(cfg(mtp_weight=0.0), seed=5)
    assert len(a.reference_parameters()) == len(b.reference_parameters())
    assert torch.equal(a.loss(TOK, TGT), b.loss(TOK, TGT))


def test_mtp_on_adds_exactly_one_head_tensor():
    a, b = DecoderLM(cfg(), seed=6), DecoderLM(cfg(mtp_weight=0.3), seed=6)
    assert len(b.reference_parameters()) == len(a.reference_parameters()) + 1
    assert b.wout_mtp.shape == (16, 17)


def test_mtp_targets_shift_into_the_future_and_mask_the_tail():
    t = torch.tensor([[10, 11, 12, 13, 14]])
    out = mtp_targets(t, 2, -1)
    assert out.tolist() == [[11, 12, 13, 14, -1]]
    out3 = mtp_targets(t, 3, -1)
    assert out3.tolist() == [[12, 13, 14, -1, -1]]


def test_mtp_training_lowers_both_heads():
    m = DecoderLM(cfg(mtp_weight=0.5), seed=7)
    with torch.no_grad():
        main0, mtp0 = m.heads(TOK)
    train(m)
    with torch.no_grad():
        main1, mtp1 = m.heads(TOK)
    ce = torch.nn.functional.cross_entropy
    fut = mtp_targets(TGT, 2, -1)
    assert float(ce(main1[0], TGT[0])) < float(ce(main0[0], TGT[0]))
    assert float(ce(mtp1[0], fut[0], ignore_index=-1)) < float(ce(mtp0[0], fut[0], ignore_index=-1))


# ---------------------------------------------------------------- latent plan
def test_zero_plan_leaves_the_forward_unchanged():
    a, b = DecoderLM(cfg(), seed=8), DecoderLM(cfg(use_plan=True), seed=8)
    assert torch.equal(a(TOK), b(TOK))


def test_plan_api_validates():
    m = DecoderLM(cfg(), seed=9)
    with pytest.raises(RuntimeError):
        m.settle_plan(TOK[0], 3, 0.1)
    p = DecoderLM(cfg(use_plan=True), seed=9)
    with pytest.raises(ValueError):
        p.settle_plan(TOK[0, :1], 3, 0.1)
    with pytest.raises(ValueError):
        p.settle_plan(TOK[0], 0, 0.1)


def test_settling_descends_the_prompt_loss_and_moves_only_the_plan():
    m = DecoderLM(cfg(use_plan=True), seed=10)
    before = {n: p.detach().clone() for n, p in m.named_parameters() if n != "plan"}
    trace = m.settle_plan(torch.tensor([1, 2, 3, 4, 5, 6, 7, 8, 9]), 20, 0.5)
    assert trace[-1] < trace[0]
    assert float(m.plan.abs().sum()) > 0
    for n, p in m.named_parameters():
        if n != "plan":
            assert torch.equal(p, before[n]), n


# ---------------------------------------------------------------- hybrid (attention + temporal blocks)
def test_all_attention_pattern_is_identical_to_no_pattern():
    a = DecoderLM(cfg(use_rms_norm=False, use_rope=False), seed=11)
    b = DecoderLM(cfg(use_rms_norm=False, use_rope=False, block_pattern="AA"), seed=11)
    assert torch.equal(a(TOK), b(TOK))


def test_block_pattern_validation():
    with pytest.raises(ValueError):
        cfg(use_rms_norm=False, use_rope=False, block_pattern="A").validate()      # wrong length
    with pytest.raises(ValueError):
        cfg(use_rms_norm=False, use_rope=False, block_pattern="AX").validate()     # unknown letter
    with pytest.raises(ValueError):
        cfg(block_pattern="AT").validate()                                         # RMSNorm/RoPE are attention-only


def test_gated_recurrent_scan_gradients():
    a = torch.rand(2, 5, 3, dtype=torch.float64, requires_grad=True)
    b = torch.randn(2, 5, 3, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(recurrent_scan, (a, b))
    s = recurrent_scan(a, b)
    ref = torch.zeros(2, 3, dtype=torch.float64)
    for t in range(5):
        ref = a[:, t] * ref + b[:, t]
        assert torch.allclose(s[:, t], ref)


def test_pure_temporal_model_learns_to_echo_the_previous_token():
    """Target t = token t-1 with no attention at all: the recurrent state must carry the previous token."""
    c = DecoderLmConfig(13, 16, 2, 1, 32, 8, block_pattern="TT")
    m = DecoderLM(c, seed=4)
    toks = torch.tensor([5, 2, 7, 3, 9, 4])
    tgts = torch.tensor([-1, 5, 2, 7, 3, 9])
    opt = torch.optim.Adam(m.parameters(), lr=1e-2)
    first = float(m.loss(toks, tgts, ignore_index=-1))
    for _ in range(250):
        loss = m.loss(toks, tgts, ignore_index=-1, training=True)
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert float(m.loss(toks, tgts, ignore_index=-1)) < 0.4 * first
