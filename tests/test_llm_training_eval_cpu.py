"""LLM training and evaluation properties (the checks of PredictiveCoding.UnitTests' LlmTrainingTests and
LlmEvalTests, restated for this package): schedule, clipping, Adam, dropout, gradient-averaging steps,
perplexity and the activation probe."""
import math

import pytest
import torch

from predicitivecoding_b200.llm import trainer
from predicitivecoding_b200.llm.eval import ActivationProbe, evaluate
from predicitivecoding_b200.llm.gpt import GptModel, TransformerConfig
from predicitivecoding_b200.models.config import DecoderLmConfig
from predicitivecoding_b200.models.decoder_lm import DecoderLM
from predicitivecoding_b200.optim.adam import Adam, LrSchedule, clip_global_norm


def tiny(**kw):
    base = dict(vocab=11, dim=16, num_blocks=2, num_heads=2, ff_dim=32, max_seq=8)
    base.update(kw)
    return DecoderLmConfig(**base)


WINDOWS = [([1, 2, 3, 4, 5, 6], [2, 3, 4, 5, 6, 7]), ([3, 4, 5, 6, 7, 8], [4, 5, 6, 7, 8, 9])]


def test_schedule_warms_up_then_decays_to_the_floor():
    s = LrSchedule(peak_lr=1.0, min_lr=0.1, warmup_steps=4, total_steps=20)
    warm = [s.at(i) for i in range(4)]
    assert warm == sorted(warm) and warm[-1] == pytest.approx(1.0)
    decay = [s.at(i) for i in range(4, 20)]
    assert decay == sorted(decay, reverse=True)
    assert s.at(25) == pytest.approx(0.1)


def test_clipping_bounds_the_global_norm_and_zeroes_non_finite():
    a = torch.zeros(3, requires_grad=True)
    b = torch.zeros(2, requires_grad=True)
    a.grad = torch.tensor([3.0, 4.0, float("nan")])
    b.grad = torch.tensor([0.0, float("inf")])
    norm = clip_global_norm([a, b], 1.0)
    assert norm == pytest.approx(5.0)
    total = math.sqrt(float((a.grad ** 2).sum() + (b.grad ** 2).sum()))
    assert total == pytest.approx(1.0) and torch.isfinite(a.grad).all() and torch.isfinite(b.grad).all()


def test_adam_decay_after_the_step_and_loss_goes_down():
    w = torch.tensor([2.0], requires_grad=True)
    opt = Adam(weight_decay=0.5)
    w.grad = torch.tensor([1.0])
    opt.step([w], 0.1)
    # step 1: mhat = 1, vhat = 1 -> w = 2 - 0.1 * 1 / (1 + eps); then decay w -= 0.1 * 0.5 * w
    expect = (2.0 - 0.1 / (1 + 1e-8)) * (1 - 0.05)
    assert float(w.detach()) == pytest.approx(expect, rel=1e-6)
    m = DecoderLM(tiny(), seed=1)
    opt = Adam()
    losses = []
    for _ in range(40):
        loss = m.loss(torch.tensor([WINDOWS[0][0]]), torch.tensor([WINDOWS[0][1]]))
        m.zero_grad()
        loss.backward()
        opt.step(list(m.parameters()), 1e-2)
        losses.append(float(loss.detach()))
    assert losses[-1] < 0.5 * losses[0]


def test_dropout_masks_in_training_and_is_identity_in_inference():
    m = DecoderLM(tiny(dropout=0.5), seed=2)
    x = torch.tensor([WINDOWS[0][0]])
    torch.manual_seed(0)
    a = m(x, training=True)
    torch.manual_seed(1)
    b = m(x, training=True)
    assert not torch.equal(a, b)
    assert torch.equal(m(x), m(x))
    loss = m.loss(x, torch.tensor([WINDOWS[0][1]]), training=True)
    loss.backward()
    assert all(p.grad is not None for p in m.parameters() if p.requires_grad and p is not m.plan)


def test_trainer_step_averages_window_gradients():
    m = DecoderLM(tiny(), seed=3)
    params = list(m.parameters())
    fn = lambda t, y, training: m.loss(t[None], y[None], training=training)
    # reference: mean of the per-window gradients
    grads = []
    for w in WINDOWS:
        m.zero_grad()
        fn(torch.tensor(w[0]), torch.tensor(w[1]), False).backward()
        grads.append([p.grad.clone() for p in params])
    mean = [sum(g[i] for g in grads) / len(grads) for i in range(len(params))]

    class Capture(Adam):
        def step(self, ps, lr):
            self.seen = [p.grad.clone() for p in ps]

    cap = Capture()
    loss = trainer.step(params, WINDOWS, fn, cap, 0.0, training=False)
    assert all(torch.allclose(a, b, atol=1e-6) for a, b in zip(cap.seen, mean))
    assert math.isfinite(loss)


def test_trainer_steps_reduce_the_loss():
    m = DecoderLM(tiny(), seed=4)
    params = list(m.parameters())
    fn = lambda t, y, training: m.loss(t[None], y[None], training=training)
    opt = Adam()
    first = trainer.step(params, WINDOWS, fn, opt, 1e-2, clip_norm=1.0)
    for _ in range(40):
        last = trainer.step(params, WINDOWS, fn, opt, 1e-2, clip_norm=1.0)
    assert last < 0.5 * first


def test_perplexity_of_a_zero_model_is_the_vocabulary_size():
    m = DecoderLM(tiny(), seed=5)
    with torch.no_grad():
        for p in m.parameters():
            p.zero_()
    r = evaluate(m, WINDOWS)
    assert r.perplexity == pytest.approx(11.0, rel=1e-5)


def test_perplexity_is_deterministic_and_skips_ignored_targets():
    m = DecoderLM(tiny(), seed=6)
    a, b = evaluate(m, WINDOWS), evaluate(m, WINDOWS)
    assert a.perplexity == b.perplexity and a.tokens == 12
    masked = [(WINDOWS[0][0], [-1, -1, 4, 5, 6, 7])]
    assert evaluate(m, masked).tokens == 4
    with pytest.raises(RuntimeError):
        evaluate(m, [(WINDOWS[0][0], [-1] * 6)])


def test_probe_records_blocks_and_sink_shares_and_changes_nothing():
    m = DecoderLM(tiny(), seed=7)
    x = torch.tensor([WINDOWS[0][0]])
    probe = ActivationProbe()
    with torch.no_grad():
        plain = m(x)
        probed = m(x, probe=probe)
    assert torch.allclose(plain, probed, atol=1e-6)
    assert set(probe.blocks) == {0, 1} and set(probe.sink_share) == {0, 1}
    assert all(0.0 <= v <= 1.0 for v in probe.sink_share.values())


def test_probe_on_gpt_step_records_one_entry_per_layer():
    g = GptModel(TransformerConfig(vocab_size=20, max_seq_len=16, embed_dim=16, num_heads=2, num_layers=3,
                                   feed_forward_dim=32), seed=1)
    cache = g.create_cache()
    probe = ActivationProbe()
    g.step(3, 0, cache, probe)
    assert set(probe.blocks) == {0, 1, 2}
