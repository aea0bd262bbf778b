"""Predictive-coding layer, serializer and network edge cases (the properties of
PredictiveCoding.UnitTests/BugAndCrashTests.cs, restated for this package): serializer round trips and
size checks, precision updates, energies, clone depth, priors, input/label validation, inference traces,
concurrent use, MoE gates and temporal resets."""
import math
import threading

import pytest
import torch

from predicitivecoding_b200.io import layer_serializer as ser
from predicitivecoding_b200.pc.layer import Layer
from predicitivecoding_b200.pc.network import Network, NetworkConfig
from predicitivecoding_b200.pc.networks.moe import MixtureOfExperts, MixtureOfExpertsConfig, compute_gates
from predicitivecoding_b200.pc.networks.temporal import TemporalNetwork


def gen(seed=0):
    return torch.Generator().manual_seed(seed)


def layer(size=6, lower=4, act="tanh", seed=0):
    return Layer.create(1, size, lower, act, gen(seed))


# ---------------------------------------------------------------- serializer
def test_input_layer_round_trip():
    L = Layer.create(0, 5, 0, "tanh", gen(1))
    L.mu = torch.arange(5, dtype=torch.float32)
    back = ser.deserialize(ser.serialize(L), 0, "tanh")
    assert back.W is None and torch.equal(back.mu, L.mu)


def test_hidden_layer_round_trip():
    L = layer(seed=2)
    L.precision = 1.7
    back = ser.deserialize(ser.serialize(L), 1, "tanh")
    assert torch.equal(back.W, L.W) and torch.equal(back.b, L.b) and torch.equal(back.mu, L.mu)
    assert back.precision == pytest.approx(1.7)


def test_diagonal_precision_round_trip():
    L = layer(seed=3)
    L.init_diagonal_precision()
    L.diag_precision = torch.linspace(0.5, 2.0, L.size)
    back = ser.deserialize(ser.serialize(L), 1, "tanh")
    assert torch.equal(back.diag_precision, L.diag_precision)


@pytest.mark.parametrize("diag", [False, True])
@pytest.mark.parametrize("prior", [False, True])
def test_byte_length_matches_the_serialized_size(diag, prior):
    L = layer(seed=4)
    if diag:
        L.init_diagonal_precision()
    if prior:
        L.prior_mean = torch.ones(L.size)
    assert len(ser.serialize(L)) == ser.byte_length(L.size, L.lower_size, diag, prior)


def test_truncated_record_is_rejected():
    buf = ser.serialize(layer(seed=5))
    with pytest.raises(Exception):
        ser.deserialize(buf[:-7], 1, "tanh")


# ---------------------------------------------------------------- layer dynamics
def test_diagonal_precision_update_needs_init():
    with pytest.raises(RuntimeError):
        layer().update_diagonal_precision(0.1)


def test_diagonal_precision_stays_positive():
    L = layer()
    L.init_diagonal_precision()
    L.eps = torch.full((L.size,), 100.0)      # huge residual: the gradient pushes Pi far below 0
    L.update_diagonal_precision(10.0)
    assert bool((L.diag_precision > 0).all())


def test_energy_with_zero_diagonal_precision_is_finite():
    L = layer()
    L.init_diagonal_precision()
    L.diag_precision[::2] = 0.0
    L.eps = torch.randn(L.size)
    e = L.local_energy()
    assert math.isfinite(e) and e >= 0


def test_clone_is_deep():
    L = layer()
    c = L.clone()
    c.W += 1.0
    c.mu += 1.0
    assert not torch.equal(c.W, L.W) and not torch.equal(c.mu, L.mu)


def test_scalar_precision_is_clamped():
    L = layer()
    L.eps = torch.full((L.size,), 1e-6)
    for _ in range(100):
        L.update_precision(100.0)
    assert L.precision >= 1e-6


def test_top_layer_error_uses_the_prior_mean():
    L = layer()
    L.prior_mean = torch.full((L.size,), 0.25)
    L.set_prediction_error(None)
    assert torch.allclose(L.eps, L.mu - 0.25)
    L.prior_mean = None
    L.set_prediction_error(None)
    assert bool((L.eps == 0).all())


def test_temporal_prior_pulls_the_state_toward_the_previous_one():
    L = layer()
    L.eps = torch.zeros(L.size)
    L.temporal_prior = torch.full((L.size,), 1.0)
    L.temporal_precision = 1.0
    before = float((L.mu - 1.0).abs().sum())
    L.update_state(None, 0.1)
    assert float((L.mu - 1.0).abs().sum()) < before


def test_weight_decay_shrinks_the_weights():
    L = layer()
    L.weight_decay = 0.5
    L.compute_prediction()
    before = L.weight_norm()
    L.update_weights(torch.zeros(L.lower_size), 0.1)   # no error: only the decay acts
    assert L.weight_norm() < before


# ---------------------------------------------------------------- network API
def net(**kw):
    base = dict(layer_sizes=(6, 12, 3))
    base.update(kw)
    return Network(NetworkConfig(**base), seed=1)


def test_wrong_sizes_raise():
    n = net()
    with pytest.raises(ValueError):
        n.learn(torch.zeros(5), torch.zeros(3), 5)
    with pytest.raises(ValueError):
        n.learn(torch.zeros(6), torch.zeros(4), 5)
    with pytest.raises(ValueError):
        n.infer(torch.zeros(7), 5)
    with pytest.raises(ValueError):
        n.predict(torch.zeros(2), 5)


def test_zero_step_trace_is_empty():
    assert net().infer_trace(torch.zeros(6), 0) == []


def test_trace_decreases_after_training():
    n = net(layer_sizes=(4, 8, 2), state_lr=0.05)
    x, y = torch.tensor([0.5, -0.2, 0.1, 0.3]), torch.tensor([1.0, 0.0])
    for _ in range(50):
        n.learn(x, y, 10)
    trace = n.infer_trace(x, 15)
    assert all(b <= a + 1e-6 for a, b in zip(trace, trace[1:]))


def test_close_twice_is_harmless():
    n = net()
    n.close()
    n.close()


def test_diagonal_precision_training_keeps_weights_finite():
    n = net(use_diagonal_precision=True)
    g = gen(7)
    for _ in range(30):
        n.learn(torch.randn(6, generator=g), torch.eye(3)[int(torch.randint(0, 3, (1,), generator=g))], 8)
    assert math.isfinite(n.average_weight_norm())


def test_concurrent_learn_and_predict_finish():
    n = net()
    errors = []

    def learner():
        try:
            for _ in range(20):
                n.learn(torch.rand(6), torch.eye(3)[0], 4)
        except Exception as e:      # pragma: no cover - surfaced below
            errors.append(e)

    def reader():
        try:
            for _ in range(20):
                n.predict(torch.rand(6), 4)
        except Exception as e:      # pragma: no cover
            errors.append(e)

    ts = [threading.Thread(target=learner), threading.Thread(target=reader), threading.Thread(target=reader)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=60)
    assert not any(t.is_alive() for t in ts) and not errors


def test_single_layer_and_negative_rates_are_rejected():
    with pytest.raises(ValueError):
        NetworkConfig(layer_sizes=(4,)).validate()
    with pytest.raises(ValueError):
        NetworkConfig(state_lr=-0.1).validate()
    with pytest.raises(ValueError):
        NetworkConfig(layer_sizes=(6, 4, 2), input_shape=(2, 2)).validate()


# ---------------------------------------------------------------- MoE gates and temporal resets
def test_gates_of_equal_energies_are_uniform():
    g = compute_gates([0.0, 0.0, 0.0, 0.0], 1.0)
    assert all(abs(x - 0.25) < 1e-12 for x in g)
    g0 = compute_gates([1.0, 5.0, 9.0], 0.0)          # temperature 0: no preference
    assert all(abs(x - 1 / 3) < 1e-12 for x in g0)


def test_gates_stay_finite_at_extreme_temperatures_and_floors_sum_to_one():
    g = compute_gates([1.0, 2.0, 1e6], 1e9)
    assert all(math.isfinite(x) for x in g) and abs(sum(g) - 1) < 1e-9
    f = compute_gates([0.0, 100.0, 100.0], 10.0, min_gate=0.05)
    assert abs(sum(f) - 1) < 1e-9 and min(f) >= 0.05 / (1 + 2 * 0.05) - 1e-12


def test_moe_energies_finite_after_learning():
    cfg = MixtureOfExpertsConfig(expert_count=3, expert_config=NetworkConfig(layer_sizes=(4, 8, 2)))
    moe = MixtureOfExperts(cfg, seed=3)
    for _ in range(10):
        moe.learn(torch.rand(4), torch.tensor([1.0, 0.0]), 5)
    pred = moe.predict_detailed(torch.rand(4), 5)
    assert all(math.isfinite(e) for e in pred.expert_energies)


def test_temporal_reset_clears_the_prior():
    tn = TemporalNetwork(net(), temporal_precision=1.0)
    tn.predict(torch.rand(6), 3)                # before any step: no prior, no crash
    tn.step(torch.rand(6), torch.eye(3)[1], 3)
    assert tn.has_prior
    tn.reset()
    assert not tn.has_prior
