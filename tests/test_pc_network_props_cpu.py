"""Predictive-coding network, layer and activation properties (the checks of PredictiveCoding.UnitTests'
NetworkTests, PCLayerTests and ActivationFnTests, restated for this package)."""
import math

import pytest
import torch

from predicitivecoding_b200.pc.layer import Layer, activate, derivative, softmax
from predicitivecoding_b200.pc.network import Network, NetworkConfig


def net(sizes=(6, 12, 8, 3), seed=1, **kw):
    return Network(NetworkConfig(layer_sizes=sizes, **kw), seed=seed)


PATTERNS = [(torch.tensor([1.0, 0.9, 0.8, 0.0, 0.1, 0.0]), 0),
            (torch.tensor([0.0, 0.1, 0.0, 1.0, 0.9, 0.8]), 1),
            (torch.tensor([0.5, 0.0, 0.5, 0.0, 0.5, 0.0]), 2)]


def train(n, epochs=60, steps=10, mixed=False):
    for _ in range(epochs):
        for x, c in PATTERNS:
            n.learn(x, torch.eye(3)[c], steps, mixed=mixed)


# ---------------------------------------------------------------- activations
def test_activations_values():
    x = torch.tensor([-2.0, 0.0, 1.5])
    assert torch.equal(activate(x, "linear"), x)
    assert torch.allclose(activate(x, "tanh"), torch.tanh(x))
    assert activate(x, "relu").tolist() == [0.0, 0.0, 1.5]
    s = activate(x, "sigmoid")
    assert bool(((s > 0) & (s < 1)).all())


def test_activation_derivatives():
    pre = torch.tensor([-1.0, 0.5, 2.0])
    assert torch.equal(derivative(pre, activate(pre, "linear"), "linear"), torch.ones(3))
    t = activate(pre, "tanh")
    assert torch.allclose(derivative(pre, t, "tanh"), 1 - t * t)
    assert derivative(pre, activate(pre, "relu"), "relu").tolist() == [0.0, 1.0, 1.0]
    s = activate(pre, "sigmoid")
    assert torch.allclose(derivative(pre, s, "sigmoid"), s * (1 - s))


def test_softmax_sums_to_one_and_keeps_the_order():
    p = softmax(torch.tensor([0.3, 2.0, -1.0]))
    assert float(p.sum()) == pytest.approx(1.0) and int(p.argmax()) == 1


# ---------------------------------------------------------------- layer
def test_input_layer_has_no_weights_hidden_layer_has_both():
    g = torch.Generator().manual_seed(0)
    inp = Layer.create(0, 4, 0, "tanh", g)
    hid = Layer.create(1, 4, 3, "tanh", g)
    assert inp.W is None and inp.b is None
    assert hid.W.shape == (3, 4) and hid.b.shape == (3,)


def test_linear_prediction_is_a_matvec_plus_bias():
    L = Layer.create(1, 3, 2, "linear", torch.Generator().manual_seed(0))
    L.W = torch.tensor([[1.0, 2.0, 3.0], [0.0, -1.0, 0.5]])
    L.b = torch.tensor([0.5, -0.5])
    L.mu = torch.tensor([1.0, 1.0, 2.0])
    L.compute_prediction()
    assert L.pred.tolist() == [9.5, -0.5]


def test_prediction_error_and_energy():
    L = Layer.create(1, 3, 0, "tanh", torch.Generator().manual_seed(0))
    L.mu = torch.tensor([1.0, 2.0, 3.0])
    L.set_prediction_error(torch.tensor([0.5, 2.0, 1.0]))
    assert L.eps.tolist() == [0.5, 0.0, 2.0]
    assert L.local_energy() == pytest.approx(0.5 * (0.25 + 4.0))


def test_clamped_state_does_not_move():
    L = Layer.create(1, 3, 2, "tanh", torch.Generator().manual_seed(0))
    L.is_clamped = True
    mu = L.mu.clone()
    L.eps = torch.ones(3)
    L.update_state(torch.ones(2), 0.5)
    assert torch.equal(L.mu, mu)


# ---------------------------------------------------------------- network
def test_layer_count_energies_and_weights_after_construction():
    n = net()
    assert n.layer_count == 4
    assert n.compute_energy() >= 0
    es = n.compute_layer_energies()
    assert len(es) in (n.layer_count - 1, n.layer_count) and all(e >= 0 for e in es)
    assert n.average_weight_norm() > 0


def test_inference_is_transient():
    n = net()
    before = [n.layer(i).W.clone() for i in range(1, n.layer_count)]
    n.infer(PATTERNS[0][0], 20)
    assert all(torch.equal(b, n.layer(i + 1).W) for i, b in enumerate(before))


def test_learning_changes_weights_and_lowers_the_energy():
    n = net()
    x, c = PATTERNS[0]
    w0 = n.layer(1).W.clone()
    energies = [n.learn(x, torch.eye(3)[c], 10) for _ in range(30)]
    assert not torch.equal(w0, n.layer(1).W)
    assert energies[-1] <= energies[0] + 1e-6


def test_prediction_is_valid_and_deterministic():
    n = net()
    train(n, epochs=5)
    p = [n.predict(PATTERNS[1][0], 15) for _ in range(3)]
    assert p[0] in (0, 1, 2) and p.count(p[0]) == 3


def _separable(mixed=False):
    n = Network(NetworkConfig(layer_sizes=(4, 16, 2), state_lr=0.2, weight_lr=0.05), seed=0)
    x0, x1 = torch.zeros(4), torch.ones(4)
    for _ in range(200):
        n.learn(x0, torch.eye(2)[0], 10, mixed=mixed)
        n.learn(x1, torch.eye(2)[1], 10, mixed=mixed)
    return n, x0, x1


def test_repeated_learning_separates_linearly_separable_patterns():
    n, x0, x1 = _separable()
    assert n.predict(x0, 20) == 0 and n.predict(x1, 20) == 1


def test_feedforward_gist_start_is_finite_and_lowers_the_early_energy():
    cold = Network(NetworkConfig(layer_sizes=(4, 16, 2), state_lr=0.15, weight_lr=0.05), seed=7)
    warm = Network(NetworkConfig(layer_sizes=(4, 16, 2), state_lr=0.15, weight_lr=0.05,
                                 use_feedforward_gist_init=True), seed=7)
    x, y = torch.tensor([1.0, 0.0, 0.0, 1.0]), torch.eye(2)[0]
    for _ in range(50):
        cold.learn(x, y, 20)
        warm.learn(x, y, 20)
    cold.infer(x, 3, clamp_top=True, label=y)
    warm.infer(x, 3, clamp_top=True, label=y)
    assert math.isfinite(warm.compute_energy())
    assert warm.compute_energy() <= cold.compute_energy() + 1e-3


def test_activity_regularisation_trains_and_settles():
    n = net(activity_regularization=0.01)
    train(n, epochs=10)
    trace = n.infer_trace(PATTERNS[2][0], 20)
    assert all(math.isfinite(e) for e in trace) and trace[-1] <= trace[0] + 1e-6
    with pytest.raises(ValueError):
        NetworkConfig(activity_regularization=-0.1).validate()


def test_mixed_precision_inference_tracks_fp32():
    n = net()
    train(n, epochs=30)
    x = PATTERNS[0][0]
    a = n.infer_get_top(x, 20, reset_state=True)
    b = n.infer_get_top(x, 20, reset_state=True, mixed=True)
    assert float((a - b).abs().max()) < 5e-2 * max(1.0, float(a.abs().max()))
    ef, eh = n.class_energies(x, 15), n.class_energies(x, 15, mixed=True)
    assert int(torch.tensor(ef).argmin()) == int(torch.tensor(eh).argmin())


def test_mixed_precision_leaves_the_fp32_masters_untouched_and_learns():
    n = net()
    w = [n.layer(i).W.clone() for i in range(1, n.layer_count)]
    n.infer_mixed(PATTERNS[0][0], 10)
    assert all(torch.equal(a, n.layer(i + 1).W) for i, a in enumerate(w))
    m, x0, x1 = _separable(mixed=True)
    assert m.predict(x0, 20, mixed=True) == 0 and m.predict(x1, 20, mixed=True) == 1
