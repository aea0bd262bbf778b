"""The advanced PC architectures on the CPU: construction, learning and each one's defining behaviour."""
import torch
import pytest

from predicitivecoding_b200.pc.network import Network, NetworkConfig
from predicitivecoding_b200.pc import networks as nw

torch.manual_seed(0)
CFG = NetworkConfig(layer_sizes=(6, 12, 3), state_lr=0.1, weight_lr=0.02)


def _data(n=24, seed=0):
    g = torch.Generator().manual_seed(seed)
    protos = torch.randn(3, 6, generator=g)
    xs, ys = [], []
    for i in range(n):
        c = i % 3
        xs.append(protos[c] + 0.05 * torch.randn(6, generator=g))
        ys.append(torch.eye(3)[c])
    return xs, ys


def _train_acc(model, epochs=25, steps=10):
    xs, ys = _data()
    for _ in range(epochs):
        for x, y in zip(xs, ys):
            model.learn(x, y, steps)
    return sum(model.predict(x, steps) == int(y.argmax()) for x, y in zip(xs, ys)) / len(xs)


def test_moe_gates_and_learning():
    g = nw.compute_gates([1.0, 2.0, 3.0], 1.0, 0.05)
    assert abs(sum(g) - 1) < 1e-6 and g[0] > g[1] > g[2] >= 0.05 / 1.2
    moe = nw.MixtureOfExperts(nw.MixtureOfExpertsConfig(expert_count=2, expert_config=CFG))
    assert _train_acc(moe) >= 0.9


def test_ensemble_learns():
    ens = nw.EnsembleNetwork(nw.EnsembleConfig(member_configs=[CFG, CFG]))
    assert _train_acc(ens) >= 0.9


def test_attentive_gates_move_and_learn():
    net = nw.AttentiveNetwork(nw.AttentiveNetworkConfig(base_config=CFG))
    assert net.mean_attention(0) == pytest.approx(0.5)
    assert _train_acc(net) >= 0.9
    assert net.attention_weights(0).std() > 0


def test_residual_zero_skip_matches_plain_network():
    x, y = _data(1)[0][0], torch.eye(3)[0]
    plain = Network(CFG, seed=3)
    res = nw.ResidualNetwork(nw.ResidualNetworkConfig(base_config=CFG, skip_precision=0.0), seed=3)
    plain.learn(x, y, 10)
    res.learn(x, y, 10)
    assert torch.allclose(plain.layer(1).W, res.layer(1).W, atol=1e-6)
    res2 = nw.ResidualNetwork(nw.ResidualNetworkConfig(base_config=CFG, skip_precision=0.5), seed=3)
    w0 = res2.skip_w[0].clone()
    assert _train_acc(res2) >= 0.9 and not torch.equal(w0, res2.skip_w[0])


def test_hopfield_memory_retrieves_nearest_pattern():
    m = nw.HopfieldMemory(4)
    pats = torch.eye(4) * 3
    for p in pats:
        m.store(p)
    out = m.retrieve(pats[2] + 0.3 * torch.randn(4), beta=8.0, iterations=3)
    assert torch.allclose(out, pats[2], atol=1e-2)
    hn = nw.HopfieldNetwork(nw.HopfieldNetworkConfig(network_config=NetworkConfig(layer_sizes=(6, 8, 4))))
    xs, _ = _data(6)
    for x in xs:
        hn.learn(x, 5)
        hn.store(x, 5)
    assert hn.recall(xs[0], 5).shape == (6,) and hn.memory.count == 6


def test_hierarchical_generative_and_deep_recurrent():
    h = nw.HierarchicalNetwork(nw.HierarchicalNetworkConfig(modules=[NetworkConfig(layer_sizes=(6, 8, 5)),
                                                                     NetworkConfig(layer_sizes=(5, 6, 3))]))
    xs, _ = _data(6)
    before = sum(h.reconstruction_error(x, 10) for x in xs)
    for _ in range(20):
        for x in xs:
            h.learn(x, 10)
    assert [z.numel() for z in h.encode_all(xs[0], 5)] == [5, 3]
    assert sum(h.reconstruction_error(x, 10) for x in xs) < before
    gen = nw.GenerativeNetwork(nw.GenerativeNetworkConfig(network_config=NetworkConfig(layer_sizes=(6, 8, 3))))
    gen.learn(xs[0], 5)
    assert gen.sample(5, torch.Generator().manual_seed(0)).shape == (6,)
    dr = nw.DeepRecurrentNetwork(nw.DeepRecurrentNetworkConfig(
        stages=[NetworkConfig(layer_sizes=(6, 8, 5)), NetworkConfig(layer_sizes=(5, 6, 3))],
        temporal_precision=[0.5]))
    assert not dr.has_context
    for x in xs:
        z = dr.step(x, 5)
    assert z.shape == (3,) and dr.has_context
    dr.reset()
    assert not dr.has_context


def test_gated_state_memory_follows_big_changes():
    gs = nw.GatedStateNetwork(nw.GatedStateNetworkConfig(network_config=CFG))
    xs, ys = _data(6)
    m1 = gs.step(xs[0], 5)
    m2 = gs.step(xs[0], 5)
    assert torch.allclose(m1, m2, atol=0.2)
    gs.learn(xs[1], ys[1], 5)
    assert gs.predict(xs[1], 5) in (0, 1, 2)
    gs.reset()
    assert gs.memory is None


def test_active_inference_picks_goal_reaching_action():
    def env(obs, a):
        return obs + (0.5 if a == 1 else -0.5) * torch.ones(2)

    act = nw.ActiveNetwork(nw.ActiveNetworkConfig(observation_dim=2, action_count=2,
                                                  world_model_config=NetworkConfig(layer_sizes=(4, 16, 2),
                                                                                   weight_lr=0.05)))
    g = torch.Generator().manual_seed(1)
    for _ in range(300):
        o = torch.rand(2, generator=g) - 0.5
        a = int(torch.randint(0, 2, (1,), generator=g))
        act.observe(o, a, env(o, a), 50)
    o = torch.zeros(2)
    assert act.act(o, torch.ones(2) * 0.5, 50) == 1
    assert act.act(o, -torch.ones(2) * 0.5, 50) == 0


def test_graph_completion_moves_toward_neighbours():
    gp = nw.GraphPredictiveNetwork(nw.GraphPredictiveNetworkConfig(
        edge_predictor_config=NetworkConfig(layer_sizes=(4, 8, 4), weight_lr=0.05)))
    feats = [torch.tensor([0.5, 0.5, 0.0, 0.0])] * 3 + [torch.zeros(4)]
    nbrs = [[1], [0, 2], [1, 3], [2]]
    gp.learn(feats, nbrs, 5)
    out = gp.complete(feats, nbrs, [True, True, True, False], 5, 3)
    assert torch.equal(out[0], feats[0]) and not torch.equal(out[3], feats[3])
    assert gp.graph_energy(feats, nbrs, 5) >= 0
    with pytest.raises(ValueError):
        gp.learn(feats, [[5]] * 4, 5)


def test_spiking_network_learns_and_predicts():
    sn = nw.SpikingNetwork(nw.SpikingNetworkConfig(layer_sizes=(6, 16, 3), ticks=16))
    xs, ys = _data(9)
    e0 = sn.infer_energy(xs[0])
    for _ in range(5):
        for x, y in zip(xs, ys):
            sn.learn(x, y)
    assert sn.infer(xs[0]).shape == (3,) and e0 >= 0
    assert sn.predict(xs[0]) in (0, 1, 2)


def test_memory_bank_and_memory_network():
    mb = nw.MemoryBank(2, 3, 3)
    mb.write([1, 0, 0], [1, 1, 1])
    mb.write([0, 1, 0], [2, 2, 2])
    mb.write([0, 0, 1], [3, 3, 3])   # ring buffer overwrote the first entry
    top = mb.query_top_k([0, 0.9, 0.1], 1)
    assert mb.count == 2 and top[0][0][0] == 2
    mn = nw.MemoryNetwork(nw.MemoryNetworkConfig(network_config=CFG, memory_capacity=8))
    assert _train_acc(mn, epochs=15) >= 0.8
    assert mn.memory_count == 8


def test_multimodal_and_cross_modal_generation():
    cfg = nw.MultiModalNetworkConfig(
        modalities=[nw.ModalityConfig("a", NetworkConfig(layer_sizes=(6, 8, 4))),
                    nw.ModalityConfig("b", NetworkConfig(layer_sizes=(5, 8, 4)))],
        associative_config=NetworkConfig(layer_sizes=(8, 10, 3)), train_associative_generatively=True)
    mm = nw.MultiModalNetwork(cfg)
    xs, ys = _data(6)
    for x, y in zip(xs, ys):
        mm.learn({0: x, 1: x[:5]}, y, 5)
    assert mm.predict({0: xs[0]}, 5) in (0, 1, 2) and mm.modality_name(1) == "b"
    assert mm.cross_modal_generate(0, xs[0], 1, 5).shape == (5,)


def test_routed_network():
    cfg = nw.RoutedNetworkConfig(expert_config=CFG, router_config=NetworkConfig(layer_sizes=(6, 8, 3)),
                                 expert_count=3, top_k=2)
    rn = nw.RoutedNetwork(cfg)
    acc = _train_acc(rn, epochs=20)
    p = rn.predict_detailed(_data(1)[0][0], 10)
    assert len(p.active_experts) == 2 and abs(sum(p.router_gates) - 1) < 1e-5
    assert abs(sum(rn.last_gate_weights) - 1) < 1e-5 and acc >= 0.8


def test_temporal_wrappers():
    tn = nw.TemporalNetwork(Network(CFG), temporal_precision=0.5)
    xs, ys = _data(6)
    for x, y in zip(xs, ys):
        tn.step(x, y, 5)
    assert tn.has_prior and tn.predict(xs[0], 5) in (0, 1, 2)
    tm = nw.TemporalMixtureOfExperts(nw.TemporalMoEConfig(expert_count=2, expert_config=CFG))
    for x, y in zip(xs, ys):
        tm.step(x, y, 5)
    assert tm.predict(xs[0], 5) in (0, 1, 2)
    hm = nw.HierarchicalMixtureOfExperts(nw.HierarchicalMoEConfig(expert_config=CFG))
    for x, y in zip(xs, ys):
        hm.learn(x, y, 5)
    assert hm.predict(xs[0], 5) in (0, 1, 2)
