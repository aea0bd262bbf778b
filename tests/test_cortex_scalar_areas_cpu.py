"""Cortex areas without learned networks, property by property (the checks of
PredictiveCoding.UnitTests' CortexNeuromodulation, CortexLimbic, CortexReward, CortexSubcortical,
CortexAssociation, CortexSensoryExtra and CortexArea tests that need no training, restated for this
package)."""
import math

import numpy as np
import pytest
import torch

from predicitivecoding_b200.pc.network import Network, NetworkConfig
from predicitivecoding_b200.systems import cortex as cx


# ---------------------------------------------------------------- neuromodulation
def test_dopamine_rpe_terminal_and_discounted():
    d = cx.DopaminergicSystem(discount=0.9)
    assert d.reward_prediction_error(1.0, 0.4) == pytest.approx(0.6)
    assert d.reward_prediction_error(1.0, 0.4, 0.5) == pytest.approx(1.0 + 0.9 * 0.5 - 0.4)


def test_dopamine_baseline_tracks_the_average_reward_and_the_error_shrinks():
    d = cx.DopaminergicSystem(baseline_lr=0.2)
    errors = [abs(d.step(1.0)) for _ in range(40)]
    assert d.baseline == pytest.approx(1.0, abs=1e-3)
    assert errors[-1] < errors[0] * 0.01


def test_dopamine_scales_learning_with_surprise_and_rejects_bad_settings():
    d = cx.DopaminergicSystem(tonic_level=0.1)
    assert d.modulate_learning_rate(0.01, 2.0) > d.modulate_learning_rate(0.01, 0.1)
    assert d.modulate_learning_rate(0.01, 0.0) == pytest.approx(0.001)
    with pytest.raises(ValueError):
        cx.DopaminergicSystem(discount=1.5)
    with pytest.raises(ValueError):
        d.modulate_learning_rate(-1.0, 0.5)


def test_locus_coeruleus_bursts_on_a_surprise_spike_only():
    lc = cx.LocusCoeruleus(adaptation=0.1, phasic_threshold=1.5, phasic_gain=4.0, tonic_gain=1.0)
    assert lc.process(1.0) == (False, 1.0)            # first observation seeds the baseline
    for _ in range(10):
        burst, gain = lc.process(1.0)                   # steady surprise: tonic
        assert not burst and gain == 1.0
    burst, gain = lc.process(5.0)
    assert burst and gain == 4.0
    with pytest.raises(ValueError):
        cx.LocusCoeruleus(phasic_threshold=1.0)
    with pytest.raises(ValueError):
        lc.process(-1.0)


def test_locus_coeruleus_reads_energies_and_writes_the_gain_into_networks():
    nets = [Network(NetworkConfig(layer_sizes=(4, 6, 2)), seed=s) for s in range(2)]
    for n in nets:
        n.infer(torch.rand(4), 3)
    lc = cx.LocusCoeruleus()
    g = lc.modulate(nets)
    assert g == lc.tg
    for n in nets:
        assert n.layer(n.layer_count - 1).precision == pytest.approx(g)


def test_nucleus_basalis_favours_uncertain_areas_and_smooths():
    nb = cx.NucleusBasalis(areas=2, adaptation=0.5)
    ach = nb.update([1.0, 4.0])
    assert ach[1] > ach[0]
    lr = nb.modulate_learning_rates(0.01, [1.0, 4.0])
    assert lr[1] > lr[0]
    smoothed = nb.update([0.0, 0.0])
    assert 0 < smoothed[1] < 4.0                       # EMA, not a jump to the new value
    with pytest.raises(ValueError):
        nb.update([1.0])


def test_raphe_level_clamps_and_lengthens_the_horizon():
    r = cx.RapheNuclei(level=2.0)
    assert r.level == 1.0
    r.level = -1.0
    assert r.level == 0.0
    lo = (r.discount_factor(), r.time_horizon())
    r.level = 0.9
    hi = (r.discount_factor(), r.time_horizon())
    assert hi[0] > lo[0] and hi[1] > lo[1]


# ---------------------------------------------------------------- limbic, reward
def test_cingulate_conflict_high_on_ties_low_with_a_winner():
    cc = cx.CingulateCortex(temperature=1.0)
    assert cc.conflict([1.0, 1.0, 1.0]) == pytest.approx(1.0)
    assert cc.conflict([0.0, 20.0, 20.0]) < 0.05
    assert cc.needs_control([1.0, 1.0]) and not cc.needs_control([0.0, 30.0])


def test_hypothalamus_drive_is_setpoint_minus_current():
    h = cx.Hypothalamus([1.0, 0.5])
    assert np.allclose(h.drive([0.2, 0.5]), [0.8, 0.0])
    assert h.need_level([1.0, 0.5]) == 0.0


def test_insula_integrates_the_interoceptive_stream():
    ins = cx.InsularCortex(cx.Hypothalamus([1.0]), smoothing=0.5)
    feelings = [ins.experience([0.0]) for _ in range(10)]
    assert all(b >= a for a, b in zip(feelings, feelings[1:]))
    assert feelings[-1] == pytest.approx(1.0, abs=1e-2)
    ins.reset()
    assert ins.feel() == 0.0


def test_accumbens_picks_the_highest_value_and_need_sharpens_the_gate():
    na = cx.NucleusAccumbens(temperature=1.0)
    assert na.select([0.2, 0.9, 0.5], need=0.0) == 1
    flat = na.gate_weights([0.2, 0.9], need=0.0)
    sharp = na.gate_weights([0.2, 0.9], need=3.0)
    assert sharp[1] > flat[1]


def test_habenula_suppresses_dopamine_on_disappointment_only():
    hb = cx.Habenula(gain=1.0)
    assert hb.suppress_dopamine(1.0, reward=0.0, expected=0.8) == pytest.approx(0.2)
    assert hb.suppress_dopamine(1.0, reward=1.0, expected=0.5) == pytest.approx(1.0)


def test_periaqueductal_gray_escalates_with_threat():
    pag = cx.PeriaqueductalGray()
    assert [pag.respond(t) for t in (0.1, 0.4, 0.7, 0.95)] == ["none", "freeze", "flight", "fight"]


# ---------------------------------------------------------------- control and association
def test_basal_ganglia_selects_the_lowest_energy_and_withholds_above_threshold():
    bg = cx.BasalGanglia(temperature=1.0, no_go_threshold=2.0)
    best, gates = bg.select([1.5, 0.5, 3.0])
    assert best == 1 and abs(sum(gates) - 1) < 1e-9
    assert bg.select([2.5, 3.0])[0] == -1
    with pytest.raises(ValueError):
        bg.select([])


def test_thalamus_gives_reliable_areas_more_precision():
    th = cx.Thalamus(temperature=1.0, base_precision=1.0)
    p = th.allocate([0.1, 2.0, 5.0])
    assert p[0] > p[1] > p[2] and sum(p) == pytest.approx(3.0)


def test_pulvinar_keeps_the_mean_precision_at_base():
    p = cx.Pulvinar(temperature=0.5, base_precision=2.0).allocate([0.3, 0.1, 1.4, 0.8])
    assert np.mean(p) == pytest.approx(2.0)


def test_temporoparietal_junction_reorients_on_surprise_not_when_focused():
    tpj = cx.TemporoparietalJunction(threshold=2.0, adaptation=0.1)
    assert not tpj.should_reorient(1.0)
    assert not any(tpj.should_reorient(1.0) for _ in range(5))
    assert tpj.should_reorient(5.0)


def test_frontopolar_switches_to_a_better_held_goal_with_margin():
    fp = cx.FrontopolarCortex(switch_threshold=1.0, decay=0.9)
    assert not fp.should_switch(2.0, 1.0)              # nothing held
    fp.hold("alt")
    results = [fp.should_switch(2.0, 1.5) for _ in range(5)]
    assert not results[0] and any(results)
    fp.clear()
    assert fp.held is None


def test_claustrum_coherence_and_binding():
    a = torch.tensor([1.0, 0.0])
    assert cx.Claustrum.coherence([a, a]) == pytest.approx(1.0)
    assert cx.Claustrum.coherence([a, -a]) == pytest.approx(-1.0)
    assert torch.allclose(cx.Claustrum.synchronize([a, torch.tensor([0.0, 1.0])]), torch.tensor([0.5, 0.5]))


# ---------------------------------------------------------------- sensory front ends
def test_retina_difference_of_gaussians_cancels_a_flat_image():
    r = cx.RetinaLgn(1, 8, 8)
    out = r.process(torch.full((64,), 0.7))
    assert out.shape == (64,) and float(out.abs().max()) < 1e-5
    edge = torch.zeros(8, 8)
    edge[:, 4:] = 1.0
    assert float(r.process(edge.reshape(-1)).abs().max()) > 0.05
    with pytest.raises(ValueError):
        cx.RetinaLgn(1, 8, 8, center_sigma=2.0, surround_sigma=1.0)


def test_superior_colliculus_fuses_modalities_with_inhibition_of_return():
    sc = cx.SuperiorColliculus(4, enhancement=1.0)
    vis, aud = [0.1, 0.9, 0.2, 0.0], [0.0, 0.1, 0.8, 0.0]
    p = sc.priority_map(vis, aud)
    assert p[2] == pytest.approx(0.2 + 0.8 + 0.2 * 0.8)      # visual + auditory + cross-modal enhancement
    path = sc.scan(vis, aud, 4)
    assert path[:2] == [2, 1] and sorted(path) == [0, 1, 2, 3]   # inhibition of return: no repeats


def test_inferior_colliculus_reports_band_energy_peaks():
    ic = cx.InferiorColliculus(bands=8)
    t = torch.arange(256, dtype=torch.float32)
    low = ic.process(torch.sin(2 * math.pi * 4 * t / 256))
    high = ic.process(torch.sin(2 * math.pi * 100 * t / 256))
    assert int(low.argmax()) < int(high.argmax())


def test_olfactory_bulb_keeps_k_strongest_normalised():
    ob = cx.OlfactoryBulb(k=2)
    out = ob.process([0.1, 3.0, 0.2, 4.0])
    assert int((out != 0).sum()) == 2 and out[3] > out[1] > 0


def test_grid_cells_are_periodic_on_the_hexagonal_lattice():
    g = cx.GridCellEncoder(modules=1, cells_per_module=9, base_frequency=1.3, ratio=1.4)
    f = float(g.freq[0])
    lx, ly = 2 * math.pi / f, 2 * math.pi / f / math.sqrt(3)   # a lattice vector of the three 60-degree waves
    a = g.encode(0.4, -0.2)
    assert torch.allclose(a, g.encode(0.4 + lx, -0.2 + ly), atol=1e-4)
    assert not torch.allclose(a, g.encode(0.4 + 0.5 * lx, -0.2), atol=1e-2)
    assert g.code_dim == 9 and float(a.min()) >= 0 and float(a.max()) <= 1
