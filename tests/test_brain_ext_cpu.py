"""Thousand-Brains extensions: 3D frames, displacement recognition, composition, heterarchical
message passing, object-model persistence and the HTML view."""
import math
import os
import tempfile

import numpy as np
import pytest

from predicitivecoding_b200.systems.brain import CorticalColumnConfig, MultiColumnSystem, PoseEncoder, Sdr
from predicitivecoding_b200.systems.brain_ext import (
    BehaviorSequence, CompositeObject, CompositionLibrary, ConceptualFrame, ConnectionType, DisplacementModule,
    DisplacementRecognizer, FeaturePoint, FeaturePoint3D, HeterarchicalGraph, HeterarchicalMessagePassing,
    HtmlVisualizer, ObjectModelStore, PathIntegrator3D, Pose3D, PoseEncoder3D, RigidPose2D, SdrCodec,
    SyntheticObject, VizBenchmarkRow, VizData, VizEpisode, VizObject, VizPoint, VizPoseInvariance, VizPoseRow)


def test_pose3d_compose_inverse_and_angles():
    p = Pose3D(1, 2, 3).compose(Pose3D.from_yaw_pitch_roll(30, 20, 10))
    q = p.compose(p.inverse())
    assert max(abs(v) for v in (q.x, q.y, q.z)) < 1e-9
    assert abs(abs(q.rotation.w) - 1) < 1e-9
    y, pt, r = Pose3D.from_yaw_pitch_roll(30, 20, 10).to_yaw_pitch_roll()
    assert (round(y, 6), round(pt, 6), round(r, 6)) == (30.0, 20.0, 10.0)
    # yaw 90: +x maps to +y
    x, yy, z = Pose3D.from_yaw_pitch_roll(90, 0, 0).apply(1, 0, 0)
    assert abs(x) < 1e-9 and abs(yy - 1) < 1e-9 and abs(z) < 1e-9


def test_path_integrator_3d_forward_and_turn():
    enc = PoseEncoder3D(-10, 10, -10, 10, -10, 10)
    pi = PathIntegrator3D(enc)
    pi.step_forward(2.0)
    pi.rotate(90, 0, 0)
    code = pi.step_forward(3.0)
    assert abs(pi.x - 2) < 1e-9 and abs(pi.y - 3) < 1e-9 and code.size == enc.size
    assert code.cardinality == 3 * 10 + 3 * 5


def _landmarks(rng, n=6, spread=8.0):
    feats = [Sdr.random(200, 20, rng) for _ in range(n)]
    return [FeaturePoint(float(rng.uniform(0, spread)), float(rng.uniform(0, spread)), f) for f in feats]


def test_displacement_recognizer_is_pose_invariant():
    rng = np.random.default_rng(0)
    objs = {i: _landmarks(rng) for i in range(5)}
    rec = DisplacementRecognizer(min_overlap=12, distance_tolerance=0.05)
    for i, o in objs.items():
        rec.learn(i, o)
    moved = RigidPose2D(13.0, -4.0, 71.0)
    for i, o in objs.items():
        assert rec.recognize([p.transformed(moved) for p in o]) == i
    # 3D landmarks under a 3D rigid motion
    pts = [FeaturePoint3D(*rng.uniform(0, 5, 3), Sdr.random(200, 20, rng)) for _ in range(5)]
    rec3 = DisplacementRecognizer(distance_tolerance=0.05)
    rec3.learn(7, pts)
    pose = Pose3D(1, 2, 3).compose(Pose3D.from_yaw_pitch_roll(40, -25, 60))
    assert rec3.recognize([p.transformed(pose) for p in pts]) == 7
    dm = DisplacementModule(10.0)
    assert dm.encode(1.5, -2).size == dm.sdr_size and dm.between(1, 1, 4, -1) == (3, -2)


def test_composition_resolves_nested_parts_and_detects_cycles():
    rng = np.random.default_rng(1)
    lib = CompositionLibrary()
    wheel = _landmarks(rng, 3)
    lib.add_primitive(1, wheel)
    car = lib.create_composite(10).add_part(1, 0, 0).add_part(1, 5, 0, 90)
    pts = lib.resolve(10)
    assert len(pts) == 6
    x, y = RigidPose2D(5, 0, 90).apply(wheel[0].x, wheel[0].y)
    assert abs(pts[3].x - x) < 1e-9 and abs(pts[3].y - y) < 1e-9
    lib.create_composite(20).add_part(10, 1, 1)
    assert len(lib.resolve(20)) == 6
    lib.create_composite(30).add_part(31)
    lib.create_composite(31).add_part(30)
    with pytest.raises(RuntimeError):
        lib.resolve(30)
    with pytest.raises(ValueError):
        CompositeObject(3).add_part(3)
    obs = lib.to_observations(10, PoseEncoder(-20, 20, -20, 20))
    assert len(obs) == 6


def test_behavior_sequence_and_conceptual_frame():
    rng = np.random.default_rng(2)
    states = [Sdr.random(100, 10, rng) for _ in range(4)]
    b = BehaviorSequence(1)
    for s in states:
        b.append(s)
    assert b.predict_next(1) == states[2] and b.predict_next(3) is None
    assert b.match_score(states[:2], 8) == 1.0
    f = ConceptualFrame([(0, 1), (0, 10)])
    f.add_concept([0.2, 3], states[0])
    f.add_concept([0.9, 9], states[1])
    assert f.recall([0.8, 8.5]) == states[1]
    assert f.move([0.1, 1], [0.2, 2]) == pytest.approx([0.3, 3])
    assert f.encode_location([0.5, 5]).size == f.location_size


def test_heterarchical_areas_agree_faster_than_alone():
    rng = np.random.default_rng(3)
    F, L = 200, 200
    feats = [Sdr.random(F, 12, rng) for _ in range(6)]
    locs = [Sdr.random(L, 12, rng) for _ in range(8)]
    objects = [[(feats[rng.integers(6)], locs[k]) for k in rng.choice(8, 5, replace=False)] for _ in range(6)]
    g = HeterarchicalGraph()
    for a in range(2):
        sysm = MultiColumnSystem([CorticalColumnConfig(F, 128, 4, 0.04, 2, 7 * a + c) for c in range(2)])
        for o in objects:
            sysm.learn_object([o, o])
        g.add_area(a, sysm)
    g.connect(0, 1, ConnectionType.LATERAL, 1.0)
    g.connect(1, 0, ConnectionType.HETERARCHICAL, 0.5)
    with pytest.raises(ValueError):
        g.connect(0, 0)
    target = objects[2]
    inputs = {0: [target[0], target[1]], 1: [target[2], target[3]]}
    out = HeterarchicalMessagePassing(max_rounds=6).pass_messages(g, inputs)
    assert set(out) == {0, 1}
    assert all(2 in o.consensus.candidates for o in out.values())
    assert len(g.incoming(1)) == 1 and len(g.outgoing(1)) == 1


def test_object_model_store_round_trip():
    rng = np.random.default_rng(4)
    objs = [SyntheticObject(i, _landmarks(rng, 3)) for i in range(3)]
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "models.txt")
        ObjectModelStore.save(p, objs)
        text = open(p).read()
        assert text.startswith("# PredictiveCoding.Brain object models v1\nobject 0 3\n")
        back = ObjectModelStore.load(p)
    assert [o.id for o in back] == [0, 1, 2]
    for a, b in zip(objs, back):
        for p, q in zip(a.points, b.points):
            assert abs(p.x - q.x) < 1e-5 and p.feature == q.feature
    assert SdrCodec.decode(SdrCodec.encode(Sdr(9, []))) == Sdr(9, [])
    with pytest.raises(ValueError):
        ObjectModelStore.loads("object 1 2\n0 0 4|1\n")


def test_html_visualizer_is_self_contained_and_escapes_data():
    data = VizData(title="</script><b>x", benchmark=[VizBenchmarkRow("clean", 0.8, 6.1, 1.0, 3.2)],
                   episode=VizEpisode(1, 2, 3, [VizObject(1, [VizPoint(0, 0, 2), VizPoint(1, 2, 3)])],
                                      [[0, 1], [1]], [[1]]),
                   pose_invariance=VizPoseInvariance(1, 2, 30, [VizPoseRow(1, False, True)]))
    page = HtmlVisualizer.render(data)
    assert page.startswith("<!DOCTYPE html>") and "</script><b>" not in page
    assert "http" not in page and "src=" not in page
    assert '"votingAccuracy": 1.0' in page and '"columnsVoting": 3' in page
