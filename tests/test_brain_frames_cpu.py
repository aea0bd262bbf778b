"""Thousand-Brains building blocks, property by property (the checks of PredictiveCoding.UnitTests'
BrainSdrTests, BrainPathIntegrationTests and BrainSe3AndSensorTests, restated for this package): SDR
algebra and encoders, 2D dead reckoning, SE(3) poses, the 3D pose encoder and 3D path integration."""
import math

import numpy as np
import pytest

from predicitivecoding_b200.systems.brain import (CategoryEncoder, PathIntegrator, Pose2D, PoseEncoder,
                                                  ScalarEncoder, Sdr)
from predicitivecoding_b200.systems.brain_ext import (PathIntegrator3D, Pose3D, PoseEncoder3D, RigidPose2D)


def close3(a, b, tol=1e-5):
    return all(abs(x - y) < tol for x, y in zip(a, b))


# ---------------------------------------------------------------- SDR algebra
def test_construction_sorts_dedups_and_counts():
    s = Sdr(10, [5, 1, 5, 3])
    assert s.bits == (1, 3, 5) and s.cardinality == 3 and s.sparsity == pytest.approx(0.3)


def test_construction_rejects_out_of_range():
    with pytest.raises(ValueError):
        Sdr(4, [4])
    with pytest.raises(ValueError):
        Sdr(4, [-1])
    with pytest.raises(ValueError):
        Sdr(0)


def test_overlap_identical_disjoint_and_size_mismatch():
    a, b = Sdr(8, [0, 1, 2]), Sdr(8, [5, 6])
    assert a.overlap(a) == 3 and a.overlap(b) == 0 and a.overlap_score(a) == 1.0
    with pytest.raises(ValueError):
        a.overlap(Sdr(9, [0]))


def test_union_and_intersect():
    a, b = Sdr(8, [0, 1, 2]), Sdr(8, [2, 3])
    assert a.union(b).bits == (0, 1, 2, 3) and a.intersect(b).bits == (2,)


def test_random_sdr_cardinality_range_and_determinism():
    a = Sdr.random(100, 7, np.random.default_rng(3))
    b = Sdr.random(100, 7, np.random.default_rng(3))
    assert a == b and a.cardinality == 7 and all(0 <= x < 100 for x in a.bits)
    with pytest.raises(ValueError):
        Sdr.random(5, 6, np.random.default_rng(0))


def test_noise_keeps_cardinality_and_moves_exactly_the_noise_bits():
    s = Sdr.random(200, 20, np.random.default_rng(1))
    n = s.add_noise(0.25, np.random.default_rng(2))
    assert n.cardinality == 20 and s.overlap(n) == 15


def test_subsample_takes_a_subset():
    s = Sdr.random(200, 20, np.random.default_rng(4))
    sub = s.subsample(5, np.random.default_rng(5))
    assert sub.cardinality == 5 and s.overlap(sub) == 5


def test_dense_round_trip_and_value_equality():
    s = Sdr(6, [0, 4])
    assert Sdr.from_dense(s.to_dense()) == s
    assert s == Sdr(6, [4, 0]) and hash(s) == hash(Sdr(6, [0, 4])) and s != Sdr(7, [0, 4])


def test_scalar_encoder_window_overlap_and_clamp():
    e = ScalarEncoder(0.0, 10.0, 50, 8)
    a, b, far = e.encode(5.0), e.encode(5.2), e.encode(9.5)
    assert a.cardinality == 8 and a.overlap(b) > a.overlap(far)
    assert e.encode(-3.0) == e.encode(0.0) and e.encode(99.0) == e.encode(10.0)
    with pytest.raises(ValueError):
        ScalarEncoder(0.0, 1.0, 10, 10)


def test_category_encoder_blocks_are_disjoint_and_stable():
    c = CategoryEncoder(4, 5)
    codes = [c.encode(i) for i in range(4)]
    assert all(codes[i].overlap(codes[j]) == 0 for i in range(4) for j in range(4) if i != j)
    assert c.encode(2) == codes[2]
    with pytest.raises(ValueError):
        c.encode(4)


# ---------------------------------------------------------------- 2D dead reckoning
def test_steps_accumulate_world_frame_displacement():
    p = PathIntegrator()
    p.move(2.0)
    p.move(3.0, turn_deg=90.0)
    assert p.pose.x == pytest.approx(2.0) and p.pose.y == pytest.approx(3.0)
    assert p.displacement(0, 2) == pytest.approx((2.0, 3.0))


def test_closed_square_returns_to_the_start():
    p = PathIntegrator()
    for _ in range(4):
        p.move(1.5)
        p.move(0.0, turn_deg=90.0)
    assert abs(p.pose.x) < 1e-9 and abs(p.pose.y) < 1e-9


def test_heading_is_normalised_into_0_360():
    assert Pose2D().moved(0.0, -90.0).theta_deg == pytest.approx(270.0)
    assert Pose2D(theta_deg=350.0).moved(0.0, 30.0).theta_deg == pytest.approx(20.0)


def test_location_codes_overlap_more_for_nearby_poses():
    enc = PoseEncoder(0, 10, 0, 10)
    a, near, far = enc.encode(5, 5, 0), enc.encode(5.2, 5.1, 0), enc.encode(9, 1, 0)
    assert a.size == enc.size and a.overlap(near) > a.overlap(far)


# ---------------------------------------------------------------- rigid poses
def test_pose2d_identity_rotation_composition_and_inverse():
    assert RigidPose2D().apply(1.5, -2.0) == pytest.approx((1.5, -2.0))
    assert RigidPose2D(theta_deg=90.0).apply(1.0, 0.0) == pytest.approx((0.0, 1.0), abs=1e-12)
    t = RigidPose2D(1, 2).compose(RigidPose2D(3, 4))
    assert (t.x, t.y) == pytest.approx((4, 6))
    p = RigidPose2D(1.0, -2.0, 37.0)
    ident = p.compose(p.inverse()).normalized()
    assert (ident.x, ident.y) == pytest.approx((0, 0), abs=1e-12) and ident.theta_deg % 360 == pytest.approx(0, abs=1e-9)


def test_yaw_pitch_roll_conventions():
    assert close3(Pose3D.from_yaw_pitch_roll(90, 0, 0).apply(1, 0, 0), (0, 1, 0))      # yaw about z
    assert close3(Pose3D.from_yaw_pitch_roll(0, 90, 0).apply(1, 0, 0), (0, 0, 1))      # pitch lifts forward
    assert close3(Pose3D.from_yaw_pitch_roll(0, 0, 90).apply(0, 1, 0), (0, 0, 1))      # roll about forward


@pytest.mark.parametrize("ypr", [(30.0, 20.0, -40.0), (-120.0, -60.0, 10.0), (170.0, 5.0, 95.0)])
def test_yaw_pitch_roll_round_trip_inside_the_gimbal_range(ypr):
    back = Pose3D.from_yaw_pitch_roll(*ypr).to_yaw_pitch_roll()
    assert back == pytest.approx(ypr, abs=1e-4)


def test_pose3d_translation_composition_and_inverse():
    assert close3(Pose3D.from_translation(1, 2, 3).apply(0, 0, 0), (1, 2, 3))
    p = Pose3D(1.0, -2.0, 0.5, Pose3D.from_yaw_pitch_roll(40, -15, 70).rotation)
    ident = p.compose(p.inverse())
    assert close3(ident.apply(0.3, -0.7, 1.1), (0.3, -0.7, 1.1))
    a = Pose3D(0.5, 0, 0, Pose3D.from_yaw_pitch_roll(30, 0, 0).rotation)
    b = Pose3D(0, 1.0, 0, Pose3D.from_yaw_pitch_roll(0, 20, 0).rotation)
    assert close3(a.compose(b).apply(1, 2, 3), a.apply(*b.apply(1, 2, 3)))


def test_yaw_only_pose3d_matches_pose2d_in_the_plane():
    p2 = RigidPose2D(1.0, 2.0, 33.0)
    p3 = Pose3D(1.0, 2.0, 0.0, Pose3D.from_yaw_pitch_roll(33.0, 0, 0).rotation)
    for px, py in ((0.5, 0.0), (-1.0, 2.5)):
        assert close3(p3.apply(px, py, 0.0), (*p2.apply(px, py), 0.0))


# ---------------------------------------------------------------- 3D pose code and path integration
def enc3():
    return PoseEncoder3D(-5, 5, -5, 5, -5, 5)


def test_pose_encoder3d_is_deterministic_local_and_orientation_sensitive():
    e = enc3()
    a = e.encode(1, 1, 1, 0, 0, 0)
    assert a == e.encode(1, 1, 1, 0, 0, 0)
    assert a.overlap(e.encode(1.1, 1, 1, 0, 0, 0)) > a.overlap(e.encode(-4, 4, -3, 0, 0, 0))
    assert a != e.encode(1, 1, 1, 180, 0, 0)


def test_forward_steps_follow_the_heading():
    p = PathIntegrator3D(enc3(), yaw0=90.0)
    p.step_forward(2.0)
    assert close3((p.x, p.y, p.z), (0.0, 2.0, 0.0))


@pytest.mark.parametrize("turn", [(90.0, 0.0, 0.0), (0.0, 90.0, 0.0)])
def test_square_loops_return_to_the_start(turn):
    p = PathIntegrator3D(enc3())
    start = p.location_code
    for _ in range(4):
        p.step_forward(1.0)
        p.rotate(*turn)
    assert close3((p.x, p.y, p.z), (0, 0, 0)) and p.location_code == start


def test_climb_traverse_descend_closes_the_loop():
    p = PathIntegrator3D(enc3())
    for d in ((0, 0, 2), (3, 0, 0), (0, 0, -2), (-3, 0, 0)):
        p.step(*d)
    assert close3((p.x, p.y, p.z), (0, 0, 0))


def test_step_and_counter_step_return_to_the_origin():
    p = PathIntegrator3D(enc3(), yaw0=30.0, pitch0=10.0)
    code = p.location_code
    p.step_forward(1.7)
    p.step_forward(-1.7)
    assert p.location_code == code
