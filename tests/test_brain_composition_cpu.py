"""Object composition, behaviours and conceptual frames (the checks of PredictiveCoding.UnitTests'
BrainCompositionTests, restated for this package)."""
import pytest

from predicitivecoding_b200.systems.brain import ScalarEncoder, Sdr
from predicitivecoding_b200.systems.brain_ext import (BehaviorSequence, CompositeObject, CompositionLibrary,
                                                      ConceptualFrame, FeaturePoint, RigidPose2D)


def feat(i, size=64):
    return Sdr(size, range(4 * i, 4 * i + 4))


def square():
    return [FeaturePoint(0, 0, feat(0)), FeaturePoint(1, 0, feat(1)), FeaturePoint(1, 1, feat(2)),
            FeaturePoint(0, 1, feat(3))]


def pts(points):
    return sorted((round(p.x, 6), round(p.y, 6), p.feature.bits) for p in points)


def test_primitive_resolves_to_its_own_points():
    lib = CompositionLibrary()
    lib.add_primitive(1, square())
    assert pts(lib.resolve(1)) == pts(square())


def test_composite_applies_the_part_translation_and_rotation():
    lib = CompositionLibrary()
    lib.add_primitive(1, square())
    lib.create_composite(10).add_part(1, x=5.0, y=-2.0)
    assert pts(lib.resolve(10)) == pts([p.transformed(RigidPose2D(5, -2)) for p in square()])
    lib.create_composite(11).add_part(1, rotation_deg=90.0)
    rotated = {(round(p.x, 6), round(p.y, 6)) for p in lib.resolve(11)}
    assert rotated == {(0.0, 0.0), (0.0, 1.0), (-1.0, 1.0), (-1.0, 0.0)}


def test_nested_composites_compose_the_transforms_down_the_tree():
    lib = CompositionLibrary()
    lib.add_primitive(1, [FeaturePoint(1.0, 0.0, feat(5))])
    lib.create_composite(2).add_part(1, x=2.0, rotation_deg=90.0)
    lib.create_composite(3).add_part(2, y=3.0, rotation_deg=90.0)
    (p,) = lib.resolve(3)
    # inner: (1,0) -> rotate 90 -> (0,1) -> +(2,0) = (2,1); outer: rotate 90 -> (-1,2) -> +(0,3) = (-1,5)
    assert (round(p.x, 6), round(p.y, 6)) == (-1.0, 5.0)


def test_cycles_unknown_children_and_duplicate_ids_are_rejected():
    lib = CompositionLibrary()
    lib.create_composite(1).add_part(2)
    lib.create_composite(2).add_part(1)
    with pytest.raises(RuntimeError):
        lib.resolve(1)
    lib.create_composite(3).add_part(99)
    with pytest.raises(KeyError):
        lib.resolve(3)
    lib.add_primitive(7, square())
    with pytest.raises(ValueError):
        lib.add_primitive(7, square())
    with pytest.raises(ValueError):
        CompositeObject(4).add_part(4)


def test_behaviour_sequences_predict_place_and_score():
    seq = BehaviorSequence(1)
    for i in range(4):
        seq.append(feat(i))
    assert len(seq) == 4 and seq.predict_next(1) == feat(2) and seq.predict_next(3) is None
    enc = ScalarEncoder(0, 10, 40, 4)
    points = seq.to_object_points(enc)
    assert [loc for loc, _ in points] == [enc.encode(i) for i in range(4)]
    assert seq.match_score([feat(0), feat(1)], 4) == 1.0
    assert seq.match_score([feat(0), feat(9)], 4) == 0.5


def test_conceptual_frame_locality_recall_and_movement():
    cf = ConceptualFrame([(0.0, 10.0), (0.0, 10.0)])
    a, near, far = cf.encode_location([5, 5]), cf.encode_location([5.2, 5.0]), cf.encode_location([9, 1])
    assert a.overlap(near) > a.overlap(far)
    assert cf.nearest([1, 1]) is None
    cf.add_concept([1, 1], feat(1))
    cf.add_concept([8, 8], feat(2))
    assert cf.recall([2, 1]) == feat(1) and cf.recall([7, 9]) == feat(2)
    assert cf.move([1, 1], [2, 3]) == [3.0, 4.0]
    with pytest.raises(ValueError):
        cf.encode_location([1, 2, 3])
