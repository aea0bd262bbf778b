"""People tracking and counting semantics (the checks of PredictiveCoding.UnitTests' PeopleTrackingTests
and PeopleCountingSemanticsTests, restated for this package)."""
import pytest

from predicitivecoding_b200.systems.vision import Detection, LineCounter, SortTracker, ZoneCounter


def box(cx, cy, w=20.0, h=40.0):
    return Detection(cx - w / 2, cy - h / 2, cx + w / 2, cy + h / 2)


def run(tracker, frames):
    for dets in frames:
        tracker.update(dets)
    return tracker


def test_a_steady_person_is_confirmed_and_counted_once():
    t = run(SortTracker(min_hits=3), [[box(50, 50)]] * 10)
    assert t.unique_count == 1 and t.current_count == 1


def test_two_separate_people_count_as_two():
    t = run(SortTracker(), [[box(50, 50), box(200, 50)]] * 6)
    assert t.unique_count == 2 and t.current_count == 2


def test_a_moving_person_keeps_one_identity():
    frames = [[box(50 + 4 * i, 60)] for i in range(20)]
    t = run(SortTracker(), frames)
    assert t.unique_count == 1 and len({tr.id for tr in t.tracks}) == 1


def test_a_short_occlusion_does_not_create_a_new_identity():
    frames = [[box(80, 80)]] * 5 + [[]] * 3 + [[box(80, 80)]] * 5
    t = run(SortTracker(max_age=10), frames)
    assert t.unique_count == 1


def test_a_long_absence_retires_the_track_and_reentry_counts_again():
    frames = [[box(80, 80)]] * 5 + [[]] * 8 + [[box(80, 80)]] * 5
    t = run(SortTracker(max_age=4), frames)
    assert t.unique_count == 2


def test_a_brief_detection_below_min_hits_is_not_counted():
    t = run(SortTracker(min_hits=3), [[box(30, 30)]] * 2 + [[]] * 40)
    assert t.unique_count == 0


def test_the_tracker_follows_a_constant_velocity_target():
    t = SortTracker()
    for i in range(15):
        t.update([box(20 + 6 * i, 50)])
    tr = t.tracks[0]
    assert tr.vcx == pytest.approx(6.0, abs=1.0) and tr.center_x == pytest.approx(20 + 6 * 14, abs=2.0)


def test_reset_clears_tracks_and_counters():
    t = run(SortTracker(), [[box(50, 50)]] * 5)
    t.reset()
    assert t.unique_count == 0 and t.tracks == [] and t.next_id == 1


def test_line_counter_counts_directional_crossings_and_the_net():
    lc = LineCounter(0, 50, 100, 50)
    lc.update([(1, 40.0, 40.0)])
    lc.update([(1, 40.0, 60.0)])       # crosses one way
    lc.update([(2, 60.0, 70.0)])
    lc.update([(2, 60.0, 30.0)])       # crosses back the other way
    lc.update([(3, 10.0, 30.0)])
    lc.update([(3, 10.0, 80.0)])
    assert lc.inbound + lc.outbound == 3 and abs(lc.net) == 1


def test_line_counter_ignores_passes_beyond_the_segment_and_non_crossings():
    lc = LineCounter(0, 50, 100, 50)
    lc.update([(1, 150.0, 40.0)])
    lc.update([(1, 150.0, 60.0)])      # beyond the end point
    lc.update([(2, 20.0, 10.0)])
    lc.update([(2, 30.0, 20.0)])       # stays on one side
    assert lc.inbound == lc.outbound == 0
    with pytest.raises(ValueError):
        LineCounter(1, 1, 1, 1)


def test_line_counter_works_from_tracker_output():
    t, lc = SortTracker(min_hits=1), LineCounter(0, 100, 300, 100)
    for i in range(12):
        lc.update(t.update([box(60, 60 + 8 * i)]))
    assert lc.inbound + lc.outbound == 1


def test_zone_counter_occupancy_entries_and_dwell():
    z = ZoneCounter([(0, 0), (100, 0), (100, 100), (0, 100)])
    assert z.is_inside(50, 50) and not z.is_inside(150, 50)
    for _ in range(3):
        z.update([(1, 50.0, 50.0), (2, 150.0, 50.0)])
    z.update([(2, 60.0, 60.0)])
    assert z.entered == 2 and z.dwell_frames(1) == 3 and z.dwell_frames(2) == 1 and z.occupancy == 1
    with pytest.raises(ValueError):
        ZoneCounter([(0, 0), (1, 1)])
