"""The frame-slice scheduler (bl_scheduler_*, beatlm_b200.schedule) against
the reference's own cases for its Scheduler (crates/beatlm-core/src/
schedule.rs:850-2121), sync policies (sync.rs), budget (budget.rs) and beat
grids (time.rs). Host logic only; no GPU."""
import pytest

from beatlm_b200.cost import CostModel, MeanPlusSigmas
from beatlm_b200.schedule import (BeatGrid, Delivery, Due, FixedLatency, FrameInfo, Missed,
                                  OnBeat, SameFrame, ScheduleError, Scheduler, beat_map_next,
                                  budget_for_frame, max_in_flight, source_delay)

PERIOD = 1000
U64_MAX = (1 << 64) - 1


def frame(i):
    return FrameInfo(i, i * PERIOD, PERIOD)


def at(start):
    return FrameInfo(start // PERIOD, start, PERIOD)


def cost():
    """Every unmeasured slice costs 100 us."""
    return CostModel(100, MeanPlusSigmas(1.0, 0.0))


def grid():
    return BeatGrid(0, 1000)


def on_beat(margin):
    return OnBeat(margin, grid())


def beat(us):
    return Due("beat", us)


def fr(i):
    return Due("frame", i)


def runs(p):
    return [(r.job, r.position) for r in p.runs]


# ------------------------------------------------------------ time, budget, sync

def test_beat_grid_rounds_up_to_its_beats():  # time.rs tests
    g = BeatGrid(1000, 500)
    assert g.next_beat_at_or_after(10) == 1000
    assert g.next_beat_at_or_after(1000) == 1000 and g.next_beat_at_or_after(2500) == 2500
    assert g.next_beat_at_or_after(1001) == 1500 and g.next_beat_at_or_after(1999) == 2000
    assert BeatGrid(0, 1000).next_beat_at_or_after(U64_MAX - 1) == U64_MAX
    with pytest.raises(ScheduleError) as e:
        BeatGrid(0, 0)
    assert e.value.kind == "ZeroBeat"


def test_beat_map_switches_grids_at_the_change():  # time.rs tests
    changed = [(0, BeatGrid(0, 1000)), (2500, BeatGrid(2600, 300))]
    assert beat_map_next(changed, 1200) == 2000
    assert beat_map_next(changed, 2700) == 2900
    # the old grid's next beat after 2100 is 3000, past the change at 2500:
    # the new grid's first beat at or after 2500 is taken
    assert beat_map_next(changed, 2100) == 2600
    # replacing drops the grids announced at or after it
    assert beat_map_next(changed + [(2000, BeatGrid(0, 700))], 2700) == 2800


def test_budget_for_frame_subtracts_render_and_margin():  # budget.rs tests
    assert budget_for_frame(16000, 10000, 1000) == 5000
    assert budget_for_frame(16000, 15000, 2000) == 0
    assert budget_for_frame(1, U64_MAX, U64_MAX) == 0


def test_source_delay_and_in_flight_follow_the_policy():  # sync.rs tests
    assert source_delay(FixedLatency(3)) == 3 and source_delay(SameFrame()) == 0
    assert source_delay(on_beat(0)) is None
    assert max_in_flight(FixedLatency(0)) == 1 and max_in_flight(FixedLatency(2)) == 3
    assert max_in_flight(FixedLatency((1 << 32) - 1)) == (1 << 32) - 1
    assert max_in_flight(SameFrame()) == 1 and max_in_flight(on_beat(0)) is None


# ------------------------------------------------------------ scheduler

def test_replacing_beats_needs_an_on_beat_scheduler():  # schedule.rs:854
    s = Scheduler(SameFrame(), "drop", 100)
    with pytest.raises(ScheduleError) as e:
        s.replace_beat_grid(0, grid())
    assert e.value.kind == "NotOnBeat"
    Scheduler(on_beat(0), "drop", 100).replace_beat_grid(0, grid())


def test_empty_job_is_rejected():  # schedule.rs:863
    s = Scheduler(SameFrame(), "drop", 100)
    with pytest.raises(ScheduleError) as e:
        s.submit(frame(0), [], cost())
    assert e.value.kind == "EmptyJob" and s.pending() == 0


def test_job_ids_count_from_zero():  # schedule.rs:871
    s = Scheduler(SameFrame(), "drop", 100)
    c = cost()
    assert [s.submit(frame(0), [0], c) for _ in range(2)] == [0, 1]


def test_fixed_latency_delivers_exactly_on_its_frame():  # schedule.rs:879
    s = Scheduler(FixedLatency(2), "drop", 1000)
    c = cost()
    job = s.submit(frame(10), [0], c)
    assert s.due(job) == fr(12)
    p10 = s.plan_frame(frame(10), 1000, c)
    assert len(p10.runs) == 1 and not p10.delivered and not p10.missed
    p11 = s.plan_frame(frame(11), 1000, c)
    assert not p11.runs and not p11.delivered and not p11.missed and s.pending() == 1
    p12 = s.plan_frame(frame(12), 1000, c)
    assert p12.delivered == [Delivery(job, 10)] and not p12.missed
    assert s.pending() == 0 and s.due(job) is None


def test_a_lone_job_that_cannot_finish_runs_to_its_deadline_and_is_missed_there():  # :912
    s = Scheduler(FixedLatency(2), "hold_previous", 100)
    c = cost()
    job = s.submit(frame(0), [0, 1, 2, 3], c)
    for f in range(2):
        p = s.plan_frame(frame(f), 100, c)
        assert len(p.runs) == 1 and not p.delivered and not p.missed, f
    p = s.plan_frame(frame(2), 100, c)
    assert len(p.runs) == 1 and p.runs[0].position == 2 and not p.delivered
    assert p.missed == [Missed(job, 0, fr(2), "hold_previous")]
    assert s.pending() == 0
    for f in range(3, 6):
        later = s.plan_frame(frame(f), 100, c)
        assert not later.runs and not later.delivered and not later.missed


def test_a_forecast_above_the_real_budget_delays_the_miss_to_its_deadline():  # :956
    s = Scheduler(FixedLatency(2), "hold_previous", 200)
    c = cost()
    job = s.submit(frame(0), [0, 1, 2, 3], c)
    ran = 0
    for f in range(2):
        p = s.plan_frame(frame(f), 100, c)
        ran += len(p.runs)
        assert not p.delivered and not p.missed
    p = s.plan_frame(frame(2), 100, c)
    assert ran == 2 and len(p.runs) == 1 and not p.delivered
    assert [(m.job, m.due) for m in p.missed] == [(job, fr(2))]


def test_a_dip_in_one_frame_does_not_abandon_a_job_the_later_frames_finish():  # :985
    s = Scheduler(FixedLatency(2), "drop", 200)
    c = cost()
    job = s.submit(frame(0), [0, 1, 2, 3], c)
    ran = 0
    for f, b in [(0, 100), (1, 200)]:
        p = s.plan_frame(frame(f), b, c)
        ran += len(p.runs)
        assert not p.missed
    p = s.plan_frame(frame(2), 200, c)
    ran += len(p.runs)
    assert ran == 4 and [d.job for d in p.delivered] == [job]


def test_an_abandoned_job_frees_the_job_behind_it():  # :1009
    s = Scheduler(FixedLatency(1), "drop", 100)
    c = cost()
    a = s.submit(frame(0), [0, 1, 2], c)
    b = s.submit(frame(0), [3], c)
    p0 = s.plan_frame(frame(0), 100, c)
    assert [r.job for r in p0.runs] == [b]
    assert p0.missed == [Missed(a, 0, fr(1), "drop")]
    p1 = s.plan_frame(frame(1), 100, c)
    assert [d.job for d in p1.delivered] == [b]
    for f in range(2, 5):
        p = s.plan_frame(frame(f), 100, c)
        assert not p.delivered and not p.missed


def test_a_late_lone_job_is_abandoned_once_a_job_queues_behind_it():  # :1044
    s = Scheduler(FixedLatency(2), "drop", 100)
    c = cost()
    a = s.submit(frame(0), [0, 1, 2, 3], c)
    p0 = s.plan_frame(frame(0), 100, c)
    assert runs(p0) == [(a, 0)] and not p0.missed
    b = s.submit(frame(1), [4], c)
    p1 = s.plan_frame(frame(1), 100, c)
    assert runs(p1) == [(b, 0)]
    assert p1.missed == [Missed(a, 0, fr(2), "drop")]
    delivered = []
    for f in range(2, 6):
        p = s.plan_frame(frame(f), 100, c)
        assert not p.runs and not p.missed, f
        delivered += [(f, d.job) for d in p.delivered]
    assert delivered == [(3, b)]


def test_a_job_whose_deadline_has_passed_is_not_waiting_behind_a_late_one():  # :1086
    s = Scheduler(FixedLatency(2), "drop", 100)
    c = cost()
    a = s.submit(frame(2), [0, 1, 2, 3], c)
    b = s.submit(frame(0), [4], c)
    p3 = s.plan_frame(frame(3), 100, c)
    assert [r.job for r in p3.runs] == [a] and [m.job for m in p3.missed] == [b]
    p4 = s.plan_frame(frame(4), 100, c)
    assert len(p4.runs) == 1 and [(m.job, m.due) for m in p4.missed] == [(a, fr(4))]
    assert not p4.delivered


def test_miss_policy_is_carried_through():  # :1114
    s = Scheduler(SameFrame(), "drop", 50)
    c = cost()
    s.submit(frame(0), [0], c)
    assert s.plan_frame(frame(0), 50, c).missed[0].policy == "drop"


def test_budget_is_never_exceeded_and_leftover_is_not_given_to_a_later_job():  # :1123
    c = cost()
    c.record(2, 40)
    s = Scheduler(FixedLatency(5), "drop", 150)
    a = s.submit(frame(0), [0, 1], c)
    b = s.submit(frame(1), [2], c)
    p = s.plan_frame(frame(1), 150, c)
    assert runs(p) == [(a, 0)] and p.spent_estimate == 100 and p.spent_estimate <= p.budget
    p = s.plan_frame(frame(2), 150, c)
    assert runs(p) == [(a, 1), (b, 0)] and p.spent_estimate == 140
    assert sum(c.estimate(r.slice) for r in p.runs) == p.spent_estimate


def test_budget_holds_across_many_frames():  # :1157
    c = cost()
    s = Scheduler(FixedLatency(20), "drop", 250)
    for i in range(4):
        s.submit(frame(i), [0, 1, 2], c)
    for f in range(25):
        p = s.plan_frame(frame(f), 250, c)
        assert p.spent_estimate <= 250 and len(p.runs) <= 2 and not p.missed, f
    assert s.pending() == 0


def test_oldest_job_gets_slices_first_even_with_the_later_deadline():  # :1177
    s = Scheduler(FixedLatency(5), "drop", 100)
    c = cost()
    first = s.submit(frame(3), [0], c)
    second = s.submit(frame(1), [0], c)
    assert first < second
    p = s.plan_frame(frame(3), 100, c)
    assert [r.job for r in p.runs] == [first]


def test_later_job_never_gets_a_slice_while_an_earlier_job_has_slices_left():  # :1196
    c = cost()
    c.record(10, 10)
    c.record(11, 10)
    s = Scheduler(FixedLatency(6), "drop", 250)
    a = s.submit(frame(0), [0, 1, 2, 3], c)
    b = s.submit(frame(1), [10, 11], c)
    a_left, b_ran = 4, 0
    for f in range(1, 8):
        p = s.plan_frame(frame(f), 250, c)
        for r in p.runs:
            if r.job == a:
                a_left -= 1
            else:
                assert r.job == b and a_left == 0, f
                b_ran += 1
        jobs = [r.job for r in p.runs]
        if a in jobs and b in jobs:
            assert max(i for i, j in enumerate(jobs) if j == a) < jobs.index(b)
    assert (a_left, b_ran) == (0, 2)


def test_a_missed_job_does_not_hold_up_the_jobs_after_it():  # :1234
    c = cost()
    s = Scheduler(SameFrame(), "drop", 1000)
    a = s.submit(frame(0), [0, 1], c)
    b = s.submit(frame(1), [0], c)
    p = s.plan_frame(frame(1), 1000, c)
    assert [r.job for r in p.runs] == [b] and [m.job for m in p.missed] == [a]
    assert [d.job for d in p.delivered] == [b]


def test_equal_deadlines_go_to_the_lower_job_id():  # :1251
    s = Scheduler(SameFrame(), "drop", 100)
    c = cost()
    first = s.submit(frame(0), [0], c)
    s.submit(frame(0), [0], c)
    p = s.plan_frame(frame(0), 100, c)
    assert [r.job for r in p.runs] == [first] and len(p.delivered) == 1 and len(p.missed) == 1


def test_same_frame_fitting_job_is_delivered_in_the_same_plan():  # :1264
    s = Scheduler(SameFrame(), "hold_previous", 200)
    c = cost()
    job = s.submit(frame(4), [0, 1], c)
    p = s.plan_frame(frame(4), 200, c)
    assert len(p.runs) == 2 and p.delivered == [Delivery(job, 4)] and not p.missed
    assert s.pending() == 0


def test_same_frame_oversized_job_is_missed_in_the_same_plan():  # :1282
    c = cost()
    s = Scheduler(SameFrame(), "drop", 150)
    job = s.submit(frame(4), [0, 1], c)
    p = s.plan_frame(frame(4), 150, c)
    assert len(p.runs) == 1 and p.spent_estimate == 100 and not p.delivered
    assert p.missed == [Missed(job, 4, fr(4), "drop")] and s.pending() == 0
    s = Scheduler(SameFrame(), "drop", 150)
    job = s.submit(frame(4), [0, 1], c)
    nxt = s.submit(frame(4), [2], c)
    p = s.plan_frame(frame(4), 150, c)
    assert [r.job for r in p.runs] == [nxt]
    assert p.missed == [Missed(job, 4, fr(4), "drop")] and len(p.delivered) == 1


def test_on_beat_deadline_follows_the_grid():  # :1314
    c = cost()
    s = Scheduler(on_beat(50), "drop", 1000)
    job = s.submit(at(250), [0, 1], c)
    assert s.due(job) == beat(1000)
    assert len(s.plan_frame(at(250), 1000, c).runs) == 2
    for start in [500, 750, 999]:
        p = s.plan_frame(at(start), 1000, c)
        assert not p.delivered and not p.missed, start
    assert s.pending() == 1
    p = s.plan_frame(at(1000), 1000, c)
    assert p.delivered == [Delivery(job, 0)] and s.pending() == 0


def test_on_beat_skips_to_the_next_beat_when_work_does_not_fit_before_it():  # :1341
    c = cost()
    s = Scheduler(on_beat(50), "drop", 1000)
    job = s.submit(at(900), [0], c)
    s.plan_frame(at(900), 1000, c)
    for start in (1000, 1999):
        p = s.plan_frame(at(start), 1000, c)
        assert not p.delivered and not p.missed
    p = s.plan_frame(at(2000), 1000, c)
    assert [d.job for d in p.delivered] == [job]


def test_on_beat_multi_frame_job_gets_a_beat_it_can_make():  # :1359
    c = cost()
    s = Scheduler(on_beat(0), "drop", 100)
    job = s.submit(frame(0), [0, 1, 2], c)
    assert s.due(job) == beat(3000)
    for f in range(3):
        p = s.plan_frame(frame(f), 100, c)
        assert len(p.runs) == 1 and not p.delivered and not p.missed, f
    p = s.plan_frame(frame(3), 100, c)
    assert [d.job for d in p.delivered] == [job] and not p.missed


def test_on_beat_work_queued_ahead_pushes_the_beat_later():  # :1380
    c = cost()
    alone = Scheduler(on_beat(0), "drop", 100)
    assert alone.due(alone.submit(frame(0), [3], c)) == beat(1000)
    s = Scheduler(on_beat(0), "drop", 100)
    a = s.submit(frame(0), [0, 1, 2], c)
    b = s.submit(frame(0), [3], c)
    assert s.due(a) == beat(3000) and s.due(b) == beat(4000)
    delivered = []
    for f in range(5):
        p = s.plan_frame(frame(f), 100, c)
        assert not p.missed, f
        delivered += [(f, d.job) for d in p.delivered]
    assert delivered == [(3, a), (4, b)]


def test_on_beat_job_no_frame_can_run_is_decided_at_its_beat():  # :1405
    c = cost()
    s = Scheduler(on_beat(0), "hold_previous", 50)
    job = s.submit(at(0), [0], c)
    assert s.due(job) == beat(1000)
    p = s.plan_frame(at(500), 50, c)
    assert not p.runs and not p.missed and not p.delivered
    p = s.plan_frame(at(1000), 50, c)
    assert not p.runs and not p.delivered
    assert [(m.job, m.due) for m in p.missed] == [(job, beat(1000))]
    s = Scheduler(on_beat(0), "hold_previous", 50)
    job = s.submit(at(0), [0], c)
    s.plan_frame(at(500), 50, c)
    p = s.plan_frame(at(1000), 100, c)
    assert len(p.runs) == 1 and [d.job for d in p.delivered] == [job]


def test_on_beat_lone_job_a_dip_makes_late_is_kept_and_delivered_on_its_beat():  # :1436
    c = cost()
    s = Scheduler(on_beat(0), "hold_previous", 100)
    job = s.submit(frame(0), [0, 1, 2], c)
    assert s.due(job) == beat(3000)
    for f, b, ran in [(0, 0, 0), (1, 0, 0), (2, 100, 1)]:
        p = s.plan_frame(frame(f), b, c)
        assert len(p.runs) == ran and not p.missed and not p.delivered, f
    p = s.plan_frame(frame(3), 200, c)
    assert len(p.runs) == 2 and [d.job for d in p.delivered] == [job] and not p.missed


def test_on_beat_job_queued_behind_a_late_one_is_placed_as_the_plan_runs_it():  # :1460
    c = cost()
    s = Scheduler(on_beat(0), "drop", 100)
    a = s.submit(frame(0), [0, 1, 2], c)
    for f in range(2):
        assert not s.plan_frame(frame(f), 0, c).missed, f
    b = s.submit(frame(2), [3], c)
    assert s.due(b) == beat(3000)
    p2 = s.plan_frame(frame(2), 100, c)
    assert [r.job for r in p2.runs] == [b]
    assert p2.missed == [Missed(a, 0, beat(3000), "drop")]
    p3 = s.plan_frame(frame(3), 100, c)
    assert [d.job for d in p3.delivered] == [b] and not p3.missed


def test_on_beat_miss_is_reported_at_the_beat():  # :1496
    c = cost()
    s = Scheduler(on_beat(0), "hold_previous", 1000)
    job = s.submit(at(0), [0], c)
    assert not s.plan_frame(at(500), 50, c).missed
    p = s.plan_frame(at(1000), 50, c)
    assert [m.job for m in p.missed] == [job]


def test_on_beat_frame_starting_after_the_beat_still_runs_and_delivers():  # :1511
    c = cost()
    s = Scheduler(on_beat(0), "drop", 200)
    job = s.submit(at(10), [0, 1], c)
    assert s.due(job) == beat(1000)
    p = s.plan_frame(at(10), 100, c)
    assert len(p.runs) == 1 and not p.missed
    p = s.plan_frame(at(1010), 100, c)
    assert len(p.runs) == 1 and [d.job for d in p.delivered] == [job] and not p.missed


def test_on_beat_result_seen_after_a_skipped_beat_frame_is_missed():  # :1531
    c = cost()
    s = Scheduler(on_beat(0), "hold_previous", 100)
    job = s.submit(at(10), [0], c)
    assert len(s.plan_frame(at(10), 100, c).runs) == 1
    p = s.plan_frame(at(2010), 100, c)
    assert not p.delivered and [m.job for m in p.missed] == [job]


def test_a_tempo_change_moves_only_the_deadlines_fixed_after_it():  # :1545
    c = cost()
    s = Scheduler(on_beat(0), "drop", 1000)
    a = s.submit(at(0), [0], c)
    assert s.due(a) == beat(1000)
    s.plan_frame(at(0), 1000, c)
    s.replace_beat_grid(500, BeatGrid(500, 300))
    assert s.due(a) == beat(1000)
    b = s.submit(at(600), [1], c)
    assert s.due(b) == beat(800)
    p = s.plan_frame(at(600), 1000, c)
    assert not p.delivered and not p.missed
    assert [d.job for d in s.plan_frame(at(800), 1000, c).delivered] == [b]
    p = s.plan_frame(at(1000), 1000, c)
    assert [d.job for d in p.delivered] == [a] and not p.missed


def test_slice_larger_than_the_budget_is_never_run_and_its_job_is_missed():  # :1576
    c = cost()
    c.record(0, 500)
    s = Scheduler(FixedLatency(1), "drop", 499)
    job = s.submit(frame(0), [0], c)
    p0 = s.plan_frame(frame(0), 499, c)
    assert not p0.runs and p0.spent_estimate == 0 and not p0.missed and not p0.delivered
    p1 = s.plan_frame(frame(1), 499, c)
    assert not p1.runs and not p1.delivered
    assert [(m.job, m.due) for m in p1.missed] == [(job, fr(1))] and s.pending() == 0


def test_a_slice_no_frame_holds_runs_the_slices_before_it_alone_and_is_abandoned():  # :1601
    c = cost()
    c.record(0, 500)
    s = Scheduler(FixedLatency(1), "drop", 499)
    job = s.submit(frame(0), [1, 0], c)
    p0 = s.plan_frame(frame(0), 499, c)
    assert runs(p0) == [(job, 0)] and not p0.missed and not p0.delivered
    p1 = s.plan_frame(frame(1), 499, c)
    assert not p1.runs and not p1.delivered and [m.job for m in p1.missed] == [job]
    s = Scheduler(FixedLatency(1), "drop", 499)
    late = s.submit(frame(0), [1, 0], c)
    nxt = s.submit(frame(0), [2], c)
    p0 = s.plan_frame(frame(0), 499, c)
    assert [r.job for r in p0.runs] == [nxt]
    assert [(m.job, m.due) for m in p0.missed] == [(late, fr(1))]


def test_job_past_its_deadline_gets_no_slices():  # :1639
    s = Scheduler(SameFrame(), "drop", 1000)
    c = cost()
    job = s.submit(frame(0), [0], c)
    p = s.plan_frame(frame(1), 1000, c)
    assert not p.runs and [m.job for m in p.missed] == [job]


def test_finished_job_seen_after_its_frame_is_missed_not_delivered_late():  # :1651
    s = Scheduler(FixedLatency(1), "hold_previous", 100)
    c = cost()
    job = s.submit(frame(0), [0], c)
    assert len(s.plan_frame(frame(0), 100, c).runs) == 1
    p2 = s.plan_frame(frame(2), 100, c)
    assert not p2.delivered and [m.job for m in p2.missed] == [job] and s.pending() == 0


def test_slices_of_a_job_run_in_order_across_frames():  # :1671
    s = Scheduler(FixedLatency(3), "drop", 100)
    c = cost()
    s.submit(frame(0), [7, 8, 9], c)
    seen = []
    for f in range(3):
        seen += [(r.position, r.slice) for r in s.plan_frame(frame(f), 100, c).runs]
    assert seen == [(0, 7), (1, 8), (2, 9)]
    assert len(s.plan_frame(frame(3), 100, c).delivered) == 1


def _lone_stream(seeded, frames):
    """One input at a time (a job submitted only once the one before left):
    20 slices of 100 us, a 500 us budget, latency 10, each slice's estimate
    seeded with a full window of `seeded` us; a slice run in a frame is
    measured at 100 us in the next (schedule.rs:1690-1760)."""
    job = list(range(20))
    c = CostModel(2000)  # the default estimator: 0.9 quantile of the last 32
    for _ in range(32):
        for sl in job:
            c.record(sl, seeded)
    s = Scheduler(FixedLatency(10), "hold_previous", 500)
    ran = delivered = missed = early = 0
    last_miss, busy, readback = None, False, []
    for i in range(frames):
        for sl in readback:
            c.record(sl, 100)
        readback = []
        if not busy:
            s.submit(frame(i), job, c)
            busy = True
        p = s.plan_frame(frame(i), 500, c)
        assert p.spent_estimate <= p.budget, i
        ran += len(p.runs)
        readback += [r.slice for r in p.runs]
        for d in p.delivered:
            assert d.input + 10 == i
        for m in p.missed:
            last_miss = i
            early += m.due != fr(i)
        delivered += len(p.delivered)
        missed += len(p.missed)
        if p.delivered or p.missed:
            busy = False
    return ran, delivered, missed, early, last_miss, [c.estimate(sl) for sl in job]


def test_a_lone_job_estimated_far_above_its_cost_runs_and_brings_the_estimates_down():  # :1765
    ran, delivered, missed, early, last_miss, est = _lone_stream(400, 3000)
    assert ran > 0 and all(e == 100 for e in est) and early == 0
    assert (delivered, missed, last_miss) == (243, 29, 318)
    _, delivered, missed, _, _, _ = _lone_stream(100, 3000)
    assert (delivered, missed) == (272, 0)


def test_simulated_session_delivers_on_its_beats_through_budget_dips_and_a_tempo_change():
    """schedule.rs:1797: 60 Hz for 600 frames on 120 bpm beats changing to 150
    bpm at frame 300; a job of 16, 24 or 30 slices of 1 ms every fourth frame;
    a slow render every tenth frame (5 ms) and 2 ms frames 450-469. The
    scheduler is deterministic, so the figures are exact."""
    FRAME_US, FRAMES, EXPECTED, CHANGE = 16667, 600, 8000, 300
    SLOW = range(450, 470)
    change_at = CHANGE * FRAME_US
    c = CostModel(1000, MeanPlusSigmas(1.0, 0.0))
    s = Scheduler(OnBeat(2000, BeatGrid(0, 500000)), "hold_previous", EXPECTED)
    sizes = [16, 24, 30]
    fixed, ran = {}, {}
    delivered = missed = early = wasted = 0
    missed_in = []
    for i in range(FRAMES):
        f = FrameInfo(i, i * FRAME_US, FRAME_US)
        if i == CHANGE:
            s.replace_beat_grid(change_at, BeatGrid(change_at, 400000))
        if i % 4 == 0:
            job = s.submit(f, list(range(sizes[(i // 4) % 3])), c)
            due = s.due(job)
            assert due.kind == "beat"
            fixed[job] = (due.at, i >= CHANGE)
        b = 2000 if i in SLOW else 5000 if i % 10 == 9 else EXPECTED
        p = s.plan_frame(f, b, c)
        assert p.spent_estimate <= p.budget, i
        for r in p.runs:
            ran[r.job] = ran.get(r.job, 0) + 1
        for d in p.delivered:
            due, _ = fixed[d.job]
            assert f.start >= due and f.start - due < f.period, i
            delivered += 1
        for m in p.missed:
            due, _ = fixed[m.job]
            assert m.due == beat(due), i
            assert f.start < due or f.start - due < f.period, i
            early += f.start < due
            wasted += ran.get(m.job, 0)
            missed_in.append(i)
            missed += 1
    for job, (due, after) in fixed.items():
        origin, step = (change_at, 400000) if after else (0, 500000)
        assert due >= origin and (due - origin) % step == 0, job
    submitted, pending = len(fixed), s.pending()
    assert submitted == delivered + missed + pending
    assert all(i in SLOW for i in missed_in), missed_in
    assert (submitted, delivered, missed, pending, early, wasted) == (150, 144, 3, 3, 2, 25)


def test_frames_are_filled_by_the_planning_estimate():  # :1929
    from beatlm_b200.cost import FrameScaled, WARM_SAMPLES
    c = CostModel(100, FrameScaled(4, 2, 0.9))
    for sl in range(4):
        for _ in range(WARM_SAMPLES):
            c.record(sl, 100)
    c.record_frame(400, 800)
    c.record_frame(400, 800)
    assert c.estimate(0) == 100 and c.planning_estimate(0) == 200
    s = Scheduler(FixedLatency(5), "drop", 450)
    s.submit(frame(0), [0, 1, 2, 3], c)
    p = s.plan_frame(frame(0), 450, c)
    assert len(p.runs) == 2 and p.spent_estimate == 400
    assert sum(c.planning_estimate(r.slice) for r in p.runs) == p.spent_estimate


class _Sequence:
    """xorshift64*: the reference test's fixed pseudo-random sequence."""

    def __init__(self, state):
        self.s = state

    def unit(self):
        m = (1 << 64) - 1
        self.s ^= self.s >> 12
        self.s = (self.s ^ (self.s << 25)) & m
        self.s ^= self.s >> 27
        x = (self.s * 0x2545F4914F6CDD1D) & m
        return (x >> 11) / float(1 << 53)


def _fma(a, b, c):
    """a * b + c rounded once (the reference's mul_add)."""
    from fractions import Fraction
    return float(Fraction(a) * Fraction(b) + Fraction(c))


def _clustered(estimator):
    """schedule.rs:1990-2070: 3000 frames of a 4 ms budget over an endless
    queue of 48-slice jobs whose slices are slow together by frame."""
    FRAMES, WARM, BUDGET, SLICES = 3000, 400, 4000, 48
    base = lambda sl: 100 + (sl * 37 % 7) * 20
    c = CostModel(160, estimator)
    s = Scheduler(FixedLatency(40), "drop", BUDGET)
    job = list(range(SLICES))
    queued = 0
    draw = _Sequence(0x9E3779B97F4A7C15)
    counted = ran = over = 0
    fills = []
    for i in range(FRAMES):
        f = frame(i)
        while queued < len(job):
            s.submit(f, job, c)
            queued += len(job)
        p = s.plan_frame(f, BUDGET, c)
        assert p.spent_estimate <= p.budget and not p.missed, i
        queued -= len(p.runs)
        slowdown = 2.0 + draw.unit() if draw.unit() < 0.06 else 1.0
        measured, ratio, samples = 0, [0, 0], []
        for r in p.runs:
            own = 2.0 if draw.unit() < 0.15 else 1.0
            jitter = _fma(0.1, draw.unit(), 0.95)
            us = int(round_half_away(base(r.slice) * slowdown * own * jitter))
            planned = c.frame_estimate(r.slice)
            if planned is not None:
                ratio = [ratio[0] + planned, ratio[1] + us]
            samples.append((r.slice, us))
            measured += us
        for sl, us in samples:
            c.record(sl, us)
        c.record_frame(ratio[0], ratio[1])
        if i >= WARM:
            counted += 1
            ran += len(p.runs)
            over += measured > BUDGET
            fills.append(measured / BUDGET)
    fills.sort()
    return ran / counted, over / counted, fills[len(fills) // 2]


def round_half_away(x):
    import math
    return math.floor(x + 0.5) if x >= 0 else -math.floor(-x + 0.5)


def test_with_clustered_slowdowns_the_frame_scale_packs_more_than_quantiles():  # :2080
    from beatlm_b200.cost import FrameScaled, WindowedQuantile
    q = 0.9
    qs = _clustered(WindowedQuantile(32, q))
    med = _clustered(WindowedQuantile(32, 0.5))
    sc = _clustered(FrameScaled(32, 64, q))
    print("slices/frame, over, median fill: quantiles %s medians %s frame-scaled %s"
          % (qs, med, sc))
    assert qs[2] < 0.7
    assert med[1] > 0.5
    assert sc[1] <= 1.0 - q
    assert sc[0] > 1.3 * qs[0]
    assert sc[2] > qs[2] + 0.15
