"""The slice cost model (bl_cost_*, beatlm_b200.cost) against the reference's
own cases for its CostModel (crates/beatlm-core/src/cost.rs:1040-1705): the
same measurements must give the same estimates, since the scheduler plans
with them. Host logic only; no GPU."""
import math

import pytest

from beatlm_b200.cost import (MAX_WINDOW, WARM_SAMPLES, CappedDeviation, CostError, CostModel,
                              FrameScaled, Measured, MeanPlusSigmas, WarmingUp, WindowedQuantile,
                              default_estimator, micros_nearest)

S = 7
U64_MAX = (1 << 64) - 1


def mean_sigmas(prior, alpha, sigmas):
    return CostModel(prior, MeanPlusSigmas(alpha, sigmas))


def quantile(prior, window, q):
    return CostModel(prior, WindowedQuantile(window, q))


def capped(prior, alpha, sigmas, cap):
    return CostModel(prior, CappedDeviation(alpha, sigmas, cap))


def frame_scaled(prior, window, frame_window, q):
    return CostModel(prior, FrameScaled(window, frame_window, q))


def rejected(estimator) -> str:
    with pytest.raises(CostError) as e:
        CostModel(0, estimator)
    return e.value.kind


def frames(m, pairs):
    for predicted, measured in pairs:
        m.record_frame(predicted, measured)


# ------------------------------------------------------------ validation

def test_invalid_alpha_is_rejected():  # cost.rs:1048
    for alpha in [0.0, -0.5, 1.5, math.nan, math.inf]:
        assert rejected(MeanPlusSigmas(alpha, 1.0)) == "InvalidAlpha"
        assert rejected(CappedDeviation(alpha, 1.0, 1.0)) == "InvalidAlpha"


def test_invalid_sigmas_is_rejected():  # cost.rs:1068
    for sigmas in [-1.0, math.nan, math.inf]:
        assert rejected(MeanPlusSigmas(0.5, sigmas)) == "InvalidSigmas"
        assert rejected(CappedDeviation(0.5, sigmas, 1.0)) == "InvalidSigmas"


def test_invalid_window_and_quantile_are_rejected():  # cost.rs:1088
    for window in [0, MAX_WINDOW + 1]:
        assert rejected(WindowedQuantile(window, 0.5)) == "InvalidWindow"
    for q in [-0.1, 1.1, math.nan, math.inf]:
        assert rejected(WindowedQuantile(8, q)) == "InvalidQuantile"
    for window, q in [(1, 0.0), (MAX_WINDOW, 1.0)]:
        CostModel(0, WindowedQuantile(window, q))


def test_invalid_cap_is_rejected():  # cost.rs:1124
    for cap in [-0.1, math.nan, math.inf]:
        assert rejected(CappedDeviation(0.5, 1.0, cap)) == "InvalidCap"


def test_invalid_frame_scaled_parameters_are_rejected():  # cost.rs:1401
    for window in [0, MAX_WINDOW + 1]:
        assert rejected(FrameScaled(window, 8, 0.9)) == "InvalidWindow"
    for frame_window in [0, MAX_WINDOW + 1]:
        assert rejected(FrameScaled(8, frame_window, 0.9)) == "InvalidFrameWindow"
    for q in [-0.1, 1.1, math.nan, math.inf]:
        assert rejected(FrameScaled(8, 8, q)) == "InvalidQuantile"
    for window, frame_window, q in [(1, 1, 0.0), (MAX_WINDOW, MAX_WINDOW, 1.0)]:
        CostModel(0, FrameScaled(window, frame_window, q))


def test_the_default_is_the_windowed_quantile_of_32_at_0_9():  # cost.rs:416-425
    assert default_estimator() == WindowedQuantile(32, 0.9)
    assert CostModel(5).estimator == WindowedQuantile(32, 0.9)


# ------------------------------------------------------------ estimates

def test_prior_is_used_without_samples():  # cost.rs:1139
    for m in [mean_sigmas(123, 0.5, 2.0), quantile(123, 8, 0.9), capped(123, 0.5, 2.0, 0.5),
              frame_scaled(123, 8, 4, 0.9)]:
        assert m.estimate(S) == 123 and m.samples(S) == 0
        m.record(1, 5)  # another slice's measurement leaves this one at the prior
        assert m.estimate(S) == 123


def test_the_model_reports_its_estimator():  # cost.rs:1155
    e = WindowedQuantile(4, 0.5)
    assert CostModel(0, e).estimator == e


def test_alpha_one_tracks_the_last_sample():  # cost.rs:1164
    m = mean_sigmas(1, 1.0, 3.0)
    for x in [100, 400, 250]:
        m.record(S, x)
    assert m.estimate(S) == 250


def test_estimate_pads_the_mean_by_sigmas():  # cost.rs:1173
    m = mean_sigmas(1, 0.5, 2.0)
    m.record(S, 100)
    assert m.estimate(S) == 100
    m.record(S, 120)
    m.record(S, 80)
    assert m.estimate(S) == 129  # mean 95, variance 275: ceil(95 + 2 sqrt(275))


def test_samples_count_per_slice():  # cost.rs:1185
    for m in [mean_sigmas(1, 0.5, 0.0), quantile(1, 3, 0.5), capped(1, 0.5, 0.0, 0.0),
              frame_scaled(1, 3, 2, 0.5)]:
        m.record(S, 10)
        m.record(S, 10)
        m.record(8, 10)
        assert (m.samples(S), m.samples(8), m.samples(9)) == (2, 1, 0)


def test_huge_estimates_saturate():  # cost.rs:1202
    for m in [mean_sigmas(0, 1.0, 0.0), capped(0, 1.0, 0.0, 0.0), quantile(0, 2, 1.0)]:
        m.record(S, U64_MAX)
        assert m.estimate(S) == U64_MAX


def test_capped_pads_by_the_smaller_of_sigmas_and_the_cap():  # cost.rs:1217
    for cap, expected in [(1.0, 129), (0.1, 105), (0.0, 95)]:
        m = capped(1, 0.5, 2.0, cap)
        for x in [100, 120, 80]:
            m.record(S, x)
        assert m.estimate(S) == expected, cap


def test_quantile_reads_the_nearest_rank_of_the_window():  # cost.rs:1240
    for q, expected in [(0.0, 10), (0.2, 10), (0.5, 30), (0.9, 50), (1.0, 50)]:
        m = quantile(1, 8, q)
        for x in [50, 10, 40, 20, 30]:
            m.record(S, x)
        assert m.estimate(S) == expected, q


def test_a_whole_rank_is_not_pushed_up_by_rounding():  # cost.rs:1255 (through the model)
    # 0.55 of 100 is rank 55, 0.9 of 32 rank 29
    m = quantile(1, 100, 0.55)
    for x in range(1, 101):
        m.record(S, x)
    assert m.estimate(S) == 55
    m = quantile(1, 32, 0.9)
    for x in range(1, 33):
        m.record(S, x)
    assert m.estimate(S) == 29


def test_quantile_forgets_what_leaves_the_window():  # cost.rs:1264
    m = quantile(1, 3, 1.0)
    for x in [900, 10, 20]:
        m.record(S, x)
    assert m.estimate(S) == 900
    m.record(S, 30)
    assert m.estimate(S) == 30
    m.record(S, 5)
    assert m.estimate(S) == 30
    m.record(S, 6)
    m.record(S, 7)
    assert m.estimate(S) == 7 and m.samples(S) == 7


def test_a_window_of_one_tracks_the_last_sample():  # cost.rs:1282
    m = quantile(1, 1, 0.9)
    m.record(S, 100)
    m.record(S, 400)
    assert m.estimate(S) == 400


def test_windows_are_per_slice():  # cost.rs:1290
    m = quantile(1, 2, 1.0)
    m.record(S, 100)
    m.record(8, 5)
    assert (m.estimate(S), m.estimate(8)) == (100, 5)


def test_estimates_change_only_through_record():  # cost.rs:1299
    for m in [mean_sigmas(1, 0.2, 2.0), quantile(1, 8, 0.9), capped(1, 0.2, 2.0, 0.5)]:
        m.record(S, 100)
        m.record(S, 300)
        before = m.estimate(S)
        assert m.estimate(S) == before and m.clone().estimate(S) == before


def _series(i):
    return 100 + (i * 37) % 11 * 13


def test_identical_measurements_give_identical_estimates():  # cost.rs:1314
    for e in [MeanPlusSigmas(0.2, 2.0), WindowedQuantile(6, 0.9), CappedDeviation(0.2, 2.0, 0.5)]:
        a, b = CostModel(9, e), CostModel(9, e)
        for i in range(40):
            a.record(S, _series(i))
            b.record(S, _series(i))
            assert a.estimate(S) == b.estimate(S)


def _noisy(i):
    return 8000 if i % 10 == 9 else 1000 + (i % 5) * 10


def _peak_estimate(m):
    peak = 0
    for i in range(200):
        m.record(S, _noisy(i))
        if i >= 30:
            peak = max(peak, m.estimate(S))
    return peak


def test_noise_inflates_mean_plus_sigmas_but_not_the_robust_estimators():  # cost.rs:1365
    inflated = _peak_estimate(mean_sigmas(1, 0.05, 2.0))
    windowed = _peak_estimate(quantile(1, 20, 0.9))
    bounded = _peak_estimate(capped(1, 0.05, 2.0, 0.5))
    assert windowed <= 1040 and bounded <= 3000 and inflated >= 6000
    assert windowed < bounded < inflated


# ------------------------------------------------------------ frame scale

def test_frame_scaled_estimates_the_median_and_warms_up_at_the_frame_quantile():  # cost.rs:1425
    m = frame_scaled(123, 8, 3, 0.9)
    assert m.estimate(S) == 123 and m.planning_estimate(S) == 123
    for x in [50, 10, 40, 20, 30]:
        m.record(S, x)
    assert m.estimate(S) == 30
    assert m.frame_scale() == WarmingUp(0, 3)
    assert m.planning_estimate(S) == 50
    frames(m, [(100, 150), (100, 150)])
    assert m.frame_scale() == WarmingUp(2, 3)
    assert m.planning_estimate(S) == 50
    frames(m, [(100, 150)])
    assert m.frame_scale() == Measured(1.5)
    assert m.planning_estimate(S) == 45 and m.estimate(S) == 30
    assert m.planning_estimate(1) == 123
    assert m.frames_recorded() == 3


def test_the_frame_scale_is_the_nearest_rank_of_the_last_frames():  # cost.rs:1463
    m = frame_scaled(1, 4, 4, 0.75)
    frames(m, [(100, 150), (100, 120), (100, 200), (100, 110)])
    assert m.frame_scale() == Measured(1.5)
    frames(m, [(100, 130)])
    assert m.frame_scale() == Measured(1.3)
    for q, expected in [(0.0, 1.1), (1.0, 2.0)]:
        m = frame_scaled(1, 4, 4, q)
        frames(m, [(100, 150), (100, 120), (100, 200), (100, 110)])
        assert m.frame_scale() == Measured(expected), q
    m = frame_scaled(1, 4, 100, 0.55)
    frames(m, [(100, 100 + i) for i in range(1, 101)])
    assert m.frame_scale() == Measured(1.55)


def test_the_planning_estimate_is_the_median_times_the_scale_rounded_up():  # cost.rs:1486
    m = frame_scaled(1, 5, 1, 1.0)
    for _ in range(5):
        m.record(S, 101)
    frames(m, [(1000, 1234)])
    assert m.planning_estimate(S) == 125 and m.planning_estimate(S) >= m.estimate(S)
    m = frame_scaled(1, 5, 1, 1.0)
    for _ in range(5):
        m.record(S, 100)
    frames(m, [(1000, 1100)])
    assert m.planning_estimate(S) == 110  # 100 x 1.1 is 110, not 111


def test_the_frame_scale_never_plans_a_slice_below_its_median():  # cost.rs:1505
    m = frame_scaled(1, 8, 4, 0.9)
    for _ in range(5):
        m.record(S, 200)
    frames(m, [(400, 200)] * 4)
    assert m.frame_scale() == Measured(1.0)
    assert m.planning_estimate(S) == m.estimate(S) == 200


def test_a_frame_counts_as_much_as_its_predicted_time():  # cost.rs:1518
    m = frame_scaled(1, 4, 25, 0.9)
    frames(m, [(4000, 4800)] * 20)
    frames(m, [(20, 200)] * 5)
    assert m.frame_scale() == Measured(1.2) and m.frames_recorded() == 25
    unweighted = frame_scaled(1, 4, 25, 0.9)
    frames(unweighted, [(100, 120)] * 20)
    frames(unweighted, [(100, 1000)] * 5)
    assert unweighted.frame_scale() == Measured(10.0)


def test_a_frame_predicted_at_zero_is_not_recorded():  # cost.rs:1537
    m = frame_scaled(1, 4, 2, 0.9)
    frames(m, [(0, 500), (0, 0)])
    assert m.frames_recorded() == 0 and m.frame_scale() == WarmingUp(0, 2)
    frames(m, [(100, 0), (100, 0)])
    assert m.frame_scale() == Measured(1.0)


def test_the_other_estimators_ignore_frames_and_plan_at_their_estimate():  # cost.rs:1554
    for m in [mean_sigmas(1, 0.2, 2.0), quantile(1, 8, 0.9), capped(1, 0.2, 2.0, 0.5)]:
        for x in [100, 300, 200, 900]:
            m.record(S, x)
        before = m.clone()
        frames(m, [(100, 300)] * 50)
        assert m.frame_scale() is None and m.frames_recorded() == 0
        assert m.estimate(S) == before.estimate(S) == m.planning_estimate(S)
        assert m.planning_estimate(1) == 1


def test_calibration_does_not_seed_the_frame_scaled_median():  # cost.rs:1574
    m = frame_scaled(1, 32, 1, 0.9)
    for _ in range(20):
        m.record_calibration(S, 100)
    assert m.samples(S) == 20 and m.frame_estimate(S) is None
    assert m.planning_estimate(S) == 100 and m.estimate(S) == 100
    m.record_frame(100, 150)
    assert m.frame_scale() == Measured(1.5)
    for _ in range(4):
        m.record(S, 300)
    assert m.frame_estimate(S) is None and m.planning_estimate(S) == 300
    m.record(S, 300)
    assert m.frame_estimate(S) == 300 and m.estimate(S) == 300
    assert m.planning_estimate(S) == 450 and m.samples(S) == 25


def test_the_frame_scale_reads_warm_slices_and_not_stale_ones():  # cost.rs:1605
    a, b = 1, 2
    m = frame_scaled(1, 32, 8, 0.9)
    for _ in range(WARM_SAMPLES):
        m.record(a, 100)
    for _ in range(10):
        m.record_calibration(b, 50)
    m.record(b, 200)
    m.record(b, 200)
    for _ in range(8):
        predicted = measured = 0
        for slice_, took in [(a, 100), (b, 200)]:
            planned = m.frame_estimate(slice_)
            if planned is not None:
                predicted += planned
                measured += took
        m.record_frame(predicted, measured)
    assert m.frame_scale() == Measured(1.0)
    assert m.planning_estimate(a) == 100 and m.estimate(b) == 50


def test_the_other_estimators_fold_calibration_as_the_loop():  # cost.rs:1641
    for e in [MeanPlusSigmas(0.2, 2.0), WindowedQuantile(6, 0.9), CappedDeviation(0.2, 2.0, 0.5)]:
        by_record, by_calibration = CostModel(9, e), CostModel(9, e)
        for i in range(40):
            by_record.record(S, _series(i))
            if i < 20:
                by_calibration.record_calibration(S, _series(i))
            else:
                by_calibration.record(S, _series(i))
            assert by_record.estimate(S) == by_calibration.estimate(S)
            assert by_calibration.frame_estimate(S) == by_calibration.estimate(S)
        assert by_record.samples(S) == by_calibration.samples(S)
        assert by_calibration.frame_estimate(3) == 9
    assert frame_scaled(9, 4, 4, 0.9).frame_estimate(S) is None


def test_frame_scaled_is_deterministic_and_changes_only_through_records():  # cost.rs:1685
    e = FrameScaled(6, 5, 0.9)
    a, b = CostModel(9, e), CostModel(9, e)
    for i in range(40):
        measured = 1000 + (i * 53) % 17 * 31
        for m in (a, b):
            m.record(S, _series(i))
            m.record_frame(1000, measured)
        assert a.planning_estimate(S) == b.planning_estimate(S)
        assert a.frame_scale() == b.frame_scale()
        assert a.clone().planning_estimate(S) == a.planning_estimate(S)


# ------------------------------------------------------------ timer feed

def test_timer_durations_round_to_the_nearest_microsecond():  # timer.rs:811-835
    assert [micros_nearest(x) for x in (0.0, 1.499, 1.5, 2.5, -3.0, math.nan)] == [0, 1, 2, 3, 0, 0]
    assert micros_nearest(1e30) == U64_MAX


def test_collected_frames_feed_the_model_under_their_kernel_index():
    from beatlm_b200.runtime import FrameTiming
    m = quantile(7, 4, 0.5)
    cal = frame_scaled(7, 8, 2, 0.9)
    for f, (t0, t1) in enumerate([(10.4, 30.6), (11.5, 29.4), (9.6, 31.49)]):
        timing = FrameTiming(f, [(0, t0), (3, t1)], [0.0, t0])
        m.record_timing(timing)
        cal.record_timing(timing, calibration=True)
    assert (m.samples(0), m.samples(3), m.samples(1)) == (3, 3, 0)
    assert (m.estimate(0), m.estimate(3), m.estimate(1)) == (10, 31, 7)  # medians of 10 12 10 / 31 29 31
    # calibration's measurements plan a frame-scaled slice but stay out of its ratio
    assert cal.samples(0) == 3 and cal.frame_estimate(0) is None
    # a planned frame records its ratio over the slices that had an estimate
    fs = frame_scaled(7, 8, 1, 1.0)
    for f in range(WARM_SAMPLES):
        fs.record_timing(FrameTiming(f, [(0, 100.0), (1, 50.0)], [0.0, 100.0]))
    planned = fs.plan_frame([0, 1, 2])
    assert planned == {0: 100, 1: 50, 2: None}
    fs.record_timing(FrameTiming(9, [(0, 150.0), (1, 75.0), (2, 999.0)], [0.0, 150.0, 225.0]),
                     planned=planned)
    assert fs.frame_scale() == Measured(1.5)
    assert fs.planning_estimate(0) == 150 and fs.planning_estimate(1) == 75


# ------------------------------------------------------------ calibration

def test_only_the_second_half_of_the_timed_frames_counts():  # calibration.rs:96
    from beatlm_b200.calibration import CALIBRATION_FRAMES, counted
    assert not counted(1) and not counted(CALIBRATION_FRAMES // 2)
    assert counted(CALIBRATION_FRAMES // 2 + 1) and counted(CALIBRATION_FRAMES)
    assert sum(counted(f) for f in range(1, CALIBRATION_FRAMES + 1)) == CALIBRATION_FRAMES // 2


def test_a_kernel_s_duration_is_the_median_of_its_counted_measurements():  # calibration.rs:106
    from beatlm_b200.calibration import CALIBRATION_FRAMES, KernelSamples
    first = KernelSamples(2)
    half = CALIBRATION_FRAMES // 2
    first.record(half, 0, 9000)
    for frame, us in [(half + 1, 100), (half + 2, 300), (half + 3, 200)]:
        first.record(frame, 0, us)
        first.record(frame, 1, us + 1)
    first.record(half + 1, 2, 5)
    assert first.durations() == [200, 201]


def test_a_kernel_never_measured_in_a_counted_frame_is_refused():  # calibration.rs:124
    from beatlm_b200.calibration import CALIBRATION_FRAMES, KernelSamples
    first = KernelSamples(2)
    first.record(CALIBRATION_FRAMES, 0, 100)
    first.record(1, 1, 100)
    with pytest.raises(RuntimeError, match="kernel 1"):
        first.durations()


def _specs():
    """A program's specs with ViT-S shapes (host-side only: nothing is built)."""
    from beatlm_b200 import _native as N
    from beatlm_b200.runtime import Spec
    ln = N.LayerNormArgs(rows=1370, dim=384)
    gemm = N.GemmArgs(m=1370, n=1152, k=384)
    attn = N.AttentionArgs(batch=1, tokens=1370, heads=6, head_dim=64, head_begin=0,
                           head_end=6, row_begin=0, row_end=1370)
    patch = N.PatchifyArgs()
    return [Spec(ln, "norm1"), Spec(gemm, "qkv"), Spec(attn, "attention"), Spec(patch, "patch")]


def test_max_parts_follow_each_kernel_s_split_dimension():  # kernel.rs:1975
    from beatlm_b200.runtime import max_parts
    assert [max_parts(s) for s in _specs()] == [1370, 11, 11, 1]


def test_program_parts_within_splits_each_kernel_for_its_duration():  # kernel.rs:2350
    from beatlm_b200.runtime import program_parts_within, split
    specs = _specs()
    # ceil(d / bound), at least 1, at most max_parts
    assert program_parts_within(specs, [3, 5, 14, 40], 5) == [1, 1, 3, 1]
    assert program_parts_within(specs, [0, 1000, 1000, 1000], 1) == [1, 11, 11, 1]
    with pytest.raises(RuntimeError, match="ZeroBound"):
        program_parts_within(specs, [1, 1, 1, 1], 0)
    with pytest.raises(RuntimeError, match="PartCounts"):
        program_parts_within(specs, [1, 1], 5)
    parts = split(specs, [1, 1, 3, 1])
    assert [s.parts for s in parts] == [1, 1, 3, 1]
    with pytest.raises(ValueError, match="already split"):
        split(parts, [1, 1, 1, 1])


# ------------------------------------------------------------ pass cost

def test_pass_cost_variants_parse_and_time_their_passes():  # pass_cost.rs:148-222
    from beatlm_b200.pass_cost import Variant
    for text in ["per-pass", "ends", "one-pass", "every:8", "one-pass-pdl"]:
        assert Variant.parse(text).name == text
    for bad in ["every:0", "every:x", "all"]:
        with pytest.raises(ValueError):
            Variant.parse(bad)
    e = Variant.parse("every:3")
    assert [e.times_pass(i, 8) for i in range(8)] == [True, False, False, True, False, False,
                                                      True, True]
    assert all(Variant("per-pass").times_pass(i, 4) for i in range(4))
    assert not any(Variant("ends").times_pass(i, 4) or Variant("one-pass").times_pass(i, 4)
                   for i in range(4))


def test_pass_cost_derives_from_nearest_rank_medians():  # pass_cost.rs:80-105
    from beatlm_b200.pass_cost import Frame, derive, nearest_rank
    assert nearest_rank([1, 2, 3, 4], 50) == 2 and nearest_rank([5], 90) == 5
    assert nearest_rank([], 50) is None
    f = lambda span, passes=None, enc=1.0: Frame(span, span if passes is None else passes, enc, 1)
    frames = {("per-pass", 1): [f(10), f(11), f(12)], ("per-pass", 9): [f(50, 40, 9.0)],
              ("ends", 9): [f(42)], ("one-pass", 1): [f(9)], ("one-pass", 9): [f(25)]}
    d = derive(frames)
    assert d["span_us"]["[per-pass,1]"] == 11
    a = d["derived"]["[per-pass,9]"]
    assert a["per_pass_us"] == (50 - 11) / 8 and a["over_one_pass_us"] == (50 - 25) / 8
    assert a["over_ends_us"] == 1.0 and a["between_us"] == 10 and a["encode_per_pass_us"] == 1.0
    assert d["derived"]["[one-pass,9]"]["per_dispatch_us"] == 2.0
    assert "per_pass_us" not in derive(frames, trivial=False)["derived"]["[per-pass,9]"]
