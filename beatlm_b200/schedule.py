"""The frame-slice scheduler: the host mirror of the reference's
``Scheduler`` (``crates/beatlm-core/src/schedule.rs:160-790``) with its
``SyncPolicy`` / ``MissPolicy`` (``sync.rs``), ``Budget`` (``budget.rs``) and
beat grids (``time.rs``), over ``bl_scheduler_*``. It plans with a
``cost.CostModel``'s planning estimates, which this package feeds from
cudaEvent timings. Times are whole microseconds.

    s = Scheduler(FixedLatency(2), "hold_previous", expected=5000)
    job = s.submit(FrameInfo(i, start, period), slices, cost)
    plan = s.plan_frame(FrameInfo(i, start, period), budget, cost)
"""
from __future__ import annotations

import ctypes
import dataclasses

from . import _native as N

_MISS = {"hold_previous": 0, "drop": 1}
_MISS_NAME = {v: k for k, v in _MISS.items()}


class ScheduleError(ValueError):
    """ScheduleError / TimeError: ``kind`` is "EmptyJob", "NotOnBeat" or
    "ZeroBeat"."""

    def __init__(self, kind: str, message: str):
        super().__init__(message)
        self.kind = kind


def _raise(rc: int):
    if rc != 0:
        msg = N.last_error()
        kind = next((k for k in ("EmptyJob", "NotOnBeat", "ZeroBeat") if k in msg), "Invalid")
        raise ScheduleError(kind, msg)


@dataclasses.dataclass(frozen=True)
class BeatGrid:
    origin: int
    beat: int

    def __post_init__(self):
        if self.beat == 0:
            raise ScheduleError("ZeroBeat", "beat length must be greater than zero")

    def next_beat_at_or_after(self, t: int) -> int:
        return beat_map_next([(0, self)], t)


@dataclasses.dataclass(frozen=True)
class FixedLatency:
    frames: int


@dataclasses.dataclass(frozen=True)
class SameFrame:
    pass


@dataclasses.dataclass(frozen=True)
class OnBeat:
    margin: int
    grid: BeatGrid


def source_delay(policy) -> int | None:
    """SyncPolicy::source_delay (sync.rs): how many frames the host delays
    its source; None for OnBeat."""
    return policy.frames if isinstance(policy, FixedLatency) else \
        0 if isinstance(policy, SameFrame) else None


def max_in_flight(policy) -> int | None:
    """SyncPolicy::max_in_flight (sync.rs)."""
    if isinstance(policy, FixedLatency):
        return min(policy.frames + 1, (1 << 32) - 1)
    return 1 if isinstance(policy, SameFrame) else None


def budget_for_frame(period: int, render: int, margin: int) -> int:
    """Budget::for_frame (budget.rs): period - render - margin, at least 0."""
    return N.lib().bl_budget_for_frame(period, render, margin)


def beat_map_next(grids, t: int) -> int:
    """BeatMap::next_beat_at_or_after over [(from, BeatGrid), ...], the first
    in effect from 0 and each later one from its ``from``."""
    flat = []
    for frm, g in grids:
        flat += [frm, g.origin, g.beat]
    arr = (ctypes.c_uint64 * len(flat))(*flat)
    out = ctypes.c_uint64()
    _raise(N.lib().bl_beat_map_next(arr, len(grids), t, ctypes.byref(out)))
    return out.value


@dataclasses.dataclass(frozen=True)
class FrameInfo:
    index: int
    start: int
    period: int

    def _c(self):
        return N.FrameInfo(index=self.index, start_us=self.start, period_us=self.period)


@dataclasses.dataclass(frozen=True)
class Due:
    kind: str   # "frame" or "beat"
    at: int     # the frame index or the beat's instant


@dataclasses.dataclass(frozen=True)
class SliceRun:
    job: int
    slice: int
    position: int


@dataclasses.dataclass(frozen=True)
class Delivery:
    job: int
    input: int


@dataclasses.dataclass(frozen=True)
class Missed:
    job: int
    input: int
    due: Due
    policy: str


@dataclasses.dataclass
class FramePlan:
    runs: list
    delivered: list
    missed: list
    spent_estimate: int
    budget: int


def _due(d) -> Due:
    return Due("beat" if d.kind == 1 else "frame", d.at)


class Scheduler:
    """``Scheduler`` (schedule.rs:512)."""

    def __init__(self, policy, miss: str = "hold_previous", expected: int = 0):
        p = N.SyncPolicy()
        if isinstance(policy, FixedLatency):
            p.kind, p.frames = 0, policy.frames
        elif isinstance(policy, SameFrame):
            p.kind = 1
        elif isinstance(policy, OnBeat):
            p.kind, p.margin_us = 2, policy.margin
            p.grid_origin_us, p.grid_beat_us = policy.grid.origin, policy.grid.beat
        else:
            raise TypeError("policy: FixedLatency, SameFrame or OnBeat")
        self._lib = N.lib()  # kept for the destructor at interpreter exit
        h = ctypes.c_void_p()
        _raise(self._lib.bl_scheduler_create(ctypes.byref(p), _MISS[miss], expected,
                                             ctypes.byref(h)))
        self._h = h

    def set_expected_budget(self, expected: int):
        self._lib.bl_scheduler_set_expected_budget(self._h, expected)

    @property
    def expected_budget(self) -> int:
        return self._lib.bl_scheduler_expected_budget(self._h)

    def replace_beat_grid(self, from_: int, grid: BeatGrid):
        _raise(self._lib.bl_scheduler_replace_beat_grid(self._h, from_, grid.origin, grid.beat))

    def submit(self, input_: FrameInfo, slices, cost) -> int:
        arr = (ctypes.c_uint32 * max(1, len(slices)))(*slices)
        job = ctypes.c_uint64()
        _raise(self._lib.bl_scheduler_submit(self._h, ctypes.byref(input_._c()), arr, len(slices),
                                             cost._h, ctypes.byref(job)))
        return job.value

    def plan_frame(self, frame: FrameInfo, budget: int, cost) -> FramePlan:
        info = N.FramePlanInfo()
        _raise(self._lib.bl_scheduler_plan_frame(self._h, ctypes.byref(frame._c()), budget,
                                                 cost._h, ctypes.byref(info)))
        runs = (N.SliceRun * max(1, info.runs))()
        dels = (N.Delivery * max(1, info.delivered))()
        miss = (N.Missed * max(1, info.missed))()
        self._lib.bl_scheduler_plan_runs(self._h, runs, info.runs)
        self._lib.bl_scheduler_plan_delivered(self._h, dels, info.delivered)
        self._lib.bl_scheduler_plan_missed(self._h, miss, info.missed)
        return FramePlan(
            [SliceRun(r.job, r.slice, r.position) for r in runs[:info.runs]],
            [Delivery(d.job, d.input) for d in dels[:info.delivered]],
            [Missed(m.job, m.input, _due(m.due), _MISS_NAME[m.policy])
             for m in miss[:info.missed]],
            info.spent_estimate_us, info.budget_us)

    def pending(self) -> int:
        return self._lib.bl_scheduler_pending(self._h)

    def due(self, job: int) -> Due | None:
        d = N.Due()
        return _due(d) if self._lib.bl_scheduler_due(self._h, job, ctypes.byref(d)) else None

    def close(self):
        if getattr(self, "_h", None):
            self._lib.bl_scheduler_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class FrameLoop:
    """The host's side of a frame over a program (the reference host's
    `tick`, crates/beatlm/src/lib.rs:69-120): submit this frame's input as a
    job of every kernel of the program, plan the frame, encode the planned
    slices on ``stream`` with the slice timer, and fold every frame whose
    events have completed into the cost model (with its planned estimates,
    so a frame-scaled model records the frame's ratio). Nothing blocks: the
    timings of a frame arrive in a later tick.

    ``kernels`` is one program (``runtime.Kernels``) with one binding set per
    input/output slot (``model.Encoder.program``): job j runs with set
    j % sets, as the reference's Net binds its slots
    (crates/beatlm-host/src/slots.rs:1-60), so up to ``sets`` jobs in flight
    keep their own input and output."""

    def __init__(self, kernels, scheduler: Scheduler, cost, timer):
        self.kernels = kernels
        self.scheduler, self.cost, self.timer = scheduler, cost, timer
        self._planned = {}

    def slot_of(self, job: int) -> int:
        return job % self.kernels.sets

    def tick(self, frame: FrameInfo, budget: int, submit: bool, stream=None,
             write_input=None) -> FramePlan:
        """``write_input(slot)``, when given, fills the new job's input slot
        before the frame's slices are encoded."""
        if submit:
            job = self.scheduler.submit(frame, list(range(len(self.kernels))), self.cost)
            if write_input is not None:
                write_input(self.slot_of(job))
        plan = self.scheduler.plan_frame(frame, budget, self.cost)
        handle = self.timer.begin_frame(frame.index) if plan.runs else -1
        if handle >= 0:
            self._planned[frame.index] = self.cost.plan_frame({r.slice for r in plan.runs})
        for r in plan.runs:
            self.kernels.encode(r.slice, stream, self.timer if handle >= 0 else None, handle,
                                set=self.slot_of(r.job))
        if handle >= 0:
            self.timer.submitted(handle)
        self.collect()
        return plan

    def collect(self) -> int:
        """Folds every completed frame's timings; returns how many."""
        done = self.timer.collect_ready()
        for t in done:
            self.cost.record_timing(t, planned=self._planned.pop(t.frame, None))
        return len(done)
