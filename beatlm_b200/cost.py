"""Measured slice costs for the frame scheduler: the host mirror of the
reference's ``CostModel`` (``crates/beatlm-core/src/cost.rs:726-966``) over
``bl_cost_*``, fed from the cudaEvent slice timer (``runtime.SliceTimer``)
instead of wgpu timestamp queries.

Names, argument meanings and errors follow the reference: an estimator is
one of ``MeanPlusSigmas``, ``WindowedQuantile``, ``CappedDeviation`` and
``FrameScaled``; a rejected one raises ``CostError`` naming the parameter
(``cost.rs:298-325``); a slice is a kernel index of the program; every
duration is whole microseconds."""
from __future__ import annotations

import ctypes
import dataclasses

from . import _native as N

MAX_WINDOW = 4096      # cost.rs:294
WARM_SAMPLES = 5       # cost.rs:671
U64_MAX = (1 << 64) - 1

_KIND_MPS, _KIND_WQ, _KIND_CD, _KIND_FS = 0, 1, 2, 3
_ERRORS = {1: "InvalidAlpha", 2: "InvalidSigmas", 3: "InvalidWindow", 4: "InvalidQuantile",
           5: "InvalidFrameWindow", 6: "InvalidCap", 7: "UnknownEstimator"}


@dataclasses.dataclass(frozen=True)
class MeanPlusSigmas:
    alpha: float
    sigmas: float


@dataclasses.dataclass(frozen=True)
class WindowedQuantile:
    window: int = 32
    quantile: float = 0.9


@dataclasses.dataclass(frozen=True)
class CappedDeviation:
    alpha: float
    sigmas: float
    cap: float


@dataclasses.dataclass(frozen=True)
class FrameScaled:
    window: int
    frame_window: int
    frame_quantile: float


def default_estimator() -> WindowedQuantile:
    """``Estimator::default`` (cost.rs:416): the 0.9 quantile of the last 32."""
    e = N.Estimator()
    N.lib().bl_estimator_default(ctypes.byref(e))
    return _from_c(e)


@dataclasses.dataclass(frozen=True)
class WarmingUp:
    recorded: int
    needed: int


@dataclasses.dataclass(frozen=True)
class Measured:
    scale: float


FRAME_SCALE_NONE = None  # FrameScale::None


class CostError(ValueError):
    """A rejected estimator; ``kind`` is the reference's variant name."""

    def __init__(self, kind: str, message: str):
        super().__init__(message)
        self.kind = kind


def _window(w: int) -> int:
    # out-of-range windows reach the C validation as 0 (rejected) rather than
    # wrapping around the uint32 field
    return int(w) if 0 <= int(w) < (1 << 32) else 0


def _to_c(e) -> N.Estimator:
    c = N.Estimator()
    if isinstance(e, MeanPlusSigmas):
        c.kind, c.alpha, c.sigmas = _KIND_MPS, e.alpha, e.sigmas
    elif isinstance(e, WindowedQuantile):
        c.kind, c.window, c.quantile = _KIND_WQ, _window(e.window), e.quantile
    elif isinstance(e, CappedDeviation):
        c.kind, c.alpha, c.sigmas, c.cap = _KIND_CD, e.alpha, e.sigmas, e.cap
    elif isinstance(e, FrameScaled):
        c.kind, c.window, c.frame_window, c.quantile = (_KIND_FS, _window(e.window),
                                                        _window(e.frame_window), e.frame_quantile)
    else:
        c.kind = -1
    return c


def _from_c(c: N.Estimator):
    if c.kind == _KIND_MPS:
        return MeanPlusSigmas(c.alpha, c.sigmas)
    if c.kind == _KIND_WQ:
        return WindowedQuantile(c.window, c.quantile)
    if c.kind == _KIND_CD:
        return CappedDeviation(c.alpha, c.sigmas, c.cap)
    return FrameScaled(c.window, c.frame_window, c.quantile)


def micros_nearest(micros: float) -> int:
    """A timer duration in whole microseconds, rounded to nearest (timer.rs:781)."""
    return N.lib().bl_micros_nearest(float(micros))


class CostModel:
    """``CostModel`` (cost.rs:726): per-slice statistics of measured
    durations, read as the estimate the scheduler plans with."""

    def __init__(self, prior: int, estimator=None, *, _handle=None):
        self._lib = N.lib()  # kept for the destructor at interpreter exit
        if _handle is not None:
            self._h = _handle
            return
        est = default_estimator() if estimator is None else estimator
        h, err = ctypes.c_void_p(), ctypes.c_int32()
        rc = N.lib().bl_cost_create(int(prior), ctypes.byref(_to_c(est)), ctypes.byref(h),
                                    ctypes.byref(err))
        if rc != 0:
            raise CostError(_ERRORS.get(err.value, "Invalid"), N.last_error())
        self._h = h

    def clone(self) -> "CostModel":
        h = ctypes.c_void_p()
        N.check(N.lib().bl_cost_clone(self._h, ctypes.byref(h)))
        return CostModel(0, _handle=h)

    @property
    def estimator(self):
        c = N.Estimator()
        N.check(N.lib().bl_cost_estimator(self._h, ctypes.byref(c)))
        return _from_c(c)

    def record(self, slice_: int, measured: int):
        N.lib().bl_cost_record(self._h, slice_, int(measured))

    def record_calibration(self, slice_: int, measured: int):
        N.lib().bl_cost_record_calibration(self._h, slice_, int(measured))

    def frame_estimate(self, slice_: int) -> int | None:
        out = ctypes.c_uint64()
        return out.value if N.lib().bl_cost_frame_estimate(self._h, slice_, ctypes.byref(out)) \
            else None

    def record_frame(self, predicted: int, measured: int):
        N.lib().bl_cost_record_frame(self._h, int(predicted), int(measured))

    def frame_scale(self):
        scale, rec, need = ctypes.c_double(), ctypes.c_uint64(), ctypes.c_uint64()
        k = N.lib().bl_cost_frame_scale(self._h, ctypes.byref(scale), ctypes.byref(rec),
                                        ctypes.byref(need))
        if k == 1:
            return WarmingUp(rec.value, need.value)
        if k == 2:
            return Measured(scale.value)
        return FRAME_SCALE_NONE

    def frames_recorded(self) -> int:
        return N.lib().bl_cost_frames_recorded(self._h)

    def planning_estimate(self, slice_: int) -> int:
        return N.lib().bl_cost_planning_estimate(self._h, slice_)

    def estimate(self, slice_: int) -> int:
        return N.lib().bl_cost_estimate(self._h, slice_)

    def samples(self, slice_: int) -> int:
        return N.lib().bl_cost_samples(self._h, slice_)

    # ------------------------------------------------- fed by the slice timer

    def plan_frame(self, slices) -> dict:
        """What a frame's ratio takes each slice at, read when the frame is
        planned (``frame_estimate``; None = left out of the ratio)."""
        return {s: self.frame_estimate(s) for s in slices}

    def record_timing(self, timing, *, calibration: bool = False, planned: dict | None = None):
        """Folds one collected frame (``runtime.FrameTiming``): every pass's
        duration under its kernel index, as the loop's measurements or, with
        ``calibration``, calibration's (calibrate.rs:165-174). With
        ``planned`` (``plan_frame`` of this frame, taken when it was planned)
        the frame's ratio is recorded too: the planned estimates of the
        slices that have one against those slices' measured durations, as a
        host does (cost.rs:863-870)."""
        passes = (N.SliceTime * max(1, len(timing.compute)))()
        for i, (kernel, micros) in enumerate(timing.compute):
            passes[i].frame, passes[i].slice, passes[i].kernel = timing.frame, i, kernel
            passes[i].micros = micros
        N.lib().bl_cost_record_passes(self._h, passes, len(timing.compute),
                                      1 if calibration else 0)
        if planned is not None:
            predicted = measured = 0
            for kernel, micros in timing.compute:
                est = planned.get(kernel)
                if est is not None:
                    predicted = min(U64_MAX, predicted + est)
                    measured = min(U64_MAX, measured + micros_nearest(micros))
            self.record_frame(predicted, measured)

    def close(self):
        if getattr(self, "_h", None):
            self._lib.bl_cost_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
