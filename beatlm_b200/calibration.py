"""Calibration: what each kernel of a program takes run whole on this GPU,
the parts that keep each launch within a bound, and what each part takes,
measured before the frame loop into the loop's cost model. The reference's
two paced passes (``crates/beatlm-bench/src/calibrate.rs:1-188``, with the
counting rule and the per-kernel median of
``crates/beatlm-host/src/calibration.rs``), timed by the cudaEvent slice
timer instead of wgpu timestamp queries:

1. whole kernels: ``CALIBRATION_FRAMES`` timed frames after one untimed
   frame; a kernel's duration is the median of its measurements in the
   second half of the timed frames (``counted``);
2. the program split by ``Program::parts_within`` for those durations and a
   bound, run the same way; every part's counted measurements go into a
   ``CostModel`` as calibration's (``record_calibration``).

Both passes are paced at the loop's frame period (the host sleeps to each
tick), so kernels are measured with the GPU as idle between frames as the
loop will leave it."""
from __future__ import annotations

import dataclasses
import time

from . import runtime as R
from .cost import CostModel

WINDOW = 32                       # presets.rs:19
CALIBRATION_FRAMES = 2 * WINDOW   # presets.rs:71


def counted(frame: int, frames: int = CALIBRATION_FRAMES) -> bool:
    """Whether a pass keeps timed frame ``frame`` (from 1): the second half
    (calibration.rs:29)."""
    return frame > frames // 2


class KernelSamples:
    """What pass 1 keeps of each whole kernel and the median it decides on
    (calibration.rs:37-90)."""

    def __init__(self, kernels: int, frames: int = CALIBRATION_FRAMES):
        self.samples = [[] for _ in range(kernels)]
        self.frames = frames

    def record(self, frame: int, slice_: int, duration_us: int):
        if counted(frame, self.frames) and 0 <= slice_ < len(self.samples):
            self.samples[slice_].append(int(duration_us))

    def durations(self) -> list[int]:
        out = []
        for k, s in enumerate(self.samples):
            if not s:
                raise RuntimeError("calibration measured kernel %d no time" % k)
            out.append(sorted(s)[len(s) // 2])  # stats.rs:145 median
        return out


@dataclasses.dataclass
class Calibration:
    durations: list   # whole-kernel medians, microseconds
    parts: list       # part count per kernel
    specs: list       # the split program's specs
    cost: CostModel   # the split program's parts, as calibration's measurements


def _measure(program: R.Kernels, stream, frames: int, period_us: int, record):
    """One untimed frame, then ``frames`` timed frames of the whole program,
    one every ``period_us`` (0 = back to back), each waited for; ``record``
    gets (timed frame from 1, kernel, whole microseconds) per pass
    (calibrate.rs:189-246)."""
    from .cost import micros_nearest
    timer = R.SliceTimer(max(1, len(program)))
    start = time.perf_counter()
    try:
        for tick in range(frames + 1):
            if period_us > 0:
                wait = start + tick * period_us * 1e-6 - time.perf_counter()
                if wait > 0:
                    time.sleep(wait)
            handle = timer.begin_frame(tick) if tick > 0 else -1
            program.encode_all(stream, timer if handle >= 0 else None, handle)
            if handle >= 0:
                timer.submitted(handle)
            stream.synchronize()
            for timing in timer.collect_ready():
                for kernel, micros in timing.compute:
                    record(timing.frame, kernel, micros_nearest(micros))
    finally:
        timer.close()


def calibrate(specs: list, bound_us: int, *, prior_us: int = 0, estimator=None,
              frames: int = CALIBRATION_FRAMES, period_us: int = 16667, stream=None) -> Calibration:
    """Both passes over the unsplit program ``specs`` (``runtime.Spec``);
    raises for a split program, a bound of zero or a kernel or part that was
    never measured (calibrate.rs:105-186)."""
    import torch
    if any(s.parts != 1 for s in specs):
        raise ValueError("calibrate: the program is already split")
    if bound_us <= 0:
        raise ValueError("calibrate: no dispatch fits a bound of zero")
    stream = stream or torch.cuda.current_stream()

    whole = R.Kernels(specs)
    first = KernelSamples(len(whole), frames)
    try:
        _measure(whole, stream, frames, period_us, first.record)
    finally:
        whole.close()
    durations = first.durations()
    parts = R.program_parts_within(specs, durations, bound_us)
    split_specs = R.split(specs, parts)

    cost = CostModel(prior_us, estimator)
    program = R.Kernels(split_specs)
    try:
        def keep(frame, kernel, us):
            if counted(frame, frames):
                cost.record_calibration(kernel, us)
        _measure(program, stream, frames, period_us, keep)
        n = len(program)
    finally:
        program.close()
    for part in range(n):
        if cost.samples(part) == 0:
            raise RuntimeError("calibration measured part %d of the split program no time" % part)
    return Calibration(durations, parts, split_specs, cost)
