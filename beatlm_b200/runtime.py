"""Programs of prebuilt launches, CUDA-graph replay and the slice timer.

Host mirror of the reference's ``Kernels`` (``crates/beatlm/src/codegen/
kernels.rs:63-249``: build once, encode per frame) and ``SliceTimer``
(``crates/beatlm/src/gpu/timer.rs:185-470``), over ``bl_kernels_*`` and
``bl_timer_*``.
"""
from __future__ import annotations

import ctypes
import dataclasses

from . import _native as N
from .ops import _stream_ptr

OP_ATTENTION, OP_GEMM, OP_LAYERNORM, OP_PATCHIFY, OP_ALLGATHER = 1, 2, 3, 4, 5
_OP_OF = {N.AttentionArgs: OP_ATTENTION, N.GemmArgs: OP_GEMM,
          N.LayerNormArgs: OP_LAYERNORM, N.PatchifyArgs: OP_PATCHIFY,
          N.AllGatherArgs: OP_ALLGATHER}


def hold(stream, microseconds: int):
    """Holds `stream` for `microseconds` of device time (bl_stream_hold), so
    that what is enqueued behind it starts back to back on the GPU."""
    N.check(N.lib().bl_stream_hold(_stream_ptr(stream), microseconds))


@dataclasses.dataclass
class Spec:
    """One kernel of a program: its packed arguments, a label, its parts."""
    args: ctypes.Structure
    label: str
    parts: int = 1

    @property
    def op(self) -> int:
        return _OP_OF[type(self.args)]


def split_edges(extent: int, grain: int, count: int) -> list[int]:
    """Program::split's part edges (kernel.rs:2006-2029), from the library."""
    edges = (ctypes.c_uint32 * (max(count, 1) + 1))()
    c = N.lib().bl_split_edges(extent, grain, count, edges)
    return list(edges[:c + 1])


def parts_within(duration_us: int, bound_us: int, max_parts: int) -> int:
    """KernelSpec::parts_within (kernel.rs:2048-2056); 0 for a zero bound."""
    return N.lib().bl_parts_within(duration_us, bound_us, max_parts)


def _spec_array(specs: list[Spec]):
    arr = (N.KernelSpec * max(1, len(specs)))()
    labels = [s.label.encode() for s in specs]
    for i, s in enumerate(specs):
        arr[i] = N.KernelSpec(op=s.op, args=ctypes.cast(ctypes.pointer(s.args), ctypes.c_void_p),
                              label=labels[i], parts=s.parts)
    return arr, labels


def max_parts(spec: Spec) -> int:
    """KernelSpec::max_parts (kernel.rs:1975), from the library."""
    arr, _ = _spec_array([spec])
    return N.lib().bl_kernel_spec_max_parts(arr)


def program_parts_within(specs: list[Spec], durations_us: list[int], bound_us: int) -> list[int]:
    """Program::parts_within (kernel.rs:2350-2366): the part count of every
    kernel for its measured duration; raises for a bound of zero or a
    duration list of the wrong length."""
    arr, _ = _spec_array(specs)
    d = (ctypes.c_uint64 * max(1, len(durations_us)))(*durations_us)
    out = (ctypes.c_uint32 * max(1, len(specs)))()
    N.check(N.lib().bl_program_parts_within(arr, len(specs), d, len(durations_us), bound_us, out))
    return list(out[:len(specs)])


def split(specs: list[Spec], parts: list[int]) -> list[Spec]:
    """Program::split (kernel.rs:2368-2407) as specs: kernel i in parts[i]
    parts (the library clamps the count to 1..=max_parts)."""
    if len(parts) != len(specs):
        raise ValueError("split: %d part counts for %d kernels" % (len(parts), len(specs)))
    if any(s.parts != 1 for s in specs):
        raise ValueError("split: the program is already split")
    return [dataclasses.replace(s, parts=max(1, int(p))) for s, p in zip(specs, parts)]


def _substitution(pair) -> "N.Substitution":
    """(original, stand_in) tensors of one size, or (from_ptr, to_ptr, bytes)."""
    if len(pair) == 3:
        return N.Substitution(pair[0], pair[1], pair[2])
    a, b = pair
    nbytes = a.numel() * a.element_size()
    if b.numel() * b.element_size() != nbytes:
        raise ValueError("a stand-in of %d bytes for a tensor of %d bytes"
                         % (b.numel() * b.element_size(), nbytes))
    return N.Substitution(a.data_ptr(), b.data_ptr(), nbytes)


class Kernels:
    """Prebuilt launches of a program; ``len`` counts parts.

    ``sets``: binding sets (Kernels::new, kernels.rs:63-184), each a list of
    substitutions ``(original, stand_in)`` (tensors of one byte size) or
    ``(from_ptr, to_ptr, bytes)``; none means one set binding every spec as
    given. ``encode(..., set=j)`` runs kernel k over set j's tensors."""

    def __init__(self, specs: list[Spec], sets: list | None = None):
        arr, self._labels = _spec_array(specs)
        sets = sets or []
        self._subs = [(N.Substitution * max(1, len(s)))(*[_substitution(p) for p in s])
                      for s in sets]
        bs = (N.BindingSet * max(1, len(sets)))()
        for j, s in enumerate(sets):
            bs[j] = N.BindingSet(self._subs[j], len(s))
        h = ctypes.c_void_p()
        N.check(N.lib().bl_kernels_create(arr, len(specs), bs if sets else None, len(sets),
                                          ctypes.byref(h)))
        self._h = h
        self._graphs = []

    def __len__(self) -> int:
        return N.lib().bl_kernels_len(self._h)

    @property
    def sets(self) -> int:
        return N.lib().bl_kernels_sets(self._h)

    @property
    def launches(self) -> int:
        """Distinct launches built (parts x sets, less those sets share)."""
        return N.lib().bl_kernels_launches(self._h)

    def label(self, k: int) -> str:
        s = N.lib().bl_kernels_label(self._h, k)
        return s.decode() if s is not None else None

    def encode(self, k: int, stream=None, timer: "SliceTimer | None" = None, frame: int = -1,
               set: int = 0):
        N.check(N.lib().bl_kernels_encode(self._h, k, set, _stream_ptr(stream),
                                          timer._h if timer else None, frame))

    def encode_all(self, stream=None, timer: "SliceTimer | None" = None, frame: int = -1,
                   begin: int = 0, end: int | None = None, set: int = 0):
        end = len(self) if end is None else end
        N.check(N.lib().bl_kernels_encode_range(self._h, begin, end, set, _stream_ptr(stream),
                                                timer._h if timer else None, frame))

    def capture(self, stream, set: int = 0) -> "Graph":
        g = ctypes.c_void_p()
        N.check(N.lib().bl_kernels_capture(self._h, set, _stream_ptr(stream), ctypes.byref(g)))
        graph = Graph(g)
        self._graphs.append(graph)
        return graph

    def close(self):
        for g in self._graphs:
            g.close()
        self._graphs = []
        if self._h:
            N.lib().bl_kernels_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Graph:
    def __init__(self, h):
        self._h = h

    def launch(self, stream=None):
        N.check(N.lib().bl_graph_launch(self._h, _stream_ptr(stream)))

    def close(self):
        if self._h:
            N.lib().bl_graph_destroy(self._h)
            self._h = None


@dataclasses.dataclass
class FrameTiming:
    """What one frame's passes took (timer.rs:115): (kernel, micros) per
    pass in encode order, and each pass's begin relative to the first."""
    frame: int
    compute: list
    begin_us: list


class SliceTimer:
    RING_DEPTH = 3

    def __init__(self, max_slices: int):
        h = ctypes.c_void_p()
        N.check(N.lib().bl_timer_create(max_slices, ctypes.byref(h)))
        self._h = h
        self.max_slices = max_slices

    def begin_frame(self, frame: int) -> int:
        """A handle for `frame`, or -1 when its ring slot is in flight."""
        h = ctypes.c_int32()
        N.check(N.lib().bl_timer_begin_frame(self._h, frame, ctypes.byref(h)))
        return h.value

    def submitted(self, handle: int):
        N.check(N.lib().bl_timer_submitted(self._h, handle))

    def submitted_held(self, handle: int):
        N.check(N.lib().bl_timer_submitted_held(self._h, handle))

    def settle(self, handle: int, accept: bool):
        N.check(N.lib().bl_timer_settle(self._h, handle, 1 if accept else 0))

    def drop(self, handle: int):
        N.check(N.lib().bl_timer_drop(self._h, handle))

    def invalidate_submitted(self) -> int:
        return N.lib().bl_timer_invalidate_submitted(self._h)

    def in_flight(self) -> int:
        return N.lib().bl_timer_in_flight(self._h)

    def collect_ready(self) -> list[FrameTiming]:
        cap = self.max_slices * self.RING_DEPTH
        buf = (N.SliceTime * cap)()
        n, frames = ctypes.c_size_t(), ctypes.c_size_t()
        N.check(N.lib().bl_timer_collect_ready(self._h, buf, cap, ctypes.byref(n),
                                               ctypes.byref(frames)))
        out: list[FrameTiming] = []
        for i in range(n.value):
            e = buf[i]
            if not out or out[-1].frame != e.frame or e.slice == 0:
                out.append(FrameTiming(e.frame, [], []))
            out[-1].compute.append((e.kernel, e.micros))
            out[-1].begin_us.append(e.begin_us)
        return out

    def stats(self) -> dict:
        s = N.TimerStats()
        N.check(N.lib().bl_timer_get_stats(self._h, ctypes.byref(s)))
        return {"frames_skipped": s.frames_skipped, "frames_collected": s.frames_collected,
                "frames_failed": s.frames_failed}

    def close(self):
        if self._h:
            N.lib().bl_timer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class InputPipeline:
    """Host-to-device copies of one input a step ahead, over two device
    buffers (input slots, as the reference's Net keeps jobs in flight,
    crates/beatlm-host/src/slots.rs:1-60). ``acquire(stream)`` returns this
    step's device buffer, whose copy was issued a step earlier beside the
    previous step's work (``stream`` waits for it), and issues the copy of
    the next step's input into the other buffer on a copy stream of its own,
    once the step that last read that buffer has ended. ``release(stream)``
    marks the end of this step's reads (on ``stream``, after its work).
    ``hosts[i]`` (pinned) is copied into ``devices[i]``; ``fill(i)``, when
    given, writes the next input into ``hosts[i]`` first, after the previous
    copy from it has completed."""

    def __init__(self, hosts: list, devices: list):
        import torch
        if len(hosts) != 2 or len(devices) != 2:
            raise ValueError("an input pipeline has two host and two device buffers")
        self.hosts, self.devices = hosts, devices
        self.copy = torch.cuda.Stream()
        self._in = [torch.cuda.Event() for _ in range(2)]    # the buffer's copy landed
        self._done = [torch.cuda.Event() for _ in range(2)]  # its last reader ended
        self._used = [False, False]
        self._primed = False
        self.k = 0

    def _issue(self, i, fill):
        import torch
        if fill is not None:
            self._in[i].synchronize()
            fill(i)
        if self._used[i]:
            self.copy.wait_event(self._done[i])
        with torch.cuda.stream(self.copy):
            self.devices[i].copy_(self.hosts[i], non_blocking=True)
        self._in[i].record(self.copy)

    def slot(self) -> int:
        """This step's buffer index."""
        return self.k % 2

    def acquire(self, stream, fill=None):
        i = self.slot()
        if not self._primed:
            self._issue(i, fill)
            self._primed = True
        self._issue(1 - i, fill)  # the next step's input, beside this step
        stream.wait_event(self._in[i])
        return self.devices[i]

    def release(self, stream):
        i = self.slot()
        self._done[i].record(stream)
        self._used[i] = True
        self.k += 1
