"""The static memory plan and its single device allocation, through the C ABI.

Mirrors the reference's ``beatlm_core::memory`` (``crates/beatlm-core/src/
memory.rs``) and ``beatlm::gpu::arenas`` (``crates/beatlm/src/gpu/arenas.rs``):
the same names, argument meanings and errors. ``MemoryPlan`` is host-only
work (no GPU); ``Arenas`` makes ONE ``cudaMalloc`` for every arena of a plan
and hands out device addresses and torch views of the placements in it.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _native as N

F32, F16, BF16 = "f32", "f16", "bf16"
_BYTES = {F32: 4, F16: 2, BF16: 2}


@dataclass(frozen=True)
class TensorDesc:
    """A tensor the planner places: its id, element type, element count and
    the operations it is in use from and to, both inclusive (memory.rs:158)."""
    id: int
    dtype: str
    elements: int
    first_use: int
    last_use: int


@dataclass(frozen=True)
class DeviceProfile:
    """The limits the plan is made against (device.rs:97-125)."""
    max_binding_bytes: int
    max_buffer_bytes: int
    offset_alignment: int

    @staticmethod
    def webgpu_baseline() -> "DeviceProfile":
        p = N.DeviceProfile()
        N.check(N.lib().bl_device_profile_webgpu_baseline(ctypes.byref(p)))
        return DeviceProfile(p.max_binding_bytes, p.max_buffer_bytes, p.offset_alignment)

    @staticmethod
    def cuda(device: int | None = None) -> "DeviceProfile":
        """The profile of CUDA device `device` (default: the current one)."""
        if device is None:
            import torch
            device = torch.cuda.current_device()
        p = N.DeviceProfile()
        N.check(N.lib().bl_device_profile_cuda(device, ctypes.byref(p)))
        return DeviceProfile(p.max_binding_bytes, p.max_buffer_bytes, p.offset_alignment)

    def max_arena_size(self) -> int:
        return min(self.max_binding_bytes, self.max_buffer_bytes)

    def _c(self):
        return N.DeviceProfile(self.max_binding_bytes, self.max_buffer_bytes,
                               self.offset_alignment)


@dataclass(frozen=True)
class Placement:
    """Where a tensor lives: arena, byte offset, reserved bytes (memory.rs:200)."""
    arena: int
    offset: int
    size: int

    def end(self) -> int:
        return self.offset + self.size

    def _c(self):
        return N.Placement(self.arena, 0, self.offset, self.size)


class PlanError(ValueError):
    """Why a set of tensors could not be planned (memory.rs:220): `kind` is
    one of KINDS; `id`, and `a`/`b` (first/last use, or size/limit) as the
    kind has them."""

    KINDS = {1: "DuplicateTensor", 2: "InvalidLifetime", 3: "EmptyTensor", 4: "SizeOverflow",
             5: "TensorTooLarge", 6: "InvalidProfile", 7: "TooManyTensors"}

    def __init__(self, kind: int, id: int, a: int, b: int, message: str):
        super().__init__(message)
        self.kind, self.id, self.a, self.b = self.KINDS.get(kind, "Invalid"), id, a, b

    def __eq__(self, other):
        return (isinstance(other, PlanError) and
                (self.kind, self.id, self.a, self.b) == (other.kind, other.id, other.a, other.b))

    __hash__ = None


class MemoryPlan:
    """MemoryPlan::new (memory.rs:285). Raises PlanError on malformed input."""

    def __init__(self, tensors, profile: DeviceProfile):
        arr = (N.TensorDesc * max(1, len(tensors)))()
        for i, t in enumerate(tensors):
            if t.elements < 0 or t.elements >= 1 << 64:
                raise PlanError(4, t.id, 0, 0, "the size of tensor %d overflows" % t.id)
            arr[i] = N.TensorDesc(t.id, _BYTES[t.dtype], t.elements, t.first_use, t.last_use)
        err = N.PlanErrorInfo()
        handle = ctypes.c_void_p()
        rc = N.lib().bl_plan_create(arr, len(tensors), ctypes.byref(profile._c()),
                                    ctypes.byref(handle), ctypes.byref(err))
        if rc != N.BL_OK:
            if err.kind:
                raise PlanError(err.kind, err.id, err.a, err.b, N.last_error())
            raise N.BackendError(rc, N.last_error())
        self._h, self._lib = handle, N.lib()  # the library outlives module teardown
        self._ids = [t.id for t in tensors]

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.bl_plan_destroy(h)
            self._h = None

    @property
    def handle(self):
        return self._h

    def arenas(self) -> list[int]:
        n = N.lib().bl_plan_arenas(self._h, None, 0)
        out = (ctypes.c_uint64 * max(1, n))()
        N.lib().bl_plan_arenas(self._h, out, n)
        return [int(out[i]) for i in range(n)]

    def placement(self, id: int) -> Placement | None:
        p = N.Placement()
        if N.lib().bl_plan_placement(self._h, id, ctypes.byref(p)) != N.BL_OK:
            return None
        return Placement(p.arena, p.offset, p.size)

    def placements(self):
        """Every tensor's placement, in id order."""
        return [(i, self.placement(i)) for i in sorted(self._ids)]

    def peak_live_bytes(self) -> int:
        return int(N.lib().bl_plan_peak_live_bytes(self._h))

    def total_bytes(self) -> int:
        return int(N.lib().bl_plan_total_bytes(self._h))

    def valid_on(self, profile: DeviceProfile) -> bool:
        return bool(N.lib().bl_plan_valid_on(self._h, ctypes.byref(profile._c())))

    def __eq__(self, other):
        return (isinstance(other, MemoryPlan) and self.arenas() == other.arenas()
                and self.placements() == other.placements()
                and self.peak_live_bytes() == other.peak_live_bytes())

    __hash__ = None


class _CudaView:
    """__cuda_array_interface__ over a device address, so torch can view a
    placement without copying."""

    def __init__(self, ptr: int, shape, typestr: str, device: int):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None,
                                         "stream": None}
        self.device = device


class Arenas:
    """Arenas::new (arenas.rs:88) as ONE device allocation holding every arena
    of `plan`. Placements are bound by device address; nothing else is ever
    allocated for the plan's tensors."""

    def __init__(self, plan: MemoryPlan, device: int | None = None):
        """`device`: the CUDA ordinal (default: the current device)."""
        if device is None:
            import torch
            device = torch.cuda.current_device()
        handle = ctypes.c_void_p()
        N.check(N.lib().bl_arenas_create(plan.handle, device, ctypes.byref(handle)))
        self._h, self.device, self.plan = handle, device, plan
        self._lib = N.lib()  # the library outlives module teardown

    def close(self):
        if getattr(self, "_h", None):
            self._lib.bl_arenas_destroy(self._h)
            self._h = None

    __del__ = close

    def bytes(self) -> int:
        return int(N.lib().bl_arenas_bytes(self._h))

    def buffer(self, arena: int) -> int:
        out = ctypes.c_void_p()
        N.check(N.lib().bl_arenas_base(self._h, arena, ctypes.byref(out)))
        return int(out.value or 0)

    def binding(self, p: Placement) -> int:
        out = ctypes.c_void_p()
        N.check(N.lib().bl_arenas_binding(self._h, ctypes.byref(p._c()), ctypes.byref(out)))
        return int(out.value or 0)

    def tensor(self, p: Placement, shape, dtype):
        """A torch view of placement `p` (no copy), valid while this object
        lives. `dtype` is a torch dtype or one of f32, f16, u8, i16, i32
        (bf16 goes through an int16 carrier: __cuda_array_interface__ has no
        bf16 type)."""
        import math
        import torch
        names = {F32: torch.float32, F16: torch.float16, "u8": torch.uint8, "i16": torch.int16,
                 "i32": torch.int32}
        dt = names.get(dtype, dtype)
        carrier = {torch.float32: "<f4", torch.float16: "<f2", torch.bfloat16: "<i2",
                   torch.uint8: "|u1", torch.int16: "<i2", torch.int32: "<i4"}[dt]
        width = torch.empty((), dtype=dt).element_size()
        if math.prod(shape) * width > p.size:
            raise ValueError("a %s view of %s needs %d bytes, the placement has %d"
                             % (dt, tuple(shape), math.prod(shape) * width, p.size))
        view = _CudaView(self.binding(p), tuple(shape), carrier, self.device)
        t = torch.as_tensor(view, device="cuda:%d" % self.device)
        return t.view(dt) if dt == torch.bfloat16 else t

    def write(self, p: Placement, host, offset: int = 0, stream=None):
        """Host -> placement bytes (weights and inputs); `host` is a
        contiguous numpy array or CPU torch tensor."""
        ptr, nbytes = _host_ptr(host)
        N.check(N.lib().bl_arenas_write(self._h, ctypes.byref(p._c()), offset, ptr, nbytes,
                                        _stream(stream)))

    def read(self, p: Placement, host, offset: int = 0, stream=None):
        ptr, nbytes = _host_ptr(host)
        N.check(N.lib().bl_arenas_read(self._h, ctypes.byref(p._c()), offset, ptr, nbytes,
                                       _stream(stream)))


def _host_ptr(host):
    if hasattr(host, "data_ptr"):
        if host.is_cuda or not host.is_contiguous():
            raise ValueError("a contiguous host tensor is needed")
        return ctypes.c_void_p(host.data_ptr()), host.numel() * host.element_size()
    if not host.flags["C_CONTIGUOUS"]:
        raise ValueError("a contiguous host array is needed")
    return ctypes.c_void_p(host.ctypes.data), host.nbytes


def _stream(stream):
    return ctypes.c_void_p(stream.cuda_stream if stream is not None else 0)
