"""Work across GPUs: one process per GPU, ``torch.distributed`` for the
plumbing (NCCL over NVLink on the B200s, gloo in the CPU tests).

The reference runs on one device, and queue order is its only
synchronisation (``beatlm-core/src/lib.rs:30-41``). The path splits across
GPUs in two ways:

* Independent streams (configs 3 and 4). Every rank runs whole frames of its
  own. There is no collective on the data path (``shard_frames``).
* Head partitioning for the long-sequence attention (config 5, T = 5477).
  Rank r holds heads ``head_slab(r, g, H)``, with Q/K/V made locally. Its
  attention kernel stores each finished output row of those heads into every
  rank's ``[T][H * 64]`` output (heads side by side, the reference's output
  layout, ``kernel.rs:157-161``) through peer memory over NVLink, and ends
  with an arrival barrier on the device (``bl_attention_peers``): one launch
  per rank per step, no separate collective, no permute. The ranks exchange
  CUDA IPC handles of their buffers once, at set-up, with one all-gather.
  ``exchange="nccl"`` keeps the plain collective form for comparison: the
  kernel writes this rank's slot of ``[g][T][H/g * 64]``, an in-place NCCL
  all-gather fills the others, and the output is a strided view of it.
"""
from __future__ import annotations

import ctypes
import math


def head_slab(rank: int, world: int, heads: int) -> tuple[int, int]:
    """Heads [h0, h1) of `rank` when `world` ranks share `heads` heads. The
    heads must divide evenly, so that every rank stores equal slabs."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank %d of world %d" % (rank, world))
    if heads % world != 0:
        raise ValueError("%d heads do not divide among %d ranks" % (heads, world))
    per = heads // world
    return rank * per, (rank + 1) * per


def shard_frames(frames: int, rank: int, world: int) -> range:
    """The frames of `frames` independent streams that `rank` runs (configs
    3 and 4: one stream per GPU when frames == world)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank %d of world %d" % (rank, world))
    per = math.ceil(frames / world)
    return range(min(frames, rank * per), min(frames, (rank + 1) * per))


def exchange_handles(handle: bytes, world: int, group=None) -> bytes:
    """Every rank's handle (equal lengths) in rank order: one all-gather on
    the group's backend (device tensors for NCCL, host tensors for gloo).
    Every rank must call it, in the same order as its other collectives."""
    import torch
    import torch.distributed as dist
    n = len(handle)
    if world == 1:
        return bytes(handle)
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    mine = torch.tensor(list(handle), dtype=torch.uint8, device=dev)
    everyone = torch.empty(world * n, dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(everyone, mine, group=group)
    return bytes(everyone.cpu().tolist())


def gather_heads(stacked, rank: int, world: int, group=None):
    """The NCCL form of the exchange: completes ``stacked`` ``[g][T][w]``,
    where this rank's slot already holds its heads' output, with an in-place
    all-gather, and returns the ``[T][g][w]`` strided view (heads side by
    side when read row by row; no copy). Every rank must call it, in the
    same order as its other collectives."""
    import torch.distributed as dist
    g, t, w = stacked.shape
    if g != world:
        raise ValueError("gather_heads: stacked %s for world %d" % (tuple(stacked.shape), world))
    if world > 1:
        dist.all_gather_into_tensor(stacked.view(g * t, w), stacked[rank], group=group)
    return stacked.permute(1, 0, 2)


class _DeviceArray:
    """A device buffer the library owns, shown to torch without a copy
    (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def device_view(ptr: int, shape: tuple, dtype):
    """A torch tensor over library-owned device memory at `ptr` (f16, bf16
    or f32); the memory must outlive the tensor."""
    import torch
    if dtype == torch.bfloat16:
        return torch.as_tensor(_DeviceArray(ptr, shape, "<i2"), device="cuda").view(torch.bfloat16)
    code = {torch.float16: "<f2", torch.float32: "<f4"}[dtype]
    return torch.as_tensor(_DeviceArray(ptr, shape, code), device="cuda")


class PeerBuffers:
    """This rank's peer buffer (``bl_peers_*``): a header of arrival flags
    and two output slots of ``slot_bytes``, mapped by every other rank."""

    def __init__(self, rank: int, world: int, slot_bytes: int):
        from . import _native as N
        self.N = N
        self.rank, self.world, self.slot_bytes = rank, world, slot_bytes
        h = ctypes.c_void_p()
        N.check(N.lib().bl_peers_create(rank, world, slot_bytes, ctypes.byref(h)))
        self._h = h

    @staticmethod
    def buffer_bytes(slot_bytes: int) -> int:
        from . import _native as N
        return int(N.lib().bl_peers_buffer_bytes(slot_bytes))

    def handle(self) -> bytes:
        buf = (ctypes.c_uint8 * self.N.PEER_HANDLE_BYTES)()
        self.N.check(self.N.lib().bl_peers_handle(self._h, buf))
        return bytes(buf)

    def open(self, handles: bytes):
        """Maps every other rank's buffer from all ranks' handles (rank order)."""
        buf = (ctypes.c_uint8 * len(handles)).from_buffer_copy(handles)
        self.N.check(self.N.lib().bl_peers_open(self._h, buf, self.world))

    def attach(self, rank: int, buffer):
        """Rank `rank`'s buffer mapped by the caller (a device tensor of at
        least ``buffer_bytes(slot_bytes)`` bytes, 256-byte aligned, zeroed)."""
        self.N.check(self.N.lib().bl_peers_attach(self._h, rank, buffer.data_ptr()))

    def slot(self, slot: int, shape: tuple, dtype):
        return device_view(self.N.lib().bl_peers_slot(self._h, slot), shape, dtype)

    def next_epoch(self) -> int:
        return int(self.N.lib().bl_peers_next_epoch(self._h))

    def close(self):
        if self._h:
            self.N.lib().bl_peers_destroy(self._h)
            self._h = None


class HeadParallelAttention:
    """Config 5 on one rank. The attention of heads ``head_slab(rank, world,
    heads)`` over this rank's packed Q/K/V ``[T][3][H/g][64]`` (Q/K of type
    `qk_dtype`, V f16), assembled on every rank as ``out`` ``[T][H * 64]``.

    ``exchange="peers"`` (default with several ranks): one
    ``bl_attention_peers`` launch per step stores the rows into every rank's
    output and waits on the device for the others (``out`` is the slot the
    launch filled). ``exchange="nccl"``: one ``bl_attention`` launch into this
    rank's slot of ``[g][T][H/g * 64]`` and an in-place NCCL all-gather
    (``out`` is a strided ``[T][g][H/g * 64]`` view).

    The output is f16 by default: 16 bits per value cross NVLink either way,
    and f16 rounding (relative 2^-11) keeps the result within relative L2
    1e-3 of the f32 reference, which bf16 (2^-8) does not."""

    def __init__(self, tokens: int, heads: int, rank: int, world: int, qk_dtype: str = "bf16",
                 out_dtype: str = "f16", device="cuda", group=None, exchange: str | None = None):
        import torch
        self.t, self.h, self.rank, self.world = tokens, heads, rank, world
        self.h0, self.h1 = head_slab(rank, world, heads)
        self.qk_dtype, self.group, self.out_dtype = qk_dtype, group, out_dtype
        self.exchange = exchange or ("peers" if world > 1 else "none")
        if self.exchange not in ("peers", "nccl", "none"):
            raise ValueError("exchange %r" % self.exchange)
        if world > 1 and self.exchange == "none":
            raise ValueError("several ranks need an exchange")
        self.td = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[out_dtype]
        w = (self.h1 - self.h0) * 64
        self.peers = None
        self.local = torch.empty((tokens, w), dtype=self.td, device=device)  # compute_local
        if self.exchange == "peers":
            self.peers = PeerBuffers(rank, world, tokens * heads * 64 * self.local.element_size())
            self.peers.open(exchange_handles(self.peers.handle(), world, group))
            self._slots = [self.peers.slot(i, (tokens, heads * 64), self.td) for i in range(2)]
            self.out = self._slots[0]
        else:
            self.stacked = torch.empty((world, tokens, w), dtype=self.td, device=device)
            self.slab = self.stacked[rank]
            self.out = self.stacked.permute(1, 0, 2) if world > 1 else self.stacked[0]

    @property
    def local_heads(self) -> int:
        return self.h1 - self.h0

    def flops(self) -> float:
        """The whole op's FLOPs (all ranks): 4 T^2 H 64."""
        return 4.0 * self.t * self.t * self.h * 64

    def exchange_name(self) -> str:
        return {"peers": "attention kernel stores rows into every rank's output over NVLink "
                         "(bl_attention_peers), device arrival barrier",
                "nccl": "NCCL all_gather_into_tensor of head slabs, strided view",
                "none": "none"}[self.exchange]

    def _args(self, qkv_local, out, out_row_stride=None):
        from . import ops
        return ops.attention_args(qkv_local, tokens=self.t, heads=self.local_heads, out=out,
                                  qk_dtype=self.qk_dtype, out_dtype=self.out_dtype,
                                  out_row_stride=out_row_stride)

    def launch_shape(self, qkv_local) -> dict:
        """The attention launch this rank runs: query tiles per CTA, key
        splits and the unsplit query groups of a mixed grid (the peer
        exchange takes two query tiles)."""
        from . import ops
        a = self._args(qkv_local, self.local)
        if self.exchange == "peers":
            a.query_tiles = 2
        qt, splits, unsplit = ops.attention_choice(a)
        return {"query_tiles": qt, "kv_splits": splits, "unsplit_groups": unsplit}

    def compute_local(self, qkv_local, stream=None):
        """This rank's heads into a local [T][H/g * 64] buffer, no exchange
        (the attention alone, for timing)."""
        from . import ops
        ops.attention(qkv_local, tokens=self.t, heads=self.local_heads, qk_dtype=self.qk_dtype,
                      out=self.local, stream=stream)
        return self.local

    def __call__(self, qkv_local, stream=None):
        from . import _native as N
        from . import ops
        if self.exchange == "peers":
            a = self._args(qkv_local, self.local, out_row_stride=self.h * 64)
            slot = ctypes.c_uint32()
            N.check(N.lib().bl_attention_peers(ctypes.byref(a), self.peers._h, self.h0 * 64,
                                               ctypes.byref(slot), ops._stream_ptr(stream)))
            self.out = self._slots[slot.value]
            return self.out
        ops.attention(qkv_local, tokens=self.t, heads=self.local_heads, qk_dtype=self.qk_dtype,
                      out=self.slab, stream=stream)
        if self.exchange == "nccl":
            import torch
            with torch.cuda.stream(stream) if stream is not None else _null():
                self.out = gather_heads(self.stacked, self.rank, self.world, group=self.group)
        return self.out

    def close(self):
        if self.peers is not None:
            self.peers.close()
            self.peers = None


def _null():
    import contextlib
    return contextlib.nullcontext()
