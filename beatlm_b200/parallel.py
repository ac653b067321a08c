"""Work across GPUs: one process per GPU, ``torch.distributed`` for the
plumbing (NCCL over NVLink on the B200s, gloo in the CPU tests).

The reference runs on one device, and queue order is its only
synchronisation (``beatlm-core/src/lib.rs:30-41``). The path splits across
GPUs in two ways:

* Independent streams (configs 3 and 4). Every rank runs whole frames of its
  own. There is no collective on the data path (``shard_frames``).
* Head partitioning for the long-sequence attention (config 5, T = 5477).
  Rank r holds heads ``head_slab(r, g, H)``, with Q/K/V made locally. It
  computes their output ``[T][H/g * 64]`` into its own slot of a
  ``[g][T][H/g * 64]`` buffer. One in-place all-gather fills the other slots,
  and a permute gives ``[T][H * 64]``: heads side by side, the reference's
  output layout (``kernel.rs:157-161``).
"""
from __future__ import annotations

import math


def head_slab(rank: int, world: int, heads: int) -> tuple[int, int]:
    """Heads [h0, h1) of `rank` when `world` ranks share `heads` heads. The
    heads must divide evenly, so that one all-gather moves equal slabs."""
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


def gather_heads(stacked, rank: int, world: int, out, group=None):
    """Completes ``stacked`` ``[g][T][w]``, where this rank's slot
    ``stacked[rank]`` already holds its heads' output, with an in-place
    all-gather. Then it writes ``out`` ``[T][g * w]``, heads side by side.
    Every rank must call it, in the same order as its other collectives."""
    import torch.distributed as dist
    g, t, w = stacked.shape
    if g != world or out.shape != (t, g * w):
        raise ValueError("gather_heads: stacked %s, out %s, world %d"
                         % (tuple(stacked.shape), tuple(out.shape), world))
    if world > 1:
        dist.all_gather_into_tensor(stacked.view(g * t, w), stacked[rank], group=group)
    out.view(t, g, w).copy_(stacked.permute(1, 0, 2))
    return out


class HeadParallelAttention:
    """Config 5 on one rank. The attention of heads ``head_slab(rank, world,
    heads)`` over this rank's packed Q/K/V ``[T][3][H/g][64]`` (Q/K of type
    `qk_dtype`, V f16). Its output goes into this rank's slot of ``stacked``.
    Then ``gather`` assembles ``out`` ``[T][H * 64]`` on every rank.

    The output is f16 by default: the all-gather moves 16 bits per value
    either way, and f16 rounding (relative 2^-11) keeps the result within
    relative L2 1e-3 of the f32 reference, which bf16 (2^-8) does not."""

    def __init__(self, tokens: int, heads: int, rank: int, world: int, qk_dtype: str = "bf16",
                 out_dtype: str = "f16", device="cuda", group=None):
        import torch
        self.t, self.h, self.rank, self.world = tokens, heads, rank, world
        self.h0, self.h1 = head_slab(rank, world, heads)
        self.qk_dtype, self.group = qk_dtype, group
        td = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[out_dtype]
        w = (self.h1 - self.h0) * 64
        self.stacked = torch.empty((world, tokens, w), dtype=td, device=device)
        self.slab = self.stacked[rank]
        self.out = (self.stacked.view(tokens, w) if world == 1 else
                    torch.empty((tokens, heads * 64), dtype=td, device=device))

    @property
    def local_heads(self) -> int:
        return self.h1 - self.h0

    def flops(self) -> float:
        """The whole op's FLOPs (all ranks): 4 T^2 H 64."""
        return 4.0 * self.t * self.t * self.h * 64

    def compute(self, qkv_local, stream=None):
        """This rank's heads into its slot (one kernel launch)."""
        from . import ops
        ops.attention(qkv_local, tokens=self.t, heads=self.local_heads, qk_dtype=self.qk_dtype,
                      out=self.slab, stream=stream)
        return self.slab

    def gather(self):
        if self.world == 1:
            return self.out
        return gather_heads(self.stacked, self.rank, self.world, self.out, group=self.group)

    def __call__(self, qkv_local, stream=None):
        self.compute(qkv_local, stream)
        return self.gather()
