"""The ViT encoder of Depth-Anything-V2 on the B200 backend.

Mirrors the reference's graph builders
(``crates/beatlm/src/model/depth_anything_v2.rs``: ``block``/``layer_of``
252-427, ``encoder`` 435-545) as fused launches of ``libbeatlm_b200.so``:

    per block (5 launches; the reference lowers the same block to 9 kernels,
    kernel.rs:3796-3844):
      qkv  = LN1(x) . Wqkv + b        GEMM, LayerNorm prologue, packed Q|K|V
                                      (Q/K in the model dtype, V in f16)
      o    = attention(qkv)           fused flash kernel (scores never stored)
      x    = x + ls1 * (o . Wo + bo)  GEMM, LayerScale + residual epilogue
      h    = gelu_erf(LN2(x) . W1 + b1)  GEMM, LayerNorm prologue, GELU epilogue
      x    = x + ls2 * (h . W2 + b2)  GEMM, LayerScale + residual epilogue
    embedding: patch matrix + class rows (1 launch pair), patch GEMM with the
    position-embedding Add in its epilogue; features: final LayerNorm with
    TokensToMap folded in.

Weights are given in the reference's layouts (linear weights ``[in][out]``,
``model/mod.rs:274-353``) as f32 and uploaded once, transposed to
``[out][in]`` and rounded to the compute type. All activation buffers are
allocated once per (frames) shape, so a forward pass allocates nothing.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np

from . import ops


@dataclasses.dataclass(frozen=True)
class ViTConfig:
    dim: int = 384
    heads: int = 6
    mlp: int = 1536
    layers: int = 12
    patch: int = 14
    side: int = 518
    cin: int = 3
    eps: float = 1e-6  # DINOV2_LAYER_NORM_EPSILON, depth_anything_v2.rs:114
    out_indices: tuple = (3, 6, 9, 12)

    @property
    def grid(self) -> int:
        return self.side // self.patch

    @property
    def tokens(self) -> int:
        return self.grid * self.grid + 1

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads

    @property
    def taps(self) -> int:
        return self.patch * self.patch * self.cin

    @property
    def k_pad(self) -> int:
        return (self.taps + 63) // 64 * 64

    @staticmethod
    def small(**kw) -> "ViTConfig":
        """Depth-Anything-V2-Small (load/depth_anything_v2.rs:126-147)."""
        return ViTConfig(**kw)

    @staticmethod
    def large(**kw) -> "ViTConfig":
        """ViT-L/14 shape of BASELINE config 4."""
        base = dict(dim=1024, heads=16, mlp=4096, layers=24, out_indices=(6, 12, 18, 24))
        base.update(kw)
        return ViTConfig(**base)

    def flops_per_frame(self) -> dict:
        t, d, m = self.tokens, self.dim, self.mlp
        linear = 2.0 * t * d * (3 * d + d + 2 * m) * self.layers
        attn = 4.0 * t * t * d * self.layers
        patch = 2.0 * (t - 1) * self.taps * d
        return {"linear": linear, "attention": attn, "patch": patch,
                "total": linear + attn + patch}


BLOCK_NAMES = ("norm1_g", "norm1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "ls1",
               "norm2_g", "norm2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "ls2")


def _lcg_uniform(seed, count, low, high):
    """The reference's seeded generator (net.rs:183-203), in numpy."""
    s = np.uint64(seed)
    mul, inc = np.uint64(6364136223846793005), np.uint64(1442695040888963407)
    out = np.empty(count, np.float32)
    # vectorised by jumping: sequential is fine at these sizes
    vals = np.empty(count, np.uint64)
    with np.errstate(over="ignore"):
        for i in range(count):
            s = s * mul + inc
            vals[i] = s
    out[:] = (vals >> np.uint64(40)).astype(np.float32) / np.float32(1 << 24)
    return (np.float32(low) + np.float32(high - low) * out).astype(np.float32)


def block_weights_by_role(seed: int, dim: int, mlp: int, uniform=None) -> dict:
    """Random block weights drawn as the reference's block test draws them
    (crates/beatlm-bench/src/vit.rs:203-238): gamma U(0.8,1.2), LayerScale
    U(0.1,1), linear weights U(+-1/sqrt(fan_in)), the rest U(+-0.1); linear
    weights in the reference's [in][out] layout."""
    u = uniform or _lcg_uniform
    fan = lambda s, n, f: u(s, n, -1 / math.sqrt(f), 1 / math.sqrt(f))
    return {
        "norm1_g": u(seed, dim, 0.8, 1.2), "norm1_b": u(seed + 1, dim, -0.1, 0.1),
        "qkv_w": fan(seed + 2, dim * 3 * dim, dim), "qkv_b": u(seed + 3, 3 * dim, -0.1, 0.1),
        "proj_w": fan(seed + 4, dim * dim, dim), "proj_b": u(seed + 5, dim, -0.1, 0.1),
        "ls1": u(seed + 6, dim, 0.1, 1.0),
        "norm2_g": u(seed + 7, dim, 0.8, 1.2), "norm2_b": u(seed + 8, dim, -0.1, 0.1),
        "fc1_w": fan(seed + 9, dim * mlp, dim), "fc1_b": u(seed + 10, mlp, -0.1, 0.1),
        "fc2_w": fan(seed + 11, mlp * dim, mlp), "fc2_b": u(seed + 12, dim, -0.1, 0.1),
        "ls2": u(seed + 13, dim, 0.1, 1.0),
    }


def block_weights_normal(rng: np.random.Generator, dim: int, mlp: int, std=0.02,
                         layer_scale=1.0) -> dict:
    """linear weights N(0, std), biases 0, LayerNorm
    gamma 1 / beta 0, LayerScale `layer_scale` (BASELINE gives no value; 1)."""
    n = lambda *s: (rng.standard_normal(int(np.prod(s)), dtype=np.float32) * std)
    z = lambda k: np.zeros(k, np.float32)
    one = lambda k: np.ones(k, np.float32)
    return {"norm1_g": one(dim), "norm1_b": z(dim), "qkv_w": n(dim, 3 * dim),
            "qkv_b": z(3 * dim), "proj_w": n(dim, dim), "proj_b": z(dim),
            "ls1": one(dim) * layer_scale, "norm2_g": one(dim), "norm2_b": z(dim),
            "fc1_w": n(dim, mlp), "fc1_b": z(mlp), "fc2_w": n(mlp, dim), "fc2_b": z(dim),
            "ls2": one(dim) * layer_scale}


def _round(x: np.ndarray, dtype: str) -> np.ndarray:
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, np.float32))
    return t.to(torch.bfloat16 if dtype == "bf16" else torch.float16).float().numpy()


class DeviceBlock:
    """One block's weights on the device: linear weights [out][in] in the
    compute type, vectors in f32."""

    def __init__(self, w: dict, dim: int, mlp: int, dtype: str = "bf16", device="cuda"):
        import torch
        td = torch.bfloat16 if dtype == "bf16" else torch.float16
        self.dtype, self.dim, self.mlp = dtype, dim, mlp
        f32 = lambda k: torch.from_numpy(np.ascontiguousarray(w[k], np.float32)).to(device)

        def lin(k, fan_in, fan_out):
            m = np.asarray(w[k], np.float32).reshape(fan_in, fan_out).T
            return torch.from_numpy(np.ascontiguousarray(m)).to(td).to(device)

        self.norm1 = (f32("norm1_g"), f32("norm1_b"))
        self.qkv_w, self.qkv_b = lin("qkv_w", dim, 3 * dim), f32("qkv_b")
        self.proj_w, self.proj_b = lin("proj_w", dim, dim), f32("proj_b")
        self.ls1 = f32("ls1")
        self.norm2 = (f32("norm2_g"), f32("norm2_b"))
        self.fc1_w, self.fc1_b = lin("fc1_w", dim, mlp), f32("fc1_b")
        self.fc2_w, self.fc2_b = lin("fc2_w", mlp, dim), f32("fc2_b")
        self.ls2 = f32("ls2")

    @staticmethod
    def rounded(w: dict, dtype: str) -> dict:
        """The weights as the device holds them, back in f32 and the
        reference layout: what an oracle comparison must be given."""
        out = dict(w)
        for k in ("qkv_w", "proj_w", "fc1_w", "fc2_w"):
            out[k] = _round(w[k], dtype)
        return out


class Buffers:
    """Activation buffers for `frames` frames of `tokens` tokens, allocated
    once (zero allocation in the forward pass). The image buffer is what a
    prebuilt program reads, so a caller writes each frame's pixels there."""

    def __init__(self, cfg: ViTConfig, frames: int, dtype: str, tokens: int | None = None,
                 device="cuda", features: bool = True, alloc=None, slots: int = 1):
        """``alloc(name, shape, torch_dtype)`` makes each buffer (default: a
        torch allocation on `device`); the static plan passes views of its
        arena instead. ``slots``: one input image and one set of feature maps
        per job in flight (the reference's Net slots,
        crates/beatlm-host/src/slots.rs:1-30): slot 0 is ``image`` /
        ``features``, slot s > 0 its own pair (``images[s]``,
        ``slot_features[s]``), live for the whole program; everything else is
        shared, since jobs run as one sequence."""
        import torch
        if alloc is None:
            alloc = lambda name, shape, dt: torch.empty(shape, dtype=dt, device=device)
        td = torch.bfloat16 if dtype == "bf16" else torch.float16
        t = cfg.tokens if tokens is None else tokens
        rows = frames * t
        self.frames, self.tokens, self.rows = frames, t, rows
        self.image = alloc("image", (frames, cfg.side, cfg.side, cfg.cin), torch.float32)
        self.image.zero_()
        self.x = alloc("x", (rows, cfg.dim), torch.float32)
        self.qkv = alloc("qkv", (rows, 3 * cfg.dim), torch.int16)
        self.o = alloc("o", (rows, cfg.dim), td)
        self.xn = alloc("xn", (rows, cfg.dim), td)
        self.h = alloc("h", (rows, cfg.mlp), td)
        self.patches = alloc("patches", (frames * (t - 1), cfg.k_pad), td)
        # per-row partial LayerNorm statistics written by the GEMMs that write
        # x: (mean, M2) for each 32-column slice
        self.stats1 = alloc("stats1", (rows, cfg.dim // 32, 2), torch.float32)
        self.stats2 = alloc("stats2", (rows, cfg.dim // 32, 2), torch.float32)
        # exchange buffer of the epilogue LayerNorm (counters, then per-slice
        # statistics); zero-filled once, every launch leaves it so
        sync_bytes = (8 * ((rows + 127) // 128) + 15) // 16 * 16 + 8 * rows * (cfg.dim // 32)
        self.norm_sync = alloc("norm_sync", (sync_bytes,), torch.uint8)
        self.norm_sync.zero_()
        self.features = ([alloc("features.%d" % i, (frames * (t - 1), cfg.dim), torch.float32)
                          for i in cfg.out_indices] if features else [])
        self.images, self.slot_features = [self.image], [self.features]
        for slot in range(1, slots):
            img = alloc("image.s%d" % slot, (frames, cfg.side, cfg.side, cfg.cin), torch.float32)
            img.zero_()
            self.images.append(img)
            self.slot_features.append(
                [alloc("features.%d.s%d" % (i, slot), (frames * (t - 1), cfg.dim), torch.float32)
                 for i in cfg.out_indices] if features else [])

    # Lifetimes for the static plan, in kernel-spec order of the encoder
    # program (spec 0 patchify, spec 1 patch GEMM, blocks from spec 2). The
    # image is refilled by the host every frame and the features are read
    # after it, so both live for the whole program, as do the weights and
    # the residual stream; the patch matrix dies at the patch GEMM and the
    # block scratch is born at the first block, so those may share bytes.
    @staticmethod
    def lifetime(name: str, last: int) -> tuple[int, int]:
        if name == "patches":
            return 0, 1
        if name in ("qkv", "o", "xn", "h", "stats1", "stats2"):
            return 2, last
        return 0, last


def _on_stream(stream):
    """A context that makes ``stream`` current (no-op for None), so torch
    copies and temporaries and every library call given no stream of its own
    run on one stream."""
    import contextlib
    import torch
    return torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext()


def _weights_gemm(w, **kw):
    """``ops.gemm_args`` for a GEMM whose B, bias and scale are model weights
    (never written by the kernel before it: fetched before that one ends)."""
    return ops.gemm_args(w, weights_static=True, **kw)


def norm_epilogue_fits(rows: int, dim: int) -> bool:
    """Whether a GEMM writing `rows` x `dim` can carry the epilogue LayerNorm:
    every 32-column tile must be resident at once, one per SM."""
    import torch
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return dim <= 512 and -(-rows // 128) * (dim // 32) <= sms


def block_specs(blk: DeviceBlock, cfg: ViTConfig, buf: Buffers, layer: int = 0,
                parts: int = 1, fused_ln=False, next_norm=None) -> list:
    """The fused kernels of one pre-norm block (reference.rs:520-544), in
    place on ``buf.x``:
    x1 = x + ls1 * proj(attention(norm1(x))); x = x1 + ls2 * fc2(gelu(fc1(norm2(x1)))).

    ``fused_ln=False`` (7 kernels): each LayerNorm is its own bandwidth-bound
    kernel writing 16-bit rows that the next GEMM loads by TMA.
    ``fused_ln=True`` (5 kernels; 7 for block 0): the GEMM that writes x also
    writes each row's partial statistics (proj for norm2, the previous block's
    fc2 for norm1: ``buf.stats2`` / ``buf.stats1``), and the QKV / fc1 GEMM
    normalises its A operand from x in its prologue with them, so no
    LayerNorm launch and no pass over the rows remain. Block 0's norm1 reads
    the embedding's output, for which no statistics exist: it stays a
    standalone LayerNorm.
    ``fused_ln="epilogue"`` (5 kernels; 6 for block 0): proj writes x and
    norm2(x) (``buf.xn``), fc2 writes x and ``next_norm`` (the next block's
    norm1 weights; none for the last block) of it, each LayerNorm computed in
    the GEMM's epilogue from statistics its column tiles exchange; QKV and
    fc1 load ``buf.xn`` by TMA. Where the GEMM has more 32-column tiles than
    the device has SMs (``norm_epilogue_fits``) the block is built as with
    ``fused_ln=False``."""
    from .runtime import Spec
    d = cfg.dim
    name = "block%d." % layer
    attn = Spec(ops.attention_args(buf.qkv, tokens=buf.tokens, heads=cfg.heads,
                                   head_dim=cfg.head_dim, batch=buf.frames, qk_dtype=blk.dtype,
                                   out=buf.o), name + "attention", parts)
    if fused_ln == "epilogue" and not norm_epilogue_fits(buf.rows, d):
        fused_ln = False
    if fused_ln == "epilogue":
        ep = lambda w: None if w is None else (w[0], w[1], cfg.eps, buf.xn)
        head = ([Spec(ops.layernorm_args(buf.x, blk.norm1[0], blk.norm1[1], cfg.eps, out=buf.xn),
                      name + "norm1", parts)] if layer == 0 else [])
        return head + [
            Spec(_weights_gemm(blk.qkv_w, a=buf.xn, bias=blk.qkv_b, out=buf.qkv,
                               out_dtype=blk.dtype, out_split=(2 * d, "f16")), name + "qkv", parts),
            attn,
            Spec(_weights_gemm(blk.proj_w, a=buf.o, bias=blk.proj_b, chan_scale=blk.ls1,
                               residual=buf.x, out=buf.x, norm=ep(blk.norm2),
                               norm_sync=buf.norm_sync), name + "proj", parts),
            Spec(_weights_gemm(blk.fc1_w, a=buf.xn, bias=blk.fc1_b, act="gelu_erf", out=buf.h),
                 name + "fc1", parts),
            Spec(_weights_gemm(blk.fc2_w, a=buf.h, bias=blk.fc2_b, chan_scale=blk.ls2,
                               residual=buf.x, out=buf.x, norm=ep(next_norm),
                               norm_sync=buf.norm_sync if next_norm is not None else None),
                 name + "fc2", parts),
        ]
    stats = (lambda s: s) if fused_ln else (lambda s: None)
    proj = Spec(_weights_gemm(blk.proj_w, a=buf.o, bias=blk.proj_b, chan_scale=blk.ls1,
                              residual=buf.x, out=buf.x, stats_out=stats(buf.stats2)),
                name + "proj", parts)
    fc2 = Spec(_weights_gemm(blk.fc2_w, a=buf.h, bias=blk.fc2_b, chan_scale=blk.ls2,
                             residual=buf.x, out=buf.x, stats_out=stats(buf.stats1)),
               name + "fc2", parts)
    if fused_ln:
        if layer == 0:
            head = [
                Spec(ops.layernorm_args(buf.x, blk.norm1[0], blk.norm1[1], cfg.eps, out=buf.xn),
                     name + "norm1", parts),
                Spec(_weights_gemm(blk.qkv_w, a=buf.xn, bias=blk.qkv_b, out=buf.qkv,
                                   out_dtype=blk.dtype, out_split=(2 * d, "f16")),
                     name + "qkv", parts)]
        else:
            head = [Spec(_weights_gemm(blk.qkv_w, ln=(buf.x, blk.norm1[0], blk.norm1[1], cfg.eps),
                                       ln_stats=buf.stats1, bias=blk.qkv_b, out=buf.qkv,
                                       out_dtype=blk.dtype, out_split=(2 * d, "f16")),
                         name + "qkv", parts)]
        return head + [
            attn, proj,
            Spec(_weights_gemm(blk.fc1_w, ln=(buf.x, blk.norm2[0], blk.norm2[1], cfg.eps),
                               ln_stats=buf.stats2, bias=blk.fc1_b, act="gelu_erf", out=buf.h),
                 name + "fc1", parts),
            fc2,
        ]
    return [
        Spec(ops.layernorm_args(buf.x, blk.norm1[0], blk.norm1[1], cfg.eps, out=buf.xn),
             name + "norm1", parts),
        Spec(_weights_gemm(blk.qkv_w, a=buf.xn, bias=blk.qkv_b, out=buf.qkv, out_dtype=blk.dtype,
                           out_split=(2 * d, "f16")), name + "qkv", parts),
        attn, proj,
        Spec(ops.layernorm_args(buf.x, blk.norm2[0], blk.norm2[1], cfg.eps, out=buf.xn),
             name + "norm2", parts),
        Spec(_weights_gemm(blk.fc1_w, a=buf.xn, bias=blk.fc1_b, act="gelu_erf", out=buf.h),
             name + "fc1", parts),
        fc2,
    ]


def run_block(blk: DeviceBlock, cfg: ViTConfig, buf: Buffers, stream=None, parts: int = 1,
              fused_ln: bool = False):
    """One block, built and encoded at once (tests; the encoder prebuilds)."""
    from .runtime import Kernels
    k = Kernels(block_specs(blk, cfg, buf, parts=parts, fused_ln=fused_ln))
    k.encode_all(stream)
    return k


class Encoder:
    """The DA-V2 ViT encoder (depth_anything_v2.rs:435-545) on the device."""

    def __init__(self, cfg: ViTConfig, weights: dict, dtype: str = "bf16", device="cuda",
                 planned_frames: int | None = None, fused_ln: bool | None = None,
                 slots: int = 1):
        """``weights``: ``blocks`` (list of per-block dicts in the reference
        layout), ``patch_w`` [patch][patch][cin][dim] (HWIO), ``patch_b`` [dim],
        ``cls`` [dim], ``pos`` [tokens][dim], ``norm_g``/``norm_b`` [dim].

        ``planned_frames``: place every weight and every activation buffer of
        the ``planned_frames``-frame program in ONE device allocation laid out
        by the static memory plan (memory.MemoryPlan, then memory.Arenas;
        the reference's MemoryPlan::new and Arenas::new). The weights are
        staged on the host and written into their placements; afterwards
        nothing is allocated. Without it each buffer is its own torch
        allocation.

        ``fused_ln``: the LayerNorms inside the blocks are fed by statistics
        from the GEMM before them (``block_specs``). Off by default: measured
        at ViT-S (one frame), the QKV and fc1 GEMMs that normalise their A
        operand from the f32 rows (brought by TMA, normalised by the epilogue
        warps) take longer than a standalone LayerNorm plus a GEMM that loads
        16-bit rows by TMA (676 against 633 us per frame). ``fused_ln="epilogue"``: the GEMMs that
        write x also write the next LayerNorm's output (``block_specs``);
        needs every 32-column tile of those GEMMs resident at once (ViT-S
        at one frame: 132 tiles). Also measured slower at ViT-S, one frame:
        668 against 640 us, the column tiles' exchange of statistics through
        L2 costing more than the LayerNorm launch it replaces.

        ``slots``: input/output slots for that many jobs in flight
        (``Buffers``); ``program(frames)`` carries one binding set per slot,
        and set s reads slot s's image and writes its feature maps."""
        import torch
        td = torch.bfloat16 if dtype == "bf16" else torch.float16
        self.cfg, self.dtype = cfg, dtype
        self.slots = max(1, int(slots))
        self.fused_ln = fused_ln if fused_ln == "epilogue" else bool(fused_ln)
        self.arena, self.plan = None, None
        stage = "cpu" if planned_frames is not None else device
        self.blocks = [DeviceBlock(w, cfg.dim, cfg.mlp, dtype, stage) for w in weights["blocks"]]
        pw = np.zeros((cfg.dim, cfg.k_pad), np.float32)
        pw[:, :cfg.taps] = np.asarray(weights["patch_w"], np.float32).reshape(cfg.taps, cfg.dim).T
        f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(stage)
        self.patch_w = torch.from_numpy(pw).to(td).to(stage)
        self.patch_b = f32(weights["patch_b"])
        self.cls = f32(weights["cls"])
        self.pos = f32(np.asarray(weights["pos"], np.float32).reshape(cfg.tokens, cfg.dim))
        self.norm = (f32(weights["norm_g"]), f32(weights["norm_b"]))
        self._buffers = {}
        self._programs = {}
        if planned_frames is not None:
            self._place_in_arena(planned_frames, torch.device(device))

    def _weights(self):
        """(owner, attribute, index or None) of every weight tensor."""
        out = []
        for owner in [self] + self.blocks:
            for attr, v in sorted(vars(owner).items()):
                if attr.startswith("_") or attr in ("blocks", "cfg"):
                    continue
                if hasattr(v, "data_ptr"):
                    out.append((owner, attr, None))
                elif isinstance(v, tuple) and v and all(hasattr(x, "data_ptr") for x in v):
                    out += [(owner, attr, i) for i in range(len(v))]
        return out

    def memory_plan(self, frames: int, profile):
        """The static plan of every weight and activation buffer of the
        `frames`-frame program against `profile` (host-only). Tensor ids:
        the weights first, in ``_weights()`` order, then the activation
        buffers in the order Buffers makes them. Returns (plan, weights,
        activations as (name, shape, torch dtype))."""
        import torch
        from .memory import F16, F32, MemoryPlan, TensorDesc
        last = len(self.specs_layout(frames)) - 1
        acts = []
        Buffers(self.cfg, frames, self.dtype, device="meta", slots=self.slots,
                alloc=lambda n, s, dt: acts.append((n, s, dt)) or torch.empty(s, dtype=dt,
                                                                              device="meta"))
        wts = self._weights()
        descs = []
        for k, (o, a, i) in enumerate(wts):
            t = getattr(o, a) if i is None else getattr(o, a)[i]
            descs.append(TensorDesc(k, F32 if t.element_size() == 4 else F16, t.numel(), 0, last))
        for k, (name, shape, dt) in enumerate(acts, start=len(wts)):
            first, end = Buffers.lifetime(name.split(".")[0], last)
            descs.append(TensorDesc(k, F32 if torch.empty((), dtype=dt).element_size() == 4
                                    else F16, int(np.prod(shape)), first, end))
        return MemoryPlan(descs, profile), wts, acts

    def _place_in_arena(self, frames: int, device):
        import torch
        from .memory import Arenas, DeviceProfile
        cfg = self.cfg
        # "cuda" without an index is the current device (one process per GPU
        # sets it first), never device 0 by default
        index = device.index if device.index is not None else torch.cuda.current_device()
        self.plan, wts, acts = self.memory_plan(frames, DeviceProfile.cuda(index))
        self.arena = Arenas(self.plan, index)
        get = lambda o, a, i: getattr(o, a) if i is None else getattr(o, a)[i]
        for k, (o, a, i) in enumerate(wts):
            src = get(o, a, i)
            view = self.arena.tensor(self.plan.placement(k), tuple(src.shape), src.dtype)
            view.copy_(src)
            if i is None:
                setattr(o, a, view)
            else:
                tup = list(getattr(o, a))
                tup[i] = view
                setattr(o, a, tuple(tup))
        views = {name: self.arena.tensor(self.plan.placement(k), shape, dt)
                 for k, (name, shape, dt) in enumerate(acts, start=len(wts))}
        self._buffers[frames] = Buffers(cfg, frames, self.dtype, slots=self.slots,
                                        alloc=lambda n, s, dt: views[n])
        torch.cuda.synchronize(device)

    def specs_layout(self, frames: int) -> list:
        """The spec labels of the encoder program, in order (no device work)."""
        cfg = self.cfg
        out = ["embed.patchify", "embed.patch"]
        for i in range(cfg.layers):
            kinds = ("norm1", "qkv", "attention", "proj", "norm2", "fc1", "fc2")
            if self._fused(frames):
                kinds = (("norm1", "qkv") if i == 0 else ("qkv",)) + ("attention", "proj", "fc1",
                                                                      "fc2")
            out += ["block%d.%s" % (i, k) for k in kinds]
            if (i + 1) in cfg.out_indices:
                out.append("features.%d" % (i + 1))
        return out

    def _fused(self, frames: int):
        """The LayerNorm mode the blocks are built with for `frames` frames."""
        if self.fused_ln == "epilogue" and not norm_epilogue_fits(frames * self.cfg.tokens,
                                                                  self.cfg.dim):
            return False
        return self.fused_ln

    def buffers(self, frames: int) -> Buffers:
        if frames not in self._buffers:
            if self.arena is not None:
                raise ValueError("this encoder's memory is planned for %s frames"
                                 % sorted(self._buffers))
            self._buffers[frames] = Buffers(self.cfg, frames, self.dtype, slots=self.slots)
        return self._buffers[frames]

    def specs(self, frames: int, layers: int | None = None, parts: int = 1,
              slot: int = 0) -> list:
        """The encoder as kernel specs over the buffers of `frames` frames,
        reading slot `slot`'s image and writing its feature maps."""
        from .runtime import Spec
        cfg, buf = self.cfg, self.buffers(frames)
        if not 0 <= slot < self.slots:
            raise ValueError("slot %d of %d" % (slot, self.slots))
        t = cfg.tokens
        out = [
            Spec(ops.patchify_args(buf.images[slot], frames=frames, side=cfg.side, patch=cfg.patch,
                                   cin=cfg.cin, k_pad=cfg.k_pad, a_out=buf.patches,
                                   a_dtype=self.dtype, cls=self.cls, pos=self.pos, x=buf.x),
                 "embed.patchify"),
            Spec(_weights_gemm(self.patch_w, a=buf.patches, bias=self.patch_b, residual=self.pos,
                               res_period=t, out=buf.x, out_row_offset=1, out_group=(t - 1, 1)),
                 "embed.patch", parts),
        ]
        n = cfg.layers if layers is None else layers
        for i in range(n):
            nxt = self.blocks[i + 1].norm1 if i + 1 < n else None
            out += block_specs(self.blocks[i], cfg, buf, i, parts, fused_ln=self.fused_ln,
                               next_norm=nxt)
            if (i + 1) in cfg.out_indices:
                f = buf.slot_features[slot][cfg.out_indices.index(i + 1)]
                out.append(Spec(ops.layernorm_args(buf.x, self.norm[0], self.norm[1], cfg.eps,
                                                   out=f, in_row_offset=1, in_group=(t - 1, 1)),
                                "features.%d" % (i + 1), parts))
        return out

    def program(self, frames: int = 1, layers: int | None = None, parts: int = 1):
        """The encoder's kernels over the buffers of `frames` frames, with one
        binding set per input/output slot (the reference's Net slots bound
        through Kernels::new's sets, crates/beatlm-host/src/slots.rs:45-60):
        set s substitutes slot s's image and feature maps for slot 0's, so
        ``encode(k, set=s)`` runs kernel k for the job in slot s; only the
        kernels that touch those tensors get launches of their own."""
        from .runtime import Kernels
        key = (frames, layers, parts)
        if key not in self._programs:
            buf = self.buffers(frames)
            n = self.cfg.layers if layers is None else layers
            taken = [j for j, i in enumerate(self.cfg.out_indices) if i <= n]
            sets = [[]] + [[(buf.images[0], buf.images[s])] +
                           [(buf.slot_features[0][j], buf.slot_features[s][j]) for j in taken]
                           for s in range(1, self.slots)]
            self._programs[key] = Kernels(self.specs(frames, layers, parts),
                                          sets=sets if self.slots > 1 else None)
        return self._programs[key]

    def features(self, frames: int, layers: int | None = None, slot: int = 0) -> list:
        n = self.cfg.layers if layers is None else layers
        buf = self.buffers(frames)
        return [buf.slot_features[slot][j] for j, i in enumerate(self.cfg.out_indices) if i <= n]

    def forward(self, image, frames: int = 1, stream=None, layers: int | None = None):
        """``image``: device f32 NHWC [frames][side][side][cin], copied into the
        program's image buffer. Returns the feature maps (device f32
        [frames * grid^2][dim] each) of the layers in ``out_indices`` (those
        within ``layers``)."""
        buf = self.buffers(frames)
        # the copy and the kernels run on one stream: `stream` when given
        # (made current for the copy), else the current stream
        with _on_stream(stream):
            buf.image.copy_(image)
            self.program(frames, layers).encode_all(None)
        return self.features(frames, layers)

    def capture_host(self, frames: int, host_image, host_features: list, stream=None):
        """One CUDA graph of a whole host-to-host pass over `frames` frames:
        the pinned ``host_image`` (f32 NHWC) copied in, the encoder program,
        and each feature map copied out to its pinned ``host_features[j]`` on
        a second stream as soon as its LayerNorm has run, so the copies of
        the early features overlap the later blocks. Returns the
        ``torch.cuda.CUDAGraph``; ``replay()`` on a stream runs one pass."""
        import torch
        prog = self.program(frames)
        buf = self.buffers(frames)
        cuts = [i + 1 for i in range(len(prog)) if prog.label(i).startswith("features.")]
        feats = self.features(frames)
        if len(host_features) != len(feats):
            raise ValueError("%d host feature buffers for %d feature maps"
                             % (len(host_features), len(feats)))
        side = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            s = torch.cuda.current_stream()
            buf.image.copy_(host_image, non_blocking=True)
            begin = 0
            for j, end in enumerate(cuts):
                prog.encode_all(s, begin=begin, end=end)
                ready = torch.cuda.Event()
                ready.record(s)
                side.wait_event(ready)
                with torch.cuda.stream(side):
                    host_features[j].copy_(feats[j], non_blocking=True)
                begin = end
            if begin < len(prog):
                prog.encode_all(s, begin=begin)
            s.wait_stream(side)
        return g

    def launches_per_frame_batch(self, layers: int | None = None, frames: int = 1) -> int:
        n = self.cfg.layers if layers is None else layers
        taken = sum(1 for i in self.cfg.out_indices if i <= n)
        fused = self._fused(frames)
        per_block = [7 if not fused else (6 if i == 0 else 5) for i in range(n)]
        return 3 + sum(per_block) + taken  # patchify (2 kernels) + patch GEMM, blocks, norms


# ------------------------------------------------------------------ DPT head

@dataclasses.dataclass
class DecoderConfig:
    """The DPT head of Depth-Anything-V2-Small (load/depth_anything_v2.rs
    Config::small): per-stage widths and resampling ("up", f) / ("keep",) /
    ("down", f), the fusion width and the head width."""
    neck: tuple = (48, 96, 192, 384)
    reassemble: tuple = (("up", 4), ("up", 2), ("keep",), ("down", 2))
    fusion: int = 64
    head: int = 32


def decoder_weights_random(cfg: ViTConfig, dcfg: DecoderConfig, seed: int = 0) -> dict:
    """Random DPT-head weights by role, HWIO convolutions: N(0, 1/sqrt(fan_in))
    weights and N(0, 0.02) biases."""
    rng = np.random.default_rng(seed)
    w = lambda *s: (rng.standard_normal(s) / math.sqrt(np.prod(s[:-1]))).astype(np.float32)
    b = lambda n: (rng.standard_normal(n) * 0.02).astype(np.float32)
    F = dcfg.fusion
    out = {"stages": [], "fusion": [], "head": {}}
    for c, rs in zip(dcfg.neck, dcfg.reassemble):
        st = {"proj_w": w(1, 1, cfg.dim, c), "proj_b": b(c), "neck_w": w(3, 3, c, F)}
        if rs[0] == "up":
            st["resize_w"], st["resize_b"] = w(rs[1], rs[1], c, c), b(c)
        elif rs[0] == "down":
            st["resize_w"], st["resize_b"] = w(3, 3, c, c), b(c)
        out["stages"].append(st)
    for _ in dcfg.neck:
        unit = lambda: {"w1": w(3, 3, F, F), "b1": b(F), "w2": w(3, 3, F, F), "b2": b(F)}
        out["fusion"].append({"unit1": unit(), "unit2": unit(), "proj_w": w(1, 1, F, F),
                              "proj_b": b(F)})
    out["head"] = {"w1": w(3, 3, F, F // 2), "b1": b(F // 2), "w2": w(3, 3, F // 2, dcfg.head),
                   "b2": b(dcfg.head), "w3": w(1, 1, dcfg.head, 1), "b3": b(1)}
    return out


class Decoder:
    """The DPT head on NHWC f32 maps (model/depth_anything_v2.rs:680-982): per
    stage a 1x1 reassembly convolution and its resampling, a 3x3 convolution
    without bias to the fusion width; fusion layers deepest first (residual
    units x + conv2(relu(conv1(relu(x)))), bilinear resampling with corners
    aligned to the next stage's size, or twice its own after the last, and a
    1x1 projection); the head (3x3 to F/2, resampling to the input's side, 3x3
    to the head width with ReLU, 1x1 to one channel with ReLU). Convolutions
    run as im2col + tcgen05 GEMM (``ops.conv2d``)."""

    def __init__(self, cfg: ViTConfig, dcfg: DecoderConfig, weights: dict, device="cuda"):
        import torch
        self.cfg, self.dcfg = cfg, dcfg
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device)
        F = dcfg.fusion
        self.stages = []
        for c, rs, w in zip(dcfg.neck, dcfg.reassemble, weights["stages"]):
            st = {"proj": (ops.conv_weights(w["proj_w"], 1, cfg.dim, c), dev(w["proj_b"])),
                  "neck": ops.conv_weights(w["neck_w"], 3, c, F), "resample": rs, "c": c}
            if rs[0] == "down":
                st["resize"] = (ops.conv_weights(w["resize_w"], 3, c, c), dev(w["resize_b"]))
            elif rs[0] == "up":
                st["resize"] = (ops.conv_transpose_weights(w["resize_w"], c, c, rs[1],
                                                           device=device), dev(w["resize_b"]))
            self.stages.append(st)
        unit = lambda u: (ops.conv_weights(u["w1"], 3, F, F), dev(u["b1"]),
                          ops.conv_weights(u["w2"], 3, F, F), dev(u["b2"]))
        self.fusion = [{"unit1": unit(f["unit1"]), "unit2": unit(f["unit2"]),
                        "proj": (ops.conv_weights(f["proj_w"], 1, F, F), dev(f["proj_b"]))}
                       for f in weights["fusion"]]
        h = weights["head"]
        self.head = {"c1": (ops.conv_weights(h["w1"], 3, F, F // 2), dev(h["b1"])),
                     "c2": (ops.conv_weights(h["w2"], 3, F // 2, dcfg.head), dev(h["b2"])),
                     "c3": (ops.conv_weights(h["w3"], 1, dcfg.head, 1), dev(h["b3"]))}

    def _unit(self, x, u, side, residual=None):
        F = self.dcfg.fusion
        first = ops.conv2d(x, u[0], u[1], side, side, F, F, relu_input=True)
        return ops.conv2d(first, u[2], u[3], side, side, F, F, relu_input=True,
                          residual=x if residual is None else residual)

    def forward(self, features: list, stream=None):
        """``features``: the encoder's feature maps, [grid^2][dim] f32 each,
        shallowest first. Returns the relative depth, [side][side] f32 (side =
        grid * patch). Every kernel and temporary of the head runs on
        ``stream`` when given (it is made current for the whole pass), else
        on the current stream."""
        with _on_stream(stream):
            return self._forward(features)

    def _forward(self, features: list):
        stream = None  # the current stream, for every op
        cfg, F = self.cfg, self.dcfg.fusion
        g = cfg.grid
        maps = []
        for feat, st in zip(features, self.stages):
            c = st["c"]
            x = ops.conv2d(feat, st["proj"][0], st["proj"][1], g, g, cfg.dim, c, ksize=1)
            side = g
            kind = st["resample"]
            if kind[0] == "up":
                x = ops.conv_transpose(x, st["resize"][0], st["resize"][1], g, g, c, c, kind[1])
                side = g * kind[1]
            elif kind[0] == "down":
                x = ops.conv2d(x, st["resize"][0], st["resize"][1], g, g, c, c, stride=kind[1])
                side = (g - 1) // kind[1] + 1
            maps.append((ops.conv2d(x, st["neck"], None, side, side, c, F), side))
        fused, side = None, None
        for layer, (stage, s) in enumerate(reversed(maps)):
            nxt = len(maps) - 2 - layer
            out_side = maps[nxt][1] if nxt >= 0 else 2 * s
            f = self.fusion[layer]
            if fused is None:
                x = stage
            else:  # unit1(stage) + previous: the previous map joins the unit's residual
                x = self._unit(stage, f["unit1"], s, residual=stage + fused)
            x = self._unit(x, f["unit2"], s)
            x = ops.resize_bilinear(x, s, s, out_side, out_side, F, stream)
            fused = ops.conv2d(x, f["proj"][0], f["proj"][1], out_side, out_side, F, F, ksize=1)
            side = out_side
        out_side = g * cfg.patch
        h = self.head
        x = ops.conv2d(fused, h["c1"][0], h["c1"][1], side, side, F, F // 2)
        x = ops.resize_bilinear(x, side, side, out_side, out_side, F // 2, stream)
        x = ops.conv2d(x, h["c2"][0], h["c2"][1], out_side, out_side, F // 2, self.dcfg.head,
                       act="relu")
        x = ops.conv2d(x, h["c3"][0], h["c3"][1], out_side, out_side, self.dcfg.head, 1,
                       ksize=1, act="relu")
        return x.reshape(out_side, out_side)

    def capture(self, features: list, stream):
        """The head as one CUDA graph on the non-default ``stream``: every
        launch's host-side preparation (tensor maps, arguments) and every
        temporary is made once, at capture; ``replay()`` reruns the kernels
        on whatever ``features`` then hold. Returns (graph, depth tensor)."""
        import torch
        with torch.cuda.stream(stream):
            self.forward(features)  # first use: allocator pools, kernel attributes
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            depth = self.forward(features)
        return g, depth
