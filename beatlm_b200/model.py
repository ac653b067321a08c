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

    @staticmethod
    def lifetime(name: str, used: list) -> tuple[int, int]:
        """A buffer's lifetime in launch order, from the launches that bind
        it (``used``: the buffer names of each launch; the reference's rule
        that lifetimes come from the kernels, kernel.rs:67-79). Images and
        feature maps are the program's inputs and outputs, written and read
        by the host between passes, so they live for the whole program, as
        does a buffer no launch binds."""
        last = len(used) - 1
        if name.startswith("image") or name.startswith("features"):
            return 0, last
        hits = [i for i, names in enumerate(used) if name in names]
        return (hits[0], hits[-1]) if hits else (0, last)


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


def norm_epilogue_fits(rows: int, dim: int, sms: int | None = None) -> bool:
    """Whether a GEMM writing `rows` x `dim` can carry the epilogue LayerNorm:
    every 32-column tile must be resident at once, one per SM (`sms`: the
    device's count, queried when not given)."""
    if sms is None:
        import torch
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return dim <= 512 and -(-rows // 128) * (dim // 32) <= sms


# ------------------------------------------------------------------ graphs
# The reference's graph builders (crates/beatlm/src/model/depth_anything_v2.rs:
# block / layer_of 252-427, encoder 435-545) over graph.py's operations; the
# program the device runs is what graph.Graph.lower makes of them.

BLOCK_ACTS = ("n1", "qkv", "scores", "scaled", "probs", "values", "proj", "ls1x", "x1",
              "n2", "hidden", "act", "out", "ls2x")


def add_block(g, cfg: ViTConfig, x: int, base: int, name: str, out: int,
              out_role: str = "activation") -> dict:
    """One pre-norm block (reference.rs:520-544) on residual stream `x`,
    writing `out`; weights at ids base + i in BLOCK_NAMES order, activations
    at base + 20 + i in BLOCK_ACTS order. Returns the ids by name."""
    from . import graph as G
    t, d, m, h, hd = cfg.tokens, cfg.dim, cfg.mlp, cfg.heads, cfg.head_dim
    sizes = {"norm1_g": d, "norm1_b": d, "qkv_w": d * 3 * d, "qkv_b": 3 * d, "proj_w": d * d,
             "proj_b": d, "ls1": d, "norm2_g": d, "norm2_b": d, "fc1_w": d * m, "fc1_b": m,
             "fc2_w": m * d, "fc2_b": d, "ls2": d}
    ids = {k: g.tensor(base + i, G.WEIGHT, sizes[k]) for i, k in enumerate(BLOCK_NAMES)}
    act_sizes = {"n1": t * d, "qkv": t * 3 * d, "scores": t * h * t, "scaled": t * h * t,
                 "probs": t * h * t, "values": t * d, "proj": t * d, "ls1x": t * d, "x1": t * d,
                 "n2": t * d, "hidden": t * m, "act": t * m, "out": t * d, "ls2x": t * d}
    for i, k in enumerate(BLOCK_ACTS):
        ids[k] = g.tensor(base + 20 + i, G.ACTIVATION, act_sizes[k])
    g.tensor(out, out_role, t * d)
    ids["x"], ids["y"] = x, out
    ln = lambda inp, gm, bt: G.LayerNorm(inp, gm, bt, t, d, cfg.eps)
    g.op(ln(x, ids["norm1_g"], ids["norm1_b"]), ids["n1"], name + "norm1")
    g.op(G.MatMul(ids["n1"], ids["qkv_w"], ids["qkv_b"], t, d, 3 * d), ids["qkv"], name + "qkv")
    g.op(G.AttentionScores(ids["qkv"], t, h, hd), ids["scores"], name + "attention")
    g.op(G.Scale(ids["scores"], 1.0 / math.sqrt(hd), t * h * t), ids["scaled"], name + "scale")
    g.op(G.Softmax(ids["scaled"], t * h, t), ids["probs"], name + "softmax")
    g.op(G.AttentionValues(ids["probs"], ids["qkv"], t, h, hd), ids["values"], name + "values")
    g.op(G.MatMul(ids["values"], ids["proj_w"], ids["proj_b"], t, d, d), ids["proj"],
         name + "proj")
    g.op(G.ChannelScale(ids["proj"], ids["ls1"], t, d), ids["ls1x"], name + "ls1")
    g.op(G.Add(ids["ls1x"], x, t * d), ids["x1"], name + "residual1")
    g.op(ln(ids["x1"], ids["norm2_g"], ids["norm2_b"]), ids["n2"], name + "norm2")
    g.op(G.MatMul(ids["n2"], ids["fc1_w"], ids["fc1_b"], t, d, m), ids["hidden"], name + "fc1")
    g.op(G.GeluErf(ids["hidden"], t * m), ids["act"], name + "gelu")
    g.op(G.MatMul(ids["act"], ids["fc2_w"], ids["fc2_b"], t, m, d), ids["out"], name + "fc2")
    g.op(G.ChannelScale(ids["out"], ids["ls2"], t, d), ids["ls2x"], name + "ls2")
    g.op(G.Add(ids["x1"], ids["ls2x"], t * d), out, name + "residual2")
    return ids


def block_graph(cfg: ViTConfig):
    """One block as a graph of its own: input x (id 0), output y (id 1)."""
    from . import graph as G
    g = G.Graph()
    g.tensor(0, G.INPUT, cfg.tokens * cfg.dim)
    ids = add_block(g, cfg, 0, 100, "block0.", 1, G.OUTPUT)
    return g, [ids]


def encoder_graph(cfg: ViTConfig, layers: int | None = None):
    """The encoder (depth_anything_v2.rs:435-545): PatchEmbed, the class
    token, the position Add, the blocks, and after each block of
    out_indices the final LayerNorm and TokensToMap (a graph output). Ids:
    image 1, patch weights 2/3, class token 4, positions 5, final norm 6/7,
    embedding activations 10-12, block i at 1000 (i + 1), features 90000 + j
    (normalised rows) and 91000 + j (maps). Returns (graph, block ids,
    feature map ids)."""
    from . import graph as G
    t, d, n = cfg.tokens, cfg.dim, cfg.layers if layers is None else layers
    g = G.Graph()
    g.tensor(1, G.INPUT, cfg.side * cfg.side * cfg.cin)
    for i, sz in ((2, cfg.taps * d), (3, d), (4, d), (5, t * d), (6, d), (7, d)):
        g.tensor(i, G.WEIGHT, sz)
    for i, sz in ((10, (t - 1) * d), (11, t * d), (12, t * d)):
        g.tensor(i, G.ACTIVATION, sz)
    g.op(G.PatchEmbed(1, 2, 3, cfg.grid, cfg.grid, cfg.patch, cfg.cin, d), 10, "embed")
    g.op(G.PrependToken(4, 10, t - 1, d), 11, "embed.cls")
    g.op(G.Add(11, 5, t * d), 12, "embed.pos")
    x, blocks, maps = 12, [], []
    for i in range(n):
        base = 1000 * (i + 1)
        ids = add_block(g, cfg, x, base, "block%d." % i, base + 99)
        blocks.append(ids)
        x = ids["y"]
        if (i + 1) in cfg.out_indices:
            j = cfg.out_indices.index(i + 1)
            g.tensor(90000 + j, G.ACTIVATION, t * d)
            g.tensor(91000 + j, G.OUTPUT, (t - 1) * d)
            g.op(G.LayerNorm(x, 6, 7, t, d, cfg.eps), 90000 + j, "features.%d" % (i + 1))
            g.op(G.TokensToMap(90000 + j, t, d), 91000 + j, "features.%d.map" % (i + 1))
            maps.append(91000 + j)
    return g, blocks, maps


def lowering_forms(fused_ln, rows: int, dim: int, sms: int | None = None) -> tuple:
    """The fused forms graph.Graph.lower applies for a LayerNorm placement:
    False (standalone LayerNorms, the fastest measured at ViT-S), True
    (LayerNorm prologues fed by the previous GEMM's row statistics) or
    "epilogue" (LayerNorms as a second output of the GEMM before them, where
    every column tile fits on the device at once; otherwise as False)."""
    from .graph import B200_FORMS
    if fused_ln == "epilogue":
        return B200_FORMS + (("ln_epilogue",) if norm_epilogue_fits(rows, dim, sms) else ())
    return B200_FORMS + (("ln_prologue",) if fused_ln else ())


class _Binder:
    """Launches for a lowered program: each kernel's tensors bound to device
    buffers (``bind``: tensor id -> (buffer name, tensor)), its main
    operation, prologue and epilogue turned into the C ABI's arguments. A
    PatchEmbed kernel becomes two launches (the patch matrix with the class
    rows, then its GEMM). Records which buffers each launch binds, from which
    the memory plan's lifetimes follow (rule 1: lifetimes come from the
    kernels)."""

    def __init__(self, program, bind: dict, cfg: ViTConfig, dtype: str, frames: int,
                 extra: dict, parts: int = 1):
        self.program, self.bind, self.cfg = program, bind, cfg
        self.dtype, self.frames, self.parts, self.extra = dtype, frames, parts, extra
        # tensors a LayerNorm prologue reads: their writer adds row statistics
        self.stats_read = {k.main.a for k in program.kernels
                           if k.prologue and k.prologue[0].kind == "layernorm"}

    def t(self, tid):
        return None if tid is None else self.bind[tid][1]

    def names(self, *tids):
        return {self.bind[t][0] for t in tids if t is not None and t in self.bind}

    def specs(self) -> tuple[list, list]:
        """(specs, buffer names each spec binds)."""
        from . import graph as G
        from .runtime import Spec
        out, used = [], []
        cfg, frames = self.cfg, self.frames
        t = cfg.tokens
        for k in self.program.kernels:
            main, label = k.main, k.label
            steps = {e.kind: e for e in k.epilogue}
            if isinstance(main, G.PatchEmbed):
                cls, pos = steps["prepend_token"].tensor, steps["add"].tensor
                image, x, patches = self.t(main.input), self.t(k.output), self.extra["patches"]
                out.append(Spec(ops.patchify_args(image, frames=frames, side=cfg.side,
                                                  patch=cfg.patch, cin=cfg.cin, k_pad=cfg.k_pad,
                                                  a_out=patches, a_dtype=self.dtype,
                                                  cls=self.t(cls), pos=self.t(pos), x=x),
                                "embed.patchify"))
                used.append(self.names(main.input, cls, pos, k.output) | {"patches"})
                out.append(Spec(_weights_gemm(self.t(main.weights), a=patches,
                                              bias=self.t(main.bias), residual=self.t(pos),
                                              res_period=t, out=x, out_row_offset=1,
                                              out_group=(t - 1, 1)), "embed.patch", self.parts))
                used.append(self.names(main.weights, main.bias, pos, k.output) | {"patches"})
            elif isinstance(main, G.LayerNorm):
                kw = dict(in_row_offset=1, in_group=(t - 1, 1)) if "tokens_to_map" in steps else {}
                out.append(Spec(ops.layernorm_args(self.t(main.input), self.t(main.gamma),
                                                   self.t(main.beta), main.eps,
                                                   out=self.t(k.output), **kw),
                                label, self.parts))
                used.append(self.names(main.input, main.gamma, main.beta, k.output))
            elif isinstance(main, G.Attention):
                out.append(Spec(ops.attention_args(self.t(main.qkv), tokens=t, heads=cfg.heads,
                                                   head_dim=cfg.head_dim, batch=frames,
                                                   qk_dtype=self.dtype, out=self.t(k.output)),
                                label, self.parts))
                used.append(self.names(main.qkv, k.output))
            elif isinstance(main, G.MatMul):
                kw = {}
                names = self.names(main.b, main.bias, k.output)
                if k.prologue:
                    p = k.prologue[0]
                    kw["ln"] = (self.t(main.a), self.t(p.tensor), self.t(p.beta), p.value)
                    kw["ln_stats"] = self.extra["stats"][main.a]
                    names |= self.names(main.a, p.tensor, p.beta)
                    names |= {self.extra["stats_name"][main.a]}
                else:
                    kw["a"] = self.t(main.a)
                    names |= self.names(main.a)
                if "gelu_erf" in steps:
                    kw["act"] = "gelu_erf"
                if "channel_scale" in steps:
                    kw["chan_scale"] = self.t(steps["channel_scale"].tensor)
                    names |= self.names(steps["channel_scale"].tensor)
                if "add" in steps:
                    kw["residual"] = self.t(steps["add"].tensor)
                    names |= self.names(steps["add"].tensor)
                if "layernorm" in steps:
                    e = steps["layernorm"]
                    kw["norm"] = (self.t(e.tensor), self.t(e.beta), e.value, self.t(e.out))
                    kw["norm_sync"] = self.extra["norm_sync"]
                    names |= self.names(e.tensor, e.beta, e.out) | {"norm_sync"}
                if k.output in self.stats_read:
                    kw["stats_out"] = self.extra["stats"][k.output]
                    names |= {self.extra["stats_name"][k.output]}
                if self.bind[k.output][0] == "qkv":  # packed Q|K|V: V in f16
                    kw["out_dtype"], kw["out_split"] = self.dtype, (2 * cfg.dim, "f16")
                out.append(Spec(_weights_gemm(self.t(main.b), bias=self.t(main.bias),
                                              out=self.t(k.output), **kw), label, self.parts))
                used.append(names)
            else:
                raise ValueError("no launch for kernel %s" % k.name())
        return out, used


def _block_binding(ids: dict, blk: "DeviceBlock", buf: "Buffers") -> dict:
    """A block's tensors on the buffers: the residual stream (x, x1, y) in
    place in buf.x (each epilogue reads a residual element and writes the
    same element), both LayerNorms' rows in buf.xn, and the weights."""
    w = {"norm1_g": blk.norm1[0], "norm1_b": blk.norm1[1], "qkv_w": blk.qkv_w,
         "qkv_b": blk.qkv_b, "proj_w": blk.proj_w, "proj_b": blk.proj_b, "ls1": blk.ls1,
         "norm2_g": blk.norm2[0], "norm2_b": blk.norm2[1], "fc1_w": blk.fc1_w,
         "fc1_b": blk.fc1_b, "fc2_w": blk.fc2_w, "fc2_b": blk.fc2_b, "ls2": blk.ls2}
    bind = {ids[k]: ("weight", v) for k, v in w.items()}
    for k, name in (("x", "x"), ("x1", "x"), ("y", "x"), ("n1", "xn"), ("n2", "xn"),
                    ("qkv", "qkv"), ("values", "o"), ("act", "h")):
        bind[ids[k]] = (name, getattr(buf, name))
    return bind


def _stats(blocks: list, buf: "Buffers") -> tuple[dict, dict]:
    """Row-statistics buffers of the residual stream's tensors: stats2 for
    each block's x1, stats1 for the stream between blocks."""
    stats, names = {}, {}
    for ids in blocks:
        for k, sb in (("x", "stats1"), ("y", "stats1"), ("x1", "stats2")):
            stats[ids[k]], names[ids[k]] = getattr(buf, sb), sb
    return stats, names


def block_specs(blk: DeviceBlock, cfg: ViTConfig, buf: Buffers, layer: int = 0,
                parts: int = 1, fused_ln=False, sms: int | None = None) -> list:
    """The kernels of one pre-norm block (reference.rs:520-544) in place on
    ``buf.x``, as graph.Graph.lower makes them of the block's graph:
    x1 = x + ls1 * proj(attention(norm1(x))); x = x1 + ls2 * fc2(gelu(fc1(norm2(x1)))).

    ``fused_ln`` (``lowering_forms``): False gives 7 kernels (each LayerNorm
    a kernel of its own writing 16-bit rows the next GEMM loads by TMA);
    True and "epilogue" fold norm2 into the GEMM after it (a prologue fed by
    the out-projection's row statistics) or before it (a second output of
    the out-projection): 6 kernels. The block's input is the graph's input,
    written by no kernel, so norm1 stays a kernel of its own either way."""
    from .graph import Fusion
    g, blocks = block_graph(cfg)
    forms = lowering_forms(fused_ln, buf.rows, cfg.dim, sms)
    prog = g.lower(Fusion.ON, forms)
    for k in prog.kernels:
        k.label = k.label.replace("block0.", "block%d." % layer)
    stats, stats_name = _stats(blocks, buf)
    extra = {"stats": stats, "stats_name": stats_name, "norm_sync": buf.norm_sync}
    specs, _ = _Binder(prog, _block_binding(blocks[0], blk, buf), cfg, blk.dtype, buf.frames,
                       extra, parts).specs()
    return specs


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
                 slots: int = 1, sms: int | None = None):
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
        and set s reads slot s's image and writes its feature maps.

        ``sms``: the device's SM count for the fusion decisions that depend
        on it (queried from the current device when not given)."""
        import torch
        td = torch.bfloat16 if dtype == "bf16" else torch.float16
        self.cfg, self.dtype = cfg, dtype
        self._sms, self._device = sms, device
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
        acts = []
        meta = Buffers(self.cfg, frames, self.dtype, device="meta", slots=self.slots,
                       alloc=lambda n, s, dt: acts.append((n, s, dt)) or torch.empty(
                           s, dtype=dt, device="meta"))
        _, used = self._launches(frames, None, 1, 0, meta)
        last = len(used) - 1
        wts = self._weights()
        descs = []
        for k, (o, a, i) in enumerate(wts):
            t = getattr(o, a) if i is None else getattr(o, a)[i]
            descs.append(TensorDesc(k, F32 if t.element_size() == 4 else F16, t.numel(), 0, last))
        for k, (name, shape, dt) in enumerate(acts, start=len(wts)):
            first, end = Buffers.lifetime(name, used)
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

    def lowered(self, frames: int, layers: int | None = None):
        """The encoder graph (``encoder_graph``) lowered with this encoder's
        LayerNorm placement for `frames` frames: (program, block ids, feature
        map ids). No device work."""
        from .graph import Fusion
        g, blocks, maps = encoder_graph(self.cfg, layers)
        forms = lowering_forms(self.fused_ln, frames * self.cfg.tokens, self.cfg.dim, self._sms)
        return g.lower(Fusion.ON, forms), blocks, maps

    def specs_layout(self, frames: int) -> list:
        """The spec labels of the encoder program, in order (no device work):
        a PatchEmbed kernel is two launches, every other kernel one."""
        from .graph import PatchEmbed
        prog, _, _ = self.lowered(frames)
        out = []
        for k in prog.kernels:
            out += (["embed.patchify", "embed.patch"] if isinstance(k.main, PatchEmbed)
                    else [k.label])
        return out

    def _launches(self, frames: int, layers, parts: int, slot: int, buf: Buffers):
        """(specs, buffer names each spec binds) of the lowered encoder over
        `buf`, reading slot `slot`'s image and writing its feature maps."""
        prog, blocks, maps = self.lowered(frames, layers)
        if not 0 <= slot < self.slots:
            raise ValueError("slot %d of %d" % (slot, self.slots))
        bind = {1: ("image", buf.images[slot]), 2: ("weight", self.patch_w),
                3: ("weight", self.patch_b), 4: ("weight", self.cls), 5: ("weight", self.pos),
                6: ("weight", self.norm[0]), 7: ("weight", self.norm[1]), 12: ("x", buf.x)}
        for i, ids in enumerate(blocks):
            bind.update(_block_binding(ids, self.blocks[i], buf))
        for j, m in enumerate(maps):
            bind[m] = ("features.%d" % self.cfg.out_indices[j], buf.slot_features[slot][j])
        stats, stats_name = _stats(blocks, buf)
        extra = {"patches": buf.patches, "stats": stats, "stats_name": stats_name,
                 "norm_sync": buf.norm_sync}
        return _Binder(prog, bind, self.cfg, self.dtype, frames, extra, parts).specs()

    def buffers(self, frames: int) -> Buffers:
        if frames not in self._buffers:
            if self.arena is not None:
                raise ValueError("this encoder's memory is planned for %s frames"
                                 % sorted(self._buffers))
            self._buffers[frames] = Buffers(self.cfg, frames, self.dtype, slots=self.slots,
                                            device=self._device)
        return self._buffers[frames]

    def specs(self, frames: int, layers: int | None = None, parts: int = 1,
              slot: int = 0) -> list:
        """The encoder as kernel specs over the buffers of `frames` frames,
        reading slot `slot`'s image and writing its feature maps: the
        launches of the lowered encoder graph (``lowered``)."""
        return self._launches(frames, layers, parts, slot, self.buffers(frames))[0]

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

    def capture(self, frames: int, stream, slot: int = 0, host_features: list | None = None,
                host_image=None):
        """One CUDA graph of the encoder over `frames` frames in slot ``slot``
        (its binding set), with each feature-map LayerNorm on a second stream:
        it forks after the block whose output it reads and joins before the
        next kernel that writes the residual stream (the next block's
        out-projection), so it leaves the chain of dependent launches. With
        ``host_features`` each map is also copied out to its pinned buffer on
        that stream right after its LayerNorm; with ``host_image`` the pinned
        image is first copied into the slot. Returns the
        ``torch.cuda.CUDAGraph``; ``replay()`` on the current stream runs
        one pass."""
        import torch
        prog = self.program(frames)
        buf = self.buffers(frames)
        n = len(prog)
        base = [prog.label(i).split(" ")[0] for i in range(n)]
        feats = self.features(frames, slot=slot)
        fidx = [i for i in range(n) if base[i].startswith("features.")]
        if host_features is not None and len(host_features) != len(feats):
            raise ValueError("%d host feature buffers for %d feature maps"
                             % (len(host_features), len(feats)))
        # the residual stream's next writer after each feature LayerNorm
        writes_x = [i for i in range(n) if base[i].endswith(".proj") or base[i].endswith(".fc2")
                    or base[i] == "embed.patch"]
        joins = {}
        for j, f in enumerate(fidx):
            nxt = [i for i in writes_x if i > f]
            joins.setdefault(nxt[0] if nxt else n, []).append(j)
        side = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            s = torch.cuda.current_stream()
            if host_image is not None:
                buf.images[slot].copy_(host_image, non_blocking=True)
            done = {}
            begin = 0
            for i in range(n + 1):
                if i in joins or i in fidx or i == n:
                    if begin < i:
                        prog.encode_all(s, begin=begin, end=i, set=slot)
                    begin = i
                for j in joins.get(i, []):
                    s.wait_event(done[j])
                if i < n and i in fidx:
                    j = fidx.index(i)
                    fork = torch.cuda.Event()
                    fork.record(s)
                    side.wait_event(fork)
                    prog.encode(i, side, set=slot)
                    # the join waits for the LayerNorm, not for its copy out
                    done[j] = torch.cuda.Event()
                    done[j].record(side)
                    if host_features is not None:
                        with torch.cuda.stream(side):
                            host_features[j].copy_(feats[j], non_blocking=True)
                    begin = i + 1
            s.wait_stream(side)
        return g

    def capture_host(self, frames: int, host_image, host_features: list, stream=None,
                     slot: int = 0):
        """One CUDA graph of a whole host-to-host pass over `frames` frames:
        the pinned ``host_image`` (f32 NHWC) copied in (None: the slot's image
        is already on the device), the encoder over slot ``slot``, and each
        feature map copied out to its pinned ``host_features[j]`` right after
        its LayerNorm, both on a second stream beside the later blocks
        (``capture``). ``replay()`` on a stream runs one pass."""
        return self.capture(frames, stream, slot=slot, host_features=host_features,
                            host_image=host_image)

    def host_pipeline(self, frames: int, host_images: list, host_features: list):
        """Frames host to host with each frame's image copy overlapping the
        previous frame's pass (``HostPipeline``): needs ``slots >= 2``;
        ``host_images[s]`` (pinned f32 NHWC) and ``host_features[s]`` (pinned,
        one per feature map) are slot s's host buffers."""
        return HostPipeline(self, frames, host_images, host_features)

    def launches_per_frame_batch(self, layers: int | None = None, frames: int = 1) -> int:
        """Kernels launched per pass: the program's specs, with the patch
        embedding counted as two (the patch matrix, whose launch also writes
        the class-token rows, and its GEMM)."""
        from .graph import PatchEmbed
        prog, _, _ = self.lowered(frames, layers)
        return sum(2 if isinstance(k.main, PatchEmbed) else 1 for k in prog.kernels)


class HostPipeline:
    """Frames from pinned host memory to pinned host memory over two input/
    output slots (the reference keeps jobs in flight through its Net slots,
    crates/beatlm-host/src/slots.rs:1-60): frame k runs in slot k % 2 as one
    ``Encoder.capture_host`` graph of that slot (the encoder, each feature map
    copied out right after its LayerNorm), and its image reaches that slot's
    device buffer through ``runtime.InputPipeline``: copied at the start of
    frame k - 1, beside that frame's pass, once frame k - 2 (which read the
    slot) has finished. So a frame's image copy leaves the critical path; its
    feature copies stay inside its own pass. ``step(stream, fill)`` runs the
    next frame on ``stream`` and returns its slot; ``fill(slot)`` (optional)
    writes the next frame's pixels into ``host_images[slot]`` before its copy
    is issued."""

    def __init__(self, enc: "Encoder", frames: int, host_images: list, host_features: list):
        from .runtime import InputPipeline
        if enc.slots < 2:
            raise ValueError("a host pipeline needs an encoder with two slots (slots=2)")
        if len(host_images) < 2 or len(host_features) < 2:
            raise ValueError("host buffers for two slots")
        self.enc, self.frames = enc, frames
        self.host_features = host_features
        self.inputs = InputPipeline(list(host_images[:2]), enc.buffers(frames).images[:2])
        self.graphs = {}

    def step(self, stream, fill=None):
        import torch
        s = self.inputs.slot()
        if s not in self.graphs:
            self.graphs[s] = self.enc.capture_host(self.frames, None, self.host_features[s],
                                                   stream, slot=s)
        self.inputs.acquire(stream, fill)
        with torch.cuda.stream(stream):
            self.graphs[s].replay()
        self.inputs.release(stream)
        return s


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


def _dt_name(weights) -> str:
    """The 16-bit operand type of a convolution's weights, by name."""
    import torch
    return "f16" if weights.dtype == torch.float16 else "bf16"


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

        def padded(b, wts):
            # a bias zero-padded to the weights' padded output channels, so
            # the convolution reads it in place (no per-call padding)
            out = np.zeros(wts.shape[0], np.float32)
            out[:len(b)] = np.asarray(b, np.float32).reshape(-1)
            return dev(out)
        F = dcfg.fusion
        self.stages = []
        for c, rs, w in zip(dcfg.neck, dcfg.reassemble, weights["stages"]):
            pw = ops.conv_weights(w["proj_w"], 1, cfg.dim, c)
            st = {"proj": (pw, padded(w["proj_b"], pw)),
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
        # the last convolution (head width -> 1 channel, 1x1) as a per-pixel
        # dot product in f32 in the epilogue of the one before: its weights
        # as a vector
        self.head = {"c1": (ops.conv_weights(h["w1"], 3, F, F // 2), dev(h["b1"])),
                     "c2": (ops.conv_weights(h["w2"], 3, F // 2, dcfg.head), dev(h["b2"])),
                     "c3": (dev(np.asarray(h["w3"], np.float32).reshape(dcfg.head)),
                            float(np.asarray(h["b3"], np.float32).reshape(-1)[0]))}

    def launches_per_frame(self) -> int:
        """The kernels one ``forward`` launches: a convolution is a gather and
        a GEMM, except a 1x1 one of 16-bit GEMM rows (the GEMM alone); a
        transposed convolution adds its block scatter; a resampling is one
        launch; the last 1x1 convolution to one channel runs in the epilogue
        of the convolution before it."""
        n = 0
        for st in self.stages:
            n += 2 + 2  # the projection and the neck convolution
            kind = st["resample"][0]
            if kind == "up":
                # the projection's padded 16-bit output is the GEMM's rows
                # when its width is cin rounded up to 64 (see _forward)
                rows = st["proj"][0].shape[0] == -(-st["c"] // 64) * 64
                n += 2 if rows else 3
            elif kind == "down":
                n += 2
        for layer in range(len(self.fusion)):
            # one residual unit in the deepest layer, two after it; the
            # resampling writes the projection's rows
            n += (4 if layer == 0 else 8) + 1 + 1
        return n + 2 + 1 + 2  # head: 3x3, resampling, 3x3 with the 1x1 to one channel

    def _unit(self, x, u, side, residual=None):
        F = self.dcfg.fusion
        # the first convolution's only reader is the second one's gather: its
        # map is stored in the operands' 16 bits (the one rounding the gather
        # of an f32 map would make), half the bytes written and read
        first = ops.conv2d(x, u[0], u[1], side, side, F, F, relu_input=True,
                           out_dtype=_dt_name(u[0]))
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
            # the reassembly projection's only reader is the next gather or
            # GEMM: its map in the operands' 16 bits, with the padded output
            # channels (zeros), which at 48 channels are the transposed
            # convolution's GEMM rows (no narrowing copy, no gather)
            dt = _dt_name(st["proj"][0])
            x = ops.conv2d(feat, st["proj"][0], st["proj"][1], g, g, cfg.dim, c, ksize=1,
                           out_dtype=dt, padded=True)
            side = g
            kind = st["resample"]
            if kind[0] == "up":
                x = ops.conv_transpose(x, st["resize"][0], st["resize"][1], g, g, c, c, kind[1],
                                       dtype=dt)
                side = g * kind[1]
            elif kind[0] == "down":
                x = ops.conv2d(x, st["resize"][0], st["resize"][1], g, g, c, c, stride=kind[1],
                               out_dtype=dt)
                side = (g - 1) // kind[1] + 1
            maps.append((ops.conv2d(x, st["neck"], None, side, side, c, F), side))
        fused, side = None, None
        for layer, (stage, s) in enumerate(reversed(maps)):
            nxt = len(maps) - 2 - layer
            out_side = maps[nxt][1] if nxt >= 0 else 2 * s
            f = self.fusion[layer]
            if fused is None:
                x = stage
            else:  # unit1(stage) + previous: `fused` already holds stage + previous
                x = self._unit(stage, f["unit1"], s, residual=fused)
            x = self._unit(x, f["unit2"], s)
            # the resampling writes the projection's 16-bit GEMM rows itself
            # (the same values a gather of its f32 output would store), and
            # the projection's epilogue adds the next layer's stage map (the
            # residual of that layer's first unit): the same arithmetic as
            # separate passes, two launches fewer
            pw = f["proj"][0]
            x = ops.resize_bilinear_rows16(x, s, s, out_side, out_side, F, pw.shape[1],
                                           _dt_name(pw), stream)
            # the last layer's map feeds only the head's first convolution:
            # 16 bits, as for a unit's first convolution
            fused = ops.conv2d(x, pw, f["proj"][1], out_side, out_side, F, F, ksize=1,
                               residual=maps[nxt][0] if nxt >= 0 else None,
                               out_dtype="f32" if nxt >= 0 else _dt_name(pw))
            side = out_side
        out_side = g * cfg.patch
        h = self.head
        x = ops.conv2d(fused, h["c1"][0], h["c1"][1], side, side, F, F // 2)
        # the resampling to full size stored in 16 bits, gathered as it is by
        # the next convolution (the same bits as an f32 map gathered)
        x = ops.resize_bilinear_rows16(x, side, side, out_side, out_side, F // 2, F // 2,
                                       _dt_name(h["c2"][0]), stream)
        # the last 1x1 convolution to one channel (with its ReLU) in this
        # convolution's epilogue: each pixel's head-width values are one
        # accumulator row of one tile, reduced there, and the full-size map
        # of head-width channels never reaches memory
        x = ops.conv2d(x, h["c2"][0], h["c2"][1], out_side, out_side, F // 2, self.dcfg.head,
                       act="relu", dot=(h["c3"][0], h["c3"][1], True))
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
