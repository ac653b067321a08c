#!/usr/bin/env python
"""Benchmark of the ViT attention hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload encoder|attention|block|vitl_block|vitl|hires|
                                decoder|depth]
                    [--no-extra] [--no-cpu-baseline]

Workloads (synthetic data, seeded):
  encoder    config 3 (default): the DA-V2-Small ViT-S/14 encoder at 518 px,
             one frame per step through a CUDA graph; frames/s.
  attention  config 1: one ViT-S self-attention op, batch 1, 6 heads x 64,
             1370 tokens, Q/K/V ~ N(0,1), scale 1/8; f16 Q/K/V, f32 output.
  block      config 2: one pre-LN ViT-S block (dim 384, 6 heads, MLP 1536,
             1370 tokens) in f16, one CUDA graph per step; TFLOP/s.
  vitl       config 4: the ViT-L/14 encoder, one independent stream per GPU.
  hires      config 5: T=5477 attention, 16 heads split over the GPUs; each
             rank's attention kernel stores its heads' rows straight into
             every rank's [T][1024] output over NVLink (peer stores, no
             separate collective); TFLOP/s of the whole op.

With the default workload the line also carries, under "configs", the other
configs measured in the same run (configs 1, 2, 4 and 5 on one GPU; 4 and 5
on several), each with its own roofline, parity against the oracle and, on
one GPU, CPU baseline. A step is one pass of the hot path over one batch.
`value` is whole-job throughput (all ranks) with the inputs resident in HBM;
L2 is flushed (a 256 MiB write) before every timed step and the flush is
outside the timed events. `e2e` is the same metric through the public call
with host buffers: the H2D copy of the step's inputs from pinned memory and
the D2H copy of its result are inside its timed region. Multi-GPU: one
process per GPU (torchrun); configs 1-4 run independent replicas or streams
(weak scaling), config 5 splits one op by heads (strong scaling); times are
the max over ranks.

`--impl reference` times the reference's CPU path (the C restatement of its
f64 interpreter, oracle/, all host threads) on the same workload, rank 0 only:
for the encoder every step is one whole frame, evaluated op by op as the
reference's `run` evaluates the encoder graph. The `cpu_baseline` leg of our
own line times the same function on the same inputs (median of 3 frames).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ViT attention TFLOP/s (% of B200 bf16 peak); DA-V2-S 518² encoder frames/s"
IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def profiled_traffic(name):
    """DRAM bytes read + written per launch of the dominant kernel, from the
    one ncu capture summarised in profiles/<name> (its
    `traffic_bytes_per_launch:` line), or None without one."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":", 1)[1])
    except OSError:
        pass
    return None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.summary = {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return
        sm = sorted(float(r[1]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if r[5 + i].strip().lower() == "active"})
        self.summary = {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": float(rows[0][2]),
                        "reasons": reasons, "samples": len(rows)}


def _rel(got, want):
    import numpy as np
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    return (float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)),
            float(np.max(np.abs(got - want))))


def _median_time(fn, repeats):
    """Median wall time of `repeats` calls of fn (after none: the oracle's
    thread pool and pages are warmed by the first repeat's own start), and
    the last call's result."""
    times, out = [], None
    for _ in range(repeats):
        t0 = time.perf_counter()
        out = fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), times, out


# ------------------------------------------------------------------ workloads

class AttentionWorkload:
    """Config 1: one ViT-S attention op (T=1370, H=6, hd=64), batch 1."""

    name = "attention"
    unit = "TFLOP/s"
    dtype = "f16 Q/K/V and P; f32 scores, softmax and accumulator"
    data = "synthetic Q/K/V ~ N(0,1), seeded"
    workload_name = "vit_s_attention_op (config 1)"
    scaling = "weak"
    T, H = 1370, 6

    def parallelism(self, world):
        return "replicas x%d (no collective)" % world

    def roofline(self, stream, avg_ms):
        return {"achieved_tflops": self.flops / (avg_ms / 1e3) / 1e12,
                "kernel": "bl::attn::attention_fwd",
                "how": "CUDA events around every timed launch (a step is one launch)"}

    @classmethod
    def host_qkv(cls, seed=1234):
        import numpy as np
        rng = np.random.default_rng(seed)
        return rng.standard_normal((1, cls.T, 3, cls.H, 64), dtype=np.float32)

    @classmethod
    def reference_step(cls, threads):
        import oracle
        t, h = cls.T, cls.H
        qkv = oracle.round_f16(cls.host_qkv()[0].reshape(t, -1))
        rows = 32
        t0 = time.perf_counter()
        oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
        per_row = (time.perf_counter() - t0) / rows
        rows = int(max(16, min(t, 1.0 / max(per_row, 1e-9))))
        fn = lambda: oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
        return fn, 4.0 * rows * t * h * 64 / 1e12, (
            "%d of %d query rows x %d heads per step (oracle/oracle.c, f64)" % (rows, t, h))

    def __init__(self, rank: int, world: int = 1):
        import torch
        import beatlm_b200 as bl
        self.bl = bl
        self.t, self.h = self.T, self.H
        self.qkv = self.host_qkv()
        self.dev = bl.pack_qkv(self.qkv, "f16")
        self.host = self.dev.cpu().pin_memory()
        self.out = torch.empty((1, self.t, self.h * 64), dtype=torch.float32, device="cuda")
        self.out_host = torch.empty(self.out.shape, dtype=torch.float32).pin_memory()
        self.flops = 4.0 * self.t * self.t * self.h * 64
        self.launches_per_step = 1

    def config(self):
        from beatlm_b200 import ops
        qt, splits, unsplit = ops.attention_choice(
            ops.attention_args(self.dev, tokens=self.t, heads=self.h, out=self.out))
        return {"workload": self.workload_name, "batch": 1, "tokens": self.t, "heads": self.h,
                "head_dim": 64, "qkv_dtype": "f16", "out_dtype": "f32",
                "attention_launch": {"query_tiles": qt, "kv_splits": splits,
                                     "unsplit_groups": unsplit},
                "l2": "flushed before every timed launch (256 MiB write)"}

    def step(self, stream):
        self.bl.attention(self.dev, tokens=self.t, heads=self.h, out=self.out, stream=stream)

    e2e_how = ("each step: the op on this step's Q/K/V, whose host-to-device copy was issued "
               "beside the previous step's launch (runtime.InputPipeline, two device buffers) "
               "and is waited for inside the step, then its result copied to pinned host "
               "memory inside the step; L2 flushed between steps")

    def step_e2e(self, stream):
        import torch
        from beatlm_b200.runtime import InputPipeline
        if getattr(self, "inputs", None) is None:
            self.inputs = InputPipeline([self.host, self.host],
                                        [self.dev, torch.empty_like(self.dev)])
        dev = self.inputs.acquire(stream)
        self.bl.attention(dev, tokens=self.t, heads=self.h, out=self.out, stream=stream)
        self.inputs.release(stream)
        self.out_host.copy_(self.out, non_blocking=True)

    def e2e_bytes(self):
        return self.host.numel() * 2, self.out_host.numel() * 4

    def units(self):
        return self.flops / 1e12  # TFLOP per step

    def parity(self):
        """A sample of 64 query rows (all heads) against the oracle fed the
        same f16 values."""
        import oracle
        rows = (0, 32), (self.t - 32, self.t)
        ref_in = oracle.round_f16(self.qkv[0].reshape(self.t, -1))
        got = self.out_host[0].numpy()
        out = []
        for r0, r1 in rows:
            want = oracle.attention(ref_in, self.t, self.h, 64, rows=(r0, r1))
            out.append((got[r0:r1].ravel(), want))
        import numpy as np
        rel, mx = _rel(np.concatenate([g for g, _ in out]), np.concatenate([w for _, w in out]))
        return {"rel_l2": rel, "max_abs": mx, "bound": 1e-3,
                "sample": "query rows 0-31 and 1338-1369, all 6 heads, vs oracle.attention"}

    def cpu_baseline(self, threads: int, budget_s: float = 8.0):
        import oracle
        qkv = oracle.round_f16(self.qkv[0].reshape(self.t, -1))
        return oracle_attention_rate(qkv, self.t, self.h, threads, budget_s)


def oracle_attention_rate(qkv, t, h, threads, budget_s):
    """The reference's CPU path for one attention op (oracle/, a C restatement
    of reference.rs:437-494, f64 accumulation) timed on a bounded sample of
    query rows of every head, in TFLOP/s: the median of three repeats."""
    import oracle
    rows = 16
    t0 = time.perf_counter()
    oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
    dt = time.perf_counter() - t0
    rows = int(min(t, max(rows, rows * budget_s / max(dt, 1e-6) / 4)))
    med, _, _ = _median_time(lambda: oracle.attention(qkv, t, h, 64, rows=(0, rows),
                                                      threads=threads), 3)
    flops = 4.0 * rows * t * h * 64
    return {"value": flops / med / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": "%d of %d query rows x %d heads, median of 3 repeats (f64 accumulation, "
                      "oracle/oracle.c)" % (rows, t, h)}


def encoder_host_inputs(cfg, seed=99):
    """The encoder's random weights (N(0, 0.02) linear weights, biases 0,
    LayerNorm gamma 1 / beta 0, LayerScale 1) and one ImageNet-normalised
    U[0,1] frame, from one seed: the same values for the GPU run, its CPU
    baseline and the reference arm."""
    import numpy as np
    from beatlm_b200.model import block_weights_normal
    rng = np.random.default_rng(seed)
    n = lambda *s: rng.standard_normal(int(np.prod(s)), dtype=np.float32) * 0.02
    w = {"blocks": [block_weights_normal(rng, cfg.dim, cfg.mlp) for _ in range(cfg.layers)],
         "patch_w": n(cfg.patch, cfg.patch, cfg.cin, cfg.dim), "patch_b": n(cfg.dim),
         "cls": n(cfg.dim), "pos": n(cfg.tokens, cfg.dim),
         "norm_g": np.ones(cfg.dim, np.float32), "norm_b": np.zeros(cfg.dim, np.float32)}
    mean = np.array(IMAGENET_MEAN, np.float32)
    std = np.array(IMAGENET_STD, np.float32)
    img = ((rng.random((1, cfg.side, cfg.side, cfg.cin), dtype=np.float32) - mean)
           / std).astype(np.float32)
    return w, img


def oracle_frame_fn(cfg, w, img, threads, dtype="bf16"):
    """One whole encoder frame through the oracle (oracle.encoder_frame: the
    reference's interpreter over the encoder graph), fed the weights and
    pixels rounded as the device holds them."""
    import oracle
    from beatlm_b200.model import DeviceBlock
    rnd = oracle.round_bf16 if dtype == "bf16" else oracle.round_f16
    wr = dict(w, patch_w=rnd(w["patch_w"]),
              blocks=[DeviceBlock.rounded(b, dtype) for b in w["blocks"]])
    image = rnd(img[0])
    return lambda: oracle.encoder_frame(image, wr, cfg.grid, cfg.patch, cfg.cin, cfg.dim,
                                        cfg.heads, cfg.mlp, cfg.eps, cfg.out_indices,
                                        qkv_round="qk_" + dtype, threads=threads)


class EncoderWorkload:
    """Config 3: the Depth-Anything-V2-Small ViT-S/14 encoder at 518 px, 12
    blocks, bf16, random N(0, 0.02) weights (LayerNorm gamma 1 / beta 0,
    LayerScale 1), one frame per forward (batch 1), input U[0,1] normalised by
    the ImageNet mean/std. A step is one frame through a captured CUDA graph of
    the whole encoder (patch embedding, 12 blocks, the four feature
    LayerNorms)."""

    name = "encoder"
    unit = "frames/s"
    dtype = "bf16 (weights, activations, Q/K); f16 V and P; f32 accumulate and residual"
    data = "synthetic: ImageNet-normalised U[0,1] 518x518x3 image, N(0,0.02) weights, seeded"
    workload_name = "da_v2_small_encoder_518 (config 3)"
    large = False
    scaling = "weak"
    launch = "graph"  # or "direct": every kernel launched from the host each step

    @classmethod
    def vit_config(cls):
        from beatlm_b200.model import ViTConfig
        return ViTConfig.large() if cls.large else ViTConfig.small()

    def attention_marginal_us(self, stream, frames: int = 30):
        """What one attention launch costs inside the graphed frame: the frame
        graph against the same graph without its attention launches (their
        outputs then stale), each timed with CUDA events over `frames` frames,
        interleaved, L2 flushed before each; the median difference over the
        frame's attention launches."""
        import numpy as np
        import torch
        from beatlm_b200.runtime import Kernels
        specs = self.enc.specs(self.frames)
        keep = [sp for sp in specs if not sp.label.endswith(".attention")]
        cut = len(specs) - len(keep)
        if cut == 0:
            return None
        without = Kernels(keep)
        graphs = [self.prog.capture(stream), without.capture(stream)]
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        times = [[], []]
        with torch.cuda.stream(stream):
            for rep in range(frames + 3):
                for i, g in enumerate(graphs):
                    flush.zero_()
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    g.launch(stream)
                    e1.record(stream)
                    e1.synchronize()
                    if rep >= 3:
                        times[i].append(e0.elapsed_time(e1) * 1e3)
        without.close()
        return (float(np.median(times[0])) - float(np.median(times[1]))) / cut

    def roofline(self, stream, avg_ms):
        prof = self.slice_profile(stream)
        n, tot, avg_us = prof["attention"]
        steps = n / self.cfg.layers
        marginal = self.attention_marginal_us(stream)
        return {"achieved_tflops": self.attn_flops / (avg_us / 1e6) / 1e12,
                "in_frame": None if marginal is None else {
                    "us_per_launch": round(marginal, 2),
                    "tflops": round(self.attn_flops / (marginal / 1e6) / 1e12, 2),
                    "how": "the frame's CUDA graph against the same graph without its attention "
                           "launches, CUDA events, L2 flushed before each frame, medians over 30 "
                           "frames each; the difference over the launches left out"},
                "kernel": "bl::attn::attention_fwd (%d launches per frame)" % self.cfg.layers,
                "how": "cudaEvent slice timer (bl_timer) around every kernel of 5 direct "
                       "(non-graph) encodes after the timed region, each queued behind a "
                       "20 ms stream hold so the kernels run back to back",
                "traffic": (None if self.large else
                            profiled_traffic("attention_fwd_encoder_vit_s_T1370_H6.md")),
                "frame_tflops": self.flops / (avg_ms / 1e3) / 1e12,
                "kernels": {k: round(v[1] / steps, 2) for k, v in sorted(prof.items())}}

    @classmethod
    def reference_step(cls, threads):
        """ViT-S: one whole frame of the oracle per step (patch embedding, 12
        blocks, the feature LayerNorms), the same function as the cpu_baseline
        leg. ViT-L: one block per step (1/24 of a frame; a frame of the f64
        oracle takes about half a minute), scaled to a frame."""
        cfg = cls.vit_config()
        if cls.large:
            return VitLWorkload.block_step(cfg, threads)
        w, img = encoder_host_inputs(cfg)
        return oracle_frame_fn(cfg, w, img, threads), 1.0, (
            "one whole ViT-S frame per step (patch embedding, 12 blocks, 4 feature "
            "LayerNorms) through oracle.encoder_frame (reference.rs run), f64 accumulation")

    def parallelism(self, world):
        return ("%d independent streams, one per GPU, no collective" % world if world > 1
                else "1 stream")

    def __init__(self, rank: int, world: int = 1, frames: int = 1):
        import torch
        from beatlm_b200.model import Encoder
        self.cfg = cfg = self.vit_config()
        self.w, img = encoder_host_inputs(cfg, seed=99 + rank)
        self.frames = frames
        # two input/output slots: the end-to-end leg keeps a frame's image
        # copy beside the previous frame's pass (model.HostPipeline)
        self.enc = Encoder(cfg, self.w, "bf16", planned_frames=frames, slots=2)
        self.img = img
        self.host = torch.from_numpy(img).pin_memory()
        self.hosts = [self.host, torch.from_numpy(img).pin_memory()]
        self.buf = self.enc.buffers(frames)
        self.buf.image.copy_(self.host)
        self.prog = self.enc.program(frames)
        self.graph = None
        self.slot_feats_host = [[torch.empty(f.shape, dtype=f.dtype).pin_memory()
                                 for f in self.enc.features(frames)] for _ in range(2)]
        self.feats_host = self.slot_feats_host[0]
        fl = cfg.flops_per_frame()
        self.flops = fl["total"] * frames
        self.attn_flops = 4.0 * cfg.tokens * cfg.tokens * cfg.dim * frames  # per layer launch
        self.launches_per_step = self.enc.launches_per_frame_batch(frames=frames)

    def config(self):
        c = self.cfg
        return {"workload": self.workload_name,
                "frames_per_step": self.frames, "tokens": c.tokens, "dim": c.dim,
                "heads": c.heads, "mlp": c.mlp, "layers": c.layers, "image": c.side,
                "weights": "random N(0,0.02), LN gamma=1 beta=0, LayerScale=1",
                "dtype": "bf16 weights/activations, f16 V and P, f32 residual",
                "launch": ("one CUDA graph per frame (%d kernels)" if self.launch == "graph" else
                           "%d direct launches per frame") % self.launches_per_step,
                "memory": "static plan: %d tensors in one device allocation of %d bytes "
                          "(peak live %d)" % (len(self.enc.plan.placements()),
                                              self.enc.arena.bytes(),
                                              self.enc.plan.peak_live_bytes()),
                "l2": "flushed before every timed step (256 MiB write)"}

    def step(self, stream):
        if self.launch == "direct":
            self.prog.encode_all(stream)
            return
        if self.graph is None:
            # the frame's kernels, the feature LayerNorms on a second stream
            # (Encoder.capture)
            self.graph = self.enc.capture(self.frames, stream)
        self.graph.replay()

    def step_e2e(self, stream):
        # Encoder.host_pipeline: each step one frame host to host, its
        # feature maps copied out inside its pass (each right after its
        # LayerNorm) and the next frame's image copied into the other slot
        # beside it; a step waits for its own image copy
        if getattr(self, "pipe", None) is None:
            self.pipe = self.enc.host_pipeline(self.frames, self.hosts, self.slot_feats_host)
        slot = self.pipe.step(stream)
        self.feats_host = self.slot_feats_host[slot]

    e2e_how = ("each step one frame from pinned host memory to pinned host memory through "
               "Encoder.host_pipeline (two slots): its image copy, issued on a copy stream "
               "during the previous step, waited for inside the step, then its pass with each "
               "feature map copied out right after its LayerNorm; L2 flushed between steps")

    def e2e_bytes(self):
        return (self.host.numel() * 4, sum(h.numel() * 4 for h in self.feats_host))

    def units(self):
        return self.frames  # frames per step

    def slice_profile(self, stream, frames: int = 5):
        """Per-kernel durations from the cudaEvent slice timer over `frames`
        direct (non-graph) encodes: {kind: (launches, total_us, avg_us)}."""
        import torch
        from beatlm_b200.runtime import SliceTimer, hold
        t = SliceTimer(max_slices=len(self.prog))
        kinds = {}
        for f in range(frames):
            h = t.begin_frame(f)
            hold(stream, 20000)  # the frame's launches queue up behind it
            self.prog.encode_all(stream, timer=t, frame=h)
            t.submitted(h)
            torch.cuda.synchronize()
            for ft in t.collect_ready():
                for k, us in ft.compute:
                    kind = self.prog.label(k).split(".")[-1].split(" ")[0]
                    n, tot = kinds.get(kind, (0, 0.0))
                    kinds[kind] = (n + 1, tot + us)
        t.close()
        return {k: (n, tot, tot / n) for k, (n, tot) in kinds.items()}

    def cpu_baseline(self, threads: int):
        """The whole frame through the oracle on every host core, three
        frames, median: the same function `--impl reference` runs per step.
        Its feature maps are kept for the parity check."""
        fn = oracle_frame_fn(self.cfg, self.w, self.img, threads)
        med, times, self._oracle_feats = _median_time(fn, 3)
        return {"value": 1.0 / med, "unit": "frames/s", "cores": threads, "kind": "port",
                "sample": "3 whole frames (patch embedding, %d blocks, %d feature LayerNorms) "
                          "through oracle.encoder_frame (reference.rs run, f64 accumulation), "
                          "median of %s s" % (self.cfg.layers, len(self.cfg.out_indices),
                                              [round(x, 2) for x in times])}

    def parity(self):
        """The feature maps of the last e2e step (host copies) against the
        oracle frame of the cpu_baseline leg, same inputs."""
        want = getattr(self, "_oracle_feats", None)
        if want is None:
            return None
        rels = [_rel(g.numpy(), w) for g, w in zip(self.feats_host, want)]
        return {"rel_l2": max(r for r, _ in rels), "max_abs": max(m for _, m in rels),
                "per_feature_rel_l2": [r for r, _ in rels], "bound": 4e-3,
                "sample": "all 4 feature maps of the frame vs oracle.encoder_frame (bf16 block "
                          "bound, as in tests/test_block_gpu.py)"}


class VitLWorkload(EncoderWorkload):
    """Config 4: a ViT-L/14-shaped encoder (24 blocks, dim 1024, 16 heads,
    MLP 4096, 1370 tokens), bf16, random N(0, 0.02) weights. Eight
    independent input streams shard one per GPU with no collective: each rank
    runs its own stream, one frame per step."""

    name = "vitl"
    large = True
    workload_name = "vit_l14_encoder (config 4)"
    data = "synthetic: ImageNet-normalised U[0,1] 518x518x3 image per stream, N(0,0.02) weights"

    @staticmethod
    def block_step(cfg, threads):
        import numpy as np
        import oracle
        from beatlm_b200.model import block_weights_normal
        rng = np.random.default_rng(5)
        w = block_weights_normal(rng, cfg.dim, cfg.mlp)
        x = rng.standard_normal(cfg.tokens * cfg.dim, dtype=np.float32)
        fn = lambda: oracle.vit_block(x, w, cfg.tokens, cfg.heads, cfg.head_dim, cfg.mlp,
                                      cfg.eps, threads=threads)
        return fn, 1.0 / cfg.layers, ("one ViT-L block (T=%d) per step = 1/%d frame, f64 "
                                      "oracle" % (cfg.tokens, cfg.layers))

    def cpu_baseline(self, threads: int):
        """One ViT-L block through the oracle on every host core (median of 3)
        times 24, plus the patch embedding: a whole ViT-L frame of the f64
        oracle takes about half a minute, so the frame is scaled from its
        blocks (stated in `sample`)."""
        import numpy as np
        import oracle
        c = self.cfg
        fn, _, _ = self.block_step(c, threads)
        med, times, _ = _median_time(fn, 3)
        pw = np.random.default_rng(6).standard_normal(c.taps * c.dim, dtype=np.float32) * 0.02
        t_embed, _, _ = _median_time(lambda: oracle.patch_embed(
            self.img[0], pw, None, c.grid, c.grid, c.patch, c.cin, c.dim, threads=threads), 1)
        frame_s = c.layers * med + t_embed
        return {"value": 1.0 / frame_s, "unit": "frames/s", "cores": threads, "kind": "port",
                "sample": "1 ViT-L block (median of %s s) x %d + patch embedding (%.2f s), f64 "
                          "oracle, %d threads" % ([round(x, 2) for x in times], c.layers,
                                                  t_embed, threads)}

    def parity(self):
        return {"sample": "not in the bench line (a 24-block oracle frame takes about half a "
                          "minute): tests/test_block_gpu.py::"
                          "test_vit_l_encoder_matches_the_reference_chain checks it"}


class BlockWorkload:
    """Config 2: one pre-LN ViT-S transformer block (dim 384, 6 heads x 64,
    MLP 1536 with GELU, 1370 tokens, batch 1) in f16, weights N(0, 0.02), LN
    gamma 1 / beta 0, LayerScale 1 (BASELINE gives no value), input
    activations N(0, 1). A step is the block's kernels (LayerNorm, QKV GEMM,
    attention, out-projection with LayerScale and residual, LayerNorm, fc1 +
    GELU-erf, fc2 with LayerScale and residual) replayed as one CUDA graph,
    in place on the f32 residual stream; TFLOP/s of the block's 7.731 GFLOP."""

    name = "block"
    unit = "TFLOP/s"
    dtype = "f16 weights and activations, f16 V and P; f32 accumulate and residual"
    data = "synthetic x ~ N(0,1), N(0,0.02) weights, seeded"
    workload_name = "vit_s_block_fp16 (config 2)"
    scaling = "weak"
    large, dt, bound = False, "f16", 1e-3

    def parallelism(self, world):
        return "replicas x%d (no collective)" % world

    @classmethod
    def host_inputs(cls, seed=2):
        import numpy as np
        from beatlm_b200.model import ViTConfig, block_weights_normal
        cfg = ViTConfig.large() if cls.large else ViTConfig.small()
        rng = np.random.default_rng(seed)
        w = block_weights_normal(rng, cfg.dim, cfg.mlp)
        x = rng.standard_normal(cfg.tokens * cfg.dim, dtype=np.float32)
        return cfg, w, x

    @classmethod
    def reference_step(cls, threads):
        import oracle
        cfg, w, x = cls.host_inputs()
        fn = lambda: oracle.vit_block(x, w, cfg.tokens, cfg.heads, cfg.head_dim, cfg.mlp,
                                      cfg.eps, threads=threads)
        return fn, cfg.flops_per_frame()["linear"] / cfg.layers / 1e12 + \
            4.0 * cfg.tokens ** 2 * cfg.dim / 1e12, "one %s block per step (oracle, f64)" % (
                "ViT-L" if cls.large else "ViT-S")

    def __init__(self, rank: int, world: int = 1):
        import torch
        from beatlm_b200.model import Buffers, DeviceBlock, block_specs
        from beatlm_b200.runtime import Kernels
        self.cfg, self.w, self.x = self.host_inputs()
        cfg = self.cfg
        self.blk = DeviceBlock(self.w, cfg.dim, cfg.mlp, self.dt)
        self.buf = Buffers(cfg, 1, self.dt, features=False)
        self.host = torch.from_numpy(self.x.reshape(cfg.tokens, cfg.dim)).pin_memory()
        self.out_host = torch.empty((cfg.tokens, cfg.dim), dtype=torch.float32).pin_memory()
        self.buf.x.copy_(self.host)
        self.prog = Kernels(block_specs(self.blk, cfg, self.buf))
        self.graph = None
        t, d, m = cfg.tokens, cfg.dim, cfg.mlp
        self.linear_flops = 2.0 * t * d * (3 * d + d + 2 * m)
        self.attn_flops = 4.0 * t * t * d
        self.flops = self.linear_flops + self.attn_flops
        self.launches_per_step = len(self.prog)

    def config(self):
        c = self.cfg
        return {"workload": self.workload_name, "tokens": c.tokens, "dim": c.dim,
                "heads": c.heads, "mlp": c.mlp, "dtype": self.dt,
                "weights": "random N(0,0.02), LN gamma=1 beta=0, LayerScale=1",
                "launch": "one CUDA graph per step (%d kernels)" % self.launches_per_step,
                "gflop_per_step": round(self.flops / 1e9, 3),
                "l2": "flushed before every timed step (256 MiB write)"}

    def step(self, stream):
        if self.graph is None:
            self.graph = self.prog.capture(stream)
        self.graph.launch(stream)

    e2e_how = ("each step: the block's input rows, whose host-to-device copy was issued beside "
               "the previous step's block into one of two staging buffers "
               "(runtime.InputPipeline), copied into the residual stream on the device, the "
               "block's graph, its output copied to pinned host memory inside the step; L2 "
               "flushed between steps")

    def step_e2e(self, stream):
        import torch
        from beatlm_b200.runtime import InputPipeline
        if getattr(self, "inputs", None) is None:
            self.inputs = InputPipeline([self.host, self.host],
                                        [torch.empty_like(self.buf.x), torch.empty_like(self.buf.x)])
        staged = self.inputs.acquire(stream)
        self.buf.x.copy_(staged, non_blocking=True)
        self.inputs.release(stream)
        self.step(stream)
        self.out_host.copy_(self.buf.x, non_blocking=True)

    def e2e_bytes(self):
        return self.host.numel() * 4, self.out_host.numel() * 4

    def units(self):
        return self.flops / 1e12

    def roofline(self, stream, avg_ms):
        import torch
        from beatlm_b200.runtime import SliceTimer, hold
        t = SliceTimer(max_slices=len(self.prog))
        kinds = {}
        for f in range(5):
            self.buf.x.copy_(self.host)
            h = t.begin_frame(f)
            hold(stream, 20000)
            self.prog.encode_all(stream, timer=t, frame=h)
            t.submitted(h)
            torch.cuda.synchronize()
            for ft in t.collect_ready():
                for k, us in ft.compute:
                    kind = self.prog.label(k).split(".")[-1]
                    kinds.setdefault(kind, []).append(us)
        t.close()
        att = statistics.mean(kinds["attention"])
        return {"achieved_tflops": self.attn_flops / (att / 1e6) / 1e12,
                "kernel": "bl::attn::attention_fwd (the block's attention)",
                "how": "cudaEvent slice timer around each kernel of 5 direct encodes, queued "
                       "behind a stream hold",
                "block_tflops": self.flops / (avg_ms / 1e3) / 1e12,
                "gemm_tflops": self.linear_flops / (sum(statistics.mean(kinds[k]) for k in
                                                        ("qkv", "proj", "fc1", "fc2")) / 1e6)
                / 1e12,
                "kernels_us": {k: round(statistics.mean(v), 2) for k, v in sorted(kinds.items())}}

    def parity(self):
        """One block from the seeded input against oracle.vit_block fed the
        weights as the device holds them and Q/K/V as stored (f16)."""
        import oracle
        import torch
        from beatlm_b200.model import DeviceBlock
        cfg = self.cfg
        self.buf.x.copy_(self.host)
        self.prog.encode_all(None)
        torch.cuda.synchronize()
        want = oracle.vit_block(self.x, DeviceBlock.rounded(self.w, self.dt), cfg.tokens,
                                cfg.heads, 64, cfg.mlp, cfg.eps, qkv_round="qk_" + self.dt)
        rel, mx = _rel(self.buf.x.cpu().numpy(), want)
        return {"rel_l2": rel, "max_abs": mx, "bound": self.bound,
                "sample": "the whole block output vs oracle.vit_block"}

    def cpu_baseline(self, threads: int):
        import oracle
        cfg = self.cfg
        fn = lambda: oracle.vit_block(self.x, self.w, cfg.tokens, cfg.heads, 64, cfg.mlp,
                                      cfg.eps, threads=threads)
        med, times, _ = _median_time(fn, 3)
        return {"value": self.flops / med / 1e12, "unit": "TFLOP/s", "cores": threads,
                "kind": "port", "sample": "the whole block through oracle.vit_block "
                                          "(reference.rs:520-544), median of %s s"
                                          % [round(x, 2) for x in times]}


class VitLBlockWorkload(BlockWorkload):
    """One block of config 4's ViT-L/14 encoder (dim 1024, 16 heads, MLP
    4096, 1370 tokens) in bf16, weights N(0, 0.02): the block workload at the
    large shapes, where the GEMMs carry enough work to study on their own."""

    name = "vitl_block"
    large, dt, bound = True, "bf16", 4e-3
    dtype = "bf16 weights and activations, f16 V and P; f32 accumulate and residual"
    workload_name = "vit_l14_block_bf16 (config 4, one block)"


class HiresWorkload:
    """Config 5: the high-resolution ViT-L attention, T = 74*74 + 1 = 5477,
    16 heads x 64, bf16 Q/K (V f16), Q/K/V ~ N(0,1), batch 1. With g ranks
    each holds 16/g heads (made locally from the seed) and its attention
    kernel stores each finished row of its heads into every rank's
    [T][1024] output (peer stores over NVLink), then waits on the device for
    the other ranks' arrival flags: the op is one launch per rank and the
    head outputs cross NVLink while the kernel still computes."""

    name = "hires"
    unit = "TFLOP/s"
    dtype = "bf16 Q/K, f16 V and P; f32 scores, softmax and accumulator; f16 output"
    data = "synthetic Q/K/V ~ N(0,1), seeded, each rank makes its own heads"
    workload_name = "hires_vit_l_attention_T5477 (config 5)"
    scaling = "strong"
    T, H = 5477, 16

    def parallelism(self, world):
        return ("heads/%d per GPU, outputs stored into every GPU by the attention kernel "
                "(peer memory over NVLink)" % world if world > 1 else "1 GPU, all heads")

    @classmethod
    def _qkv(cls, h0, h1):
        import numpy as np
        rng = np.random.default_rng(4321)
        full = rng.standard_normal((1, cls.T, 3, cls.H, 64), dtype=np.float32)
        return np.ascontiguousarray(full[:, :, :, h0:h1])

    @classmethod
    def reference_step(cls, threads):
        import oracle
        t, h = cls.T, cls.H
        qkv = cls._ref_input()
        rows = 8
        t0 = time.perf_counter()
        oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
        per_row = (time.perf_counter() - t0) / rows
        rows = int(max(8, min(t, 2.0 / max(per_row, 1e-9))))
        fn = lambda: oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
        return fn, 4.0 * rows * t * h * 64 / 1e12, (
            "%d of %d query rows x %d heads per step (oracle/oracle.c, f64)" % (rows, t, h))

    @classmethod
    def _ref_input(cls):
        """All heads' Q/K/V rounded as the device holds them (bf16 Q/K, f16 V)."""
        import oracle
        q = cls._qkv(0, cls.H)[0]
        q[:, :2] = oracle.round_bf16(q[:, :2])
        q[:, 2:] = oracle.round_f16(q[:, 2:])
        return q.reshape(cls.T, -1)

    def __init__(self, rank: int, world: int = 1):
        import torch
        import beatlm_b200 as bl
        from beatlm_b200.parallel import HeadParallelAttention
        self.world, self.rank = world, rank
        self.op = HeadParallelAttention(self.T, self.H, rank, world, out_dtype="f16")
        qkv = self._qkv(self.op.h0, self.op.h1)
        self.dev = bl.pack_qkv(qkv, "bf16")
        self.host = self.dev.cpu().pin_memory()
        self.out_host = torch.empty(self.op.out.shape, dtype=self.op.out.dtype).pin_memory()
        self.launches_per_step = 1

    def config(self):
        return {"workload": self.workload_name, "batch": 1, "tokens": self.T, "heads": self.H,
                "head_dim": 64, "heads_per_gpu": self.op.local_heads,
                "qkv_dtype": "bf16 Q/K, f16 V", "out_dtype": "f16",
                "exchange": self.op.exchange_name(),
                "attention_launch": self.op.launch_shape(self.dev),
                "l2": "flushed before every timed step (256 MiB write)"}

    def step(self, stream):
        self.op(self.dev, stream=stream)

    e2e_how = AttentionWorkload.e2e_how

    def step_e2e(self, stream):
        import torch
        from beatlm_b200.runtime import InputPipeline
        if getattr(self, "inputs", None) is None:
            self.inputs = InputPipeline([self.host, self.host],
                                        [self.dev, torch.empty_like(self.dev)])
        dev = self.inputs.acquire(stream)
        self.op(dev, stream=stream)
        self.inputs.release(stream)
        self.out_host.copy_(self.op.out, non_blocking=True)

    def e2e_bytes(self):
        return self.host.numel() * 2, self.out_host.numel() * 2

    def units(self):
        return self.op.flops() / self.world / 1e12  # this rank's share, TFLOP per step

    def roofline(self, stream, avg_ms, reps: int = 10):
        """This rank's attention alone (local heads, local output, no
        exchange), CUDA events on its stream; the exchange's share is the
        step time minus this."""
        import torch
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        ms = time_device(lambda s: self.op.compute_local(self.dev, stream=s), reps, 3, stream,
                         flush)
        avg = sum(ms) / len(ms)
        return {"achieved_tflops": self.op.flops() / self.world / (avg / 1e3) / 1e12,
                "kernel": "bl::attn::attention_fwd (%d heads of %d on this GPU)"
                          % (self.op.local_heads, self.H),
                "how": "CUDA events around %d attention-only launches (no exchange) after the "
                       "timed region, L2 flushed between them" % reps,
                # one capture of the 16-head launch; a rank with fewer heads
                # reads that share of the Q/K/V
                "traffic": (lambda b: None if b is None else
                            int(b * self.op.local_heads / self.H))(
                    profiled_traffic("attention_fwd_hires_T5477_H16.md")),
                "attention_ms": round(avg, 5),
                "step_minus_attention_ms": round(avg_ms - avg, 5),
                **self.nccl_baseline(stream)}

    def nccl_baseline(self, stream, reps: int = 10):
        """The same op with the plain collective form of the exchange (one
        attention launch into this rank's slab, then an NCCL all-gather),
        timed the same way: the baseline the fused exchange replaces. Every
        rank runs it (it holds a collective)."""
        if self.world == 1:
            return {}
        import torch
        import torch.distributed as dist
        from beatlm_b200.parallel import HeadParallelAttention
        op = HeadParallelAttention(self.T, self.H, self.rank, self.world, out_dtype="f16",
                                   exchange="nccl")
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        ms = time_device(lambda s: op(self.dev, stream=s), reps, 3, stream, flush)
        t = torch.tensor([sum(ms) / len(ms)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        avg = float(t[0])
        return {"nccl_allgather_form": {
            "tflops": round(op.flops() / (avg / 1e3) / 1e12, 2), "ms_per_step": round(avg, 5),
            "how": "attention into this rank's slab + NCCL all_gather_into_tensor, max over "
                   "ranks of %d event-timed steps" % reps}}

    def parity(self):
        """64 query rows of the assembled [T][1024] output (all 16 heads, so
        every rank's slab) on this rank, from the last e2e step's host copy,
        against the oracle fed the same 16-bit Q/K/V."""
        import numpy as np
        import oracle
        qkv = self._ref_input()
        got = self.out_host.float().numpy().reshape(self.T, self.H * 64)
        pairs = []
        for r0 in (0, self.T // 2, self.T - 16, 1000):
            want = oracle.attention(qkv, self.T, self.H, 64, rows=(r0, r0 + 16))
            pairs.append((got[r0:r0 + 16].ravel(), want))
        rel, mx = _rel(np.concatenate([g for g, _ in pairs]), np.concatenate([w for _, w in pairs]))
        return {"rel_l2": rel, "max_abs": mx, "bound": 1e-3,
                "sample": "64 query rows (0-15, 1000-1015, 2738-2753, 5461-5476) x all 16 heads "
                          "of the assembled output on rank 0, vs oracle.attention"}

    def cpu_baseline(self, threads: int, budget_s: float = 8.0):
        return oracle_attention_rate(self._ref_input(), self.T, self.H, threads, budget_s)


class DepthWorkload:
    """The whole Depth-Anything-V2-Small model at 518 px, one frame per step:
    the encoder (one CUDA graph, as the encoder workload runs it) and the DPT
    head (model.Decoder: im2col + tcgen05 GEMM convolutions, transposed
    convolutions, bilinear resampling), random weights; frames/s."""

    name = "depth"
    unit = "frames/s"
    dtype = "bf16 encoder; f16 decoder operands; f32 accumulation, residual and maps"
    data = "synthetic 518x518x3 image U[0,1] ImageNet-normalised, random weights, seeded"
    workload_name = "da_v2_small_depth_518 (encoder + DPT head)"
    scaling = "weak"

    def parallelism(self, world):
        return "replicas x%d (no collective)" % world

    @classmethod
    def reference_step(cls, threads):
        return EncoderWorkload.reference_step(threads)

    def __init__(self, rank: int, world: int = 1):
        import torch
        from beatlm_b200.model import Decoder, DecoderConfig, decoder_weights_random
        self.enc_wl = EncoderWorkload(rank)
        cfg = self.enc_wl.cfg
        self.dec = Decoder(cfg, DecoderConfig(), decoder_weights_random(cfg, DecoderConfig(),
                                                                        seed=rank))
        self.feats = self.enc_wl.enc.features(1)
        side = cfg.grid * cfg.patch
        self.depth_host = torch.empty((side, side), dtype=torch.float32).pin_memory()
        # ours in the head, counted from its structure (64 at DPT-S)
        self.launches_per_step = self.enc_wl.launches_per_step + self.dec.launches_per_frame()
        self.flops = self.enc_wl.flops

    def config(self):
        c = dict(self.enc_wl.config())
        c.update({"workload": self.workload_name,
                  "decoder": "DPT-S head: neck 48/96/192/384, fusion 64, head 32, depth 518x518",
                  "launch": "encoder: one CUDA graph; decoder: one CUDA graph"})
        return c

    def step(self, stream):
        self.enc_wl.step(stream)
        if getattr(self, "dec_graph", None) is None:  # captured once, at the first warm-up
            self.dec_graph, self.depth = self.dec.capture(self.feats, stream)
        self.dec_graph.replay()

    e2e_how = ("each step: the frame's image, whose host-to-device copy was issued beside the "
               "previous step's pass into one of two staging buffers (runtime.InputPipeline), "
               "copied into the encoder's image buffer on the device, the encoder and DPT head "
               "graphs, the depth map copied to pinned host memory inside the step; L2 flushed "
               "between steps")

    def step_e2e(self, stream):
        import torch
        from beatlm_b200.runtime import InputPipeline
        img = self.enc_wl.buf.image
        if getattr(self, "inputs", None) is None:
            self.inputs = InputPipeline([self.enc_wl.host, self.enc_wl.host],
                                        [torch.empty_like(img), torch.empty_like(img)])
        staged = self.inputs.acquire(stream)
        img.copy_(staged, non_blocking=True)
        self.inputs.release(stream)
        self.step(stream)
        self.depth_host.copy_(self.depth, non_blocking=True)

    def e2e_bytes(self):
        return self.enc_wl.host.numel() * 4, self.depth_host.numel() * 4

    def units(self):
        return 1

    def roofline(self, stream, avg_ms):
        return self.enc_wl.roofline(stream, avg_ms)

    def parity(self):
        return None

    def cpu_baseline(self, threads: int):
        """The encoder's CPU frame and one run of the DPT head through the
        oracle at 518 px, combined per frame."""
        import numpy as np
        import oracle
        from beatlm_b200.model import DecoderConfig, decoder_weights_random
        enc = self.enc_wl.cpu_baseline(threads)
        cfg, d = self.enc_wl.cfg, DecoderConfig()
        w = decoder_weights_random(cfg, d, seed=1)
        rng = np.random.default_rng(3)
        feats = [rng.standard_normal(cfg.grid * cfg.grid * cfg.dim).astype(np.float32)
                 for _ in range(4)]
        t0 = time.perf_counter()
        oracle.dpt_head(cfg.grid, cfg.patch, cfg.dim, d.neck, d.reassemble, d.fusion, d.head,
                        w, feats, threads=threads)
        t_dec = time.perf_counter() - t0
        frame_s = 1.0 / enc["value"] + t_dec
        return {"value": 1.0 / frame_s, "unit": "frames/s", "cores": threads, "kind": "port",
                "sample": "%s; plus one DPT head at 518 px through oracle/oracle.c (%.1f s)"
                          % (enc["sample"], t_dec)}


class DecoderWorkload:
    """A DPT-S fusion residual unit at the first fusion stage's 148 x 148 x 64
    map: x + conv2(relu(conv1(relu(x)))) (crates/beatlm-bench/src/
    reference.rs:190-201), two bl_im2col gathers and two tcgen05 GEMMs (the
    second adds x in its epilogue)."""

    name = "decoder"
    unit = "TFLOP/s"
    dtype = "f16 operands, f32 accumulation and maps"
    data = "synthetic map ~ N(0,1), weights N(0, 1/sqrt(9c)), seeded"
    workload_name = "dpt_s_residual_unit_148 (decoder, section 8 next row 1)"
    scaling = "weak"
    side, c = 148, 64

    def parallelism(self, world):
        return "replicas x%d (no collective)" % world

    def roofline(self, stream, avg_ms):
        return {"achieved_tflops": self.flops / (avg_ms / 1e3) / 1e12,
                "kernel": "bl::gemm::gemm_persistent (2 launches) + im2col (2 launches)",
                "how": "CUDA events around every timed step; the im2col gathers are inside the "
                       "time, so the figure is the two GEMMs' floor"}

    @classmethod
    def reference_step(cls, threads):
        import numpy as np
        import oracle
        side, c = 37, cls.c
        rng = np.random.default_rng(99)
        x = rng.standard_normal(side * side * c).astype(np.float32)
        w = (rng.standard_normal(9 * c * c) / 24).astype(np.float32)
        b = np.zeros(c, np.float32)
        fn = lambda: oracle.residual_unit(x, w, b, w, b, side, side, c)
        return fn, 2 * 2.0 * side * side * c * 9 * c / 1e12, (
            "one residual unit on a 37 x 37 x 64 map (oracle/oracle.c, f64)")

    def __init__(self, rank: int, world: int = 1):
        import ctypes
        import numpy as np
        import torch
        from beatlm_b200 import _native as N
        from beatlm_b200 import ops
        self.N, self.ctypes = N, ctypes
        side, c = self.side, self.c
        px = side * side
        rng = np.random.default_rng(77 + rank)
        self.x = torch.from_numpy(rng.standard_normal((px, c)).astype(np.float32)).cuda()
        ws = [(rng.standard_normal(9 * c * c) / 24).astype(np.float32) for _ in range(2)]
        self.w = [ops.conv_weights(w, 3, c, c) for w in ws]
        self.b = [torch.from_numpy((rng.standard_normal(c) * 0.1).astype(np.float32)).cuda()
                  for _ in range(2)]
        k_pad = self.w[0].shape[1]
        self.cols = torch.empty((px, k_pad), dtype=torch.float16, device="cuda")
        # the first convolution's map is read only by the second one's gather:
        # stored in f16 by its epilogue and copied as it is by the gather
        # (model.Decoder's residual unit; the same bits as an f32 map)
        self.mid = torch.empty((px, c), dtype=torch.float16, device="cuda")
        self.out = torch.empty((px, c), dtype=torch.float32, device="cuda")
        self.host = self.x.cpu().pin_memory()
        self.out_host = torch.empty((px, c), dtype=torch.float32).pin_memory()
        mk = lambda src, dt: N.Im2colArgs(input=src.data_ptr(), h=side, w=side, cin=c, ksize=3,
                                          stride=1, relu=1, out=self.cols.data_ptr(),
                                          out_dtype=N.BL_F16, k_pad=k_pad, in_dtype=dt)
        self.i2c = [mk(self.x, N.BL_F32), mk(self.mid, N.BL_F16)]
        self.g = [ops.gemm_args(self.w[0], a=self.cols, bias=self.b[0], out=self.mid),
                  ops.gemm_args(self.w[1], a=self.cols, bias=self.b[1], residual=self.x,
                                out=self.out)]
        self.flops = 2 * 2.0 * px * c * 9 * c
        self.launches_per_step = 4

    def config(self):
        return {"workload": self.workload_name, "map": [self.side, self.side, self.c],
                "convolutions": "2 x 3x3, padding 1, ReLU before each, residual add",
                "k": 9 * self.c, "l2": "flushed before every timed step (256 MiB write)"}

    def step(self, stream):
        from beatlm_b200.ops import _stream_ptr
        s = _stream_ptr(stream)
        L = self.N.lib()
        for i in range(2):
            self.N.check(L.bl_im2col(self.ctypes.byref(self.i2c[i]), s))
            self.N.check(L.bl_gemm(self.ctypes.byref(self.g[i]), s))

    e2e_how = ("each step: the unit's input map, whose host-to-device copy was issued beside "
               "the previous step into one of two staging buffers (runtime.InputPipeline), "
               "copied into the unit's input on the device, the two convolutions, the output "
               "copied to pinned host memory inside the step; L2 flushed between steps")

    def step_e2e(self, stream):
        import torch
        from beatlm_b200.runtime import InputPipeline
        if getattr(self, "inputs", None) is None:
            self.inputs = InputPipeline([self.host, self.host],
                                        [torch.empty_like(self.x), torch.empty_like(self.x)])
        staged = self.inputs.acquire(stream)
        self.x.copy_(staged, non_blocking=True)
        self.inputs.release(stream)
        self.step(stream)
        self.out_host.copy_(self.out, non_blocking=True)

    def e2e_bytes(self):
        return self.host.numel() * 4, self.out_host.numel() * 4

    def units(self):
        return self.flops / 1e12

    def parity(self):
        return None

    def cpu_baseline(self, threads: int):
        fn, tflop, sample = self.reference_step(threads)
        med, _, _ = _median_time(fn, 3)
        return {"value": tflop / med, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": "%s, median of 3" % sample}


WORKLOADS = {"attention": AttentionWorkload, "block": BlockWorkload,
             "vitl_block": VitLBlockWorkload, "encoder": EncoderWorkload,
             "vitl": VitLWorkload, "hires": HiresWorkload, "decoder": DecoderWorkload,
             "depth": DepthWorkload}
# the other configs carried in the default line, by GPU count
EXTRAS_ONE = ("attention", "block", "vitl", "hires")
EXTRAS_MANY = ("vitl", "hires")


# ------------------------------------------------------------------ timing

def time_device(fn, steps, warmup, stream, flush):
    import torch
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            flush.zero_()
            fn(stream)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    with torch.cuda.stream(stream):
        for i in range(steps):
            flush.zero_()
            starts[i].record(stream)
            fn(stream)
            ends[i].record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def measure(wl, steps, warmup, stream, flush, world, rank, local, cpu_threads):
    """Times one workload (device-resident and end to end), then its roofline,
    parity and (one GPU, rank 0) CPU baseline. Every rank runs the same
    collective steps in the same order. Returns the line's fields."""
    import torch
    import torch.distributed as dist

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    with Clocks(local) as clk:
        times = time_device(wl.step, steps, warmup, stream, flush)
    barrier()
    total_ms = sum(times)
    barrier()
    e2e_times = time_device(wl.step_e2e, steps, warmup, stream, flush)
    barrier()
    e2e_ms = sum(e2e_times)
    if world > 1:
        t = torch.tensor([total_ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = float(t[0]), float(t[1])
    value = wl.units() * steps * world / (total_ms / 1e3)
    e2e_value = wl.units() * steps * world / (e2e_ms / 1e3)
    extra = wl.roofline(stream, total_ms / steps)
    barrier()
    if rank != 0:
        return None
    pk = peaks()
    achieved = extra.pop("achieved_tflops")
    kernels = extra.pop("kernels", None)
    kernel, how, traffic = extra.pop("kernel"), extra.pop("how"), extra.pop("traffic", None)
    out = {
        "metric": METRIC, "value": round(value, 3), "unit": wl.unit, "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(total_ms / steps, 5),
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None,
        "dtype": wl.dtype, "data": wl.data,
        "config": dict(wl.config(), parallelism=wl.parallelism(world)),
        "e2e": dict({"value": round(e2e_value, 3), "unit": wl.unit,
                     "h2d_bytes_per_step": wl.e2e_bytes()[0],
                     "d2h_bytes_per_step": wl.e2e_bytes()[1]},
                    **({"how": wl.e2e_how} if getattr(wl, "e2e_how", None) else {})),
        "gpu_launches": wl.launches_per_step * steps,
        "roofline": dict({"bound": "tensor", "achieved": round(achieved, 2),
                          "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                          "frac": round(achieved / pk["bf16_tflops"], 4),
                          "peak_source": pk["source"] + " burst bf16 (MEASURED_PEAKS.json)",
                          "traffic": traffic, "kernel": kernel, "how": how},
                         **{k: (round(v, 3) if isinstance(v, float) else v)
                            for k, v in extra.items()}),
        "clocks": clk.summary,
    }
    if kernels:
        out["kernels_us_per_step"] = kernels
    if world == 1 and cpu_threads:
        out["cpu_baseline"] = wl.cpu_baseline(threads=cpu_threads)
    par = wl.parity()
    if par is not None:
        out["parity"] = par
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="encoder", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the cpu_baseline legs (profiling runs)")
    ap.add_argument("--no-extra", action="store_true",
                    help="measure the chosen workload only (no other configs in the line)")
    ap.add_argument("--launch", default="graph", choices=["graph", "direct"],
                    help="encoder workloads: replay one CUDA graph per step (default) or "
                         "launch every kernel from the host")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, world, rank)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    stream = torch.cuda.Stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    threads = 0 if args.no_cpu_baseline else (os.cpu_count() or 1)

    wl = WORKLOADS[args.workload](rank, world=world)
    if isinstance(wl, EncoderWorkload):
        wl.launch = args.launch
    line = measure(wl, args.steps, args.warmup, stream, flush, world, rank, local, threads)
    del wl
    torch.cuda.empty_cache()

    if args.workload == "encoder" and not args.no_extra:
        extra_steps = max(3, min(args.steps, 10))
        configs = {}
        for name in (EXTRAS_MANY if world > 1 else EXTRAS_ONE):
            sub = WORKLOADS[name](rank, world=world)
            r = measure(sub, extra_steps, 3, stream, flush, world, rank, local, threads)
            if rank == 0:
                r.pop("metric", None)
                configs[name] = r
            sub = None
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
        if rank == 0:
            line["configs"] = configs
            line["gpu_launches"] += sum(c["gpu_launches"] for c in configs.values())
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, world, rank):
    """The reference's CPU implementation of the path: the oracle port (the
    Rust reference has no toolchain here), all host threads, rank 0 only; each
    step is the workload's reference_step (the encoder: one whole frame), run
    `warmup` times untimed and `steps` times timed."""
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    step, units_per_step, sample = wl.reference_step(threads)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = units_per_step * args.steps / dt
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": wl.unit,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": wl.scaling, "vs_baseline": None, "dtype": "f64 accumulate, f32 storage",
            "data": "synthetic, seeded (the same inputs as the GPU arm's cpu_baseline leg)",
            "config": {"workload": wl.workload_name},
            "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
