#!/usr/bin/env python
"""Benchmark of the ViT attention hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload encoder|attention|vitl|hires]

Workloads (synthetic data, seeded):
  encoder    config 3 (default): the DA-V2-Small ViT-S/14 encoder at 518 px,
             one frame per step through a CUDA graph; frames/s.
  attention  config 1: one ViT-S self-attention op, batch 1, 6 heads x 64,
             1370 tokens, Q/K/V ~ N(0,1), scale 1/8; f16 Q/K/V, f32 output.
  vitl       config 4: the ViT-L/14 encoder, one independent stream per GPU.
  hires      config 5: T=5477 attention, 16 heads split over the GPUs, NCCL
             all-gather of the head outputs; TFLOP/s of the whole op.

A step is one pass of the hot path over one batch. `value` is whole-job
throughput (all ranks) with the inputs resident in HBM; L2 is flushed (a
256 MiB write) before every timed step and the flush is outside the timed
events. `e2e` is the same metric through the public call with host buffers:
the H2D copy of the step's inputs from pinned memory and the D2H copy of its
result are inside its timed region. Multi-GPU: one process per GPU
(torchrun); configs 1-4 run independent replicas or streams (weak scaling),
config 5 splits one op by heads (strong scaling); times are the max over
ranks.

`--impl reference` times the reference's CPU path (the C restatement of its
f64 interpreter, oracle/, all host threads) on the same workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ViT attention TFLOP/s (% of B200 bf16 peak); DA-V2-S 518² encoder frames/s"


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


# ------------------------------------------------------------------ workloads

class AttentionWorkload:
    """Config 1: one ViT-S attention op (T=1370, H=6, hd=64), batch 1."""

    name = "attention"
    unit = "TFLOP/s"
    dtype = "f16 Q/K/V and P; f32 scores, softmax and accumulator"
    data = "synthetic Q/K/V ~ N(0,1), seeded"
    workload_name = "vit_s_attention_op (config 1)"
    scaling = "weak"

    def parallelism(self, world):
        return "replicas x%d (no collective)" % world

    def roofline(self, stream, avg_ms):
        return {"achieved_tflops": self.flops / (avg_ms / 1e3) / 1e12,
                "kernel": "bl::attn::attention_fwd",
                "how": "CUDA events around every timed launch (a step is one launch)"}

    @classmethod
    def reference_step(cls, threads):
        import numpy as np
        import oracle
        t, h = 1370, 6
        rng = np.random.default_rng(1234)
        qkv = oracle.round_f16(rng.standard_normal((t, 3 * h * 64), dtype=np.float32))
        rows = 32
        t0 = time.perf_counter()
        oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
        per_row = (time.perf_counter() - t0) / rows
        rows = int(max(16, min(t, 1.0 / max(per_row, 1e-9))))
        fn = lambda: oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
        return fn, 4.0 * rows * t * h * 64 / 1e12, (
            "%d of %d query rows x %d heads per step (oracle/oracle.c, f64)" % (rows, t, h))

    def __init__(self, rank: int, batch: int = 1):
        import numpy as np
        import torch
        import beatlm_b200 as bl
        self.bl = bl
        self.t, self.h, self.batch = 1370, 6, batch
        rng = np.random.default_rng(1234 + rank)
        qkv = rng.standard_normal((batch, self.t, 3, self.h, 64), dtype=np.float32)
        self.dev = bl.pack_qkv(qkv, "f16")
        self.host = self.dev.cpu().pin_memory()
        self.out = torch.empty((batch, self.t, self.h * 64), dtype=torch.float32, device="cuda")
        self.out_host = torch.empty(self.out.shape, dtype=torch.float32).pin_memory()
        self.flops = 4.0 * self.t * self.t * self.h * 64 * batch
        self.unit_bytes = self.dev.numel() * 2 + self.out.numel() * 4
        self.launches_per_step = 1

    def config(self):
        return {"workload": "vit_s_attention_op (config 1)", "batch": self.batch,
                "tokens": self.t, "heads": self.h, "head_dim": 64,
                "qkv_dtype": "f16", "out_dtype": "f32",
                "l2": "flushed before every timed launch (256 MiB write)"}

    def step(self, stream):
        self.bl.attention(self.dev, tokens=self.t, heads=self.h, batch=self.batch,
                          out=self.out, stream=stream)

    def step_e2e(self, stream):
        self.dev.copy_(self.host, non_blocking=True)
        self.step(stream)
        self.out_host.copy_(self.out, non_blocking=True)

    def e2e_bytes(self):
        return self.host.numel() * 2, self.out_host.numel() * 4

    def units(self):
        return self.flops / 1e12  # TFLOP per step

    def cpu_baseline(self, threads: int, budget_s: float = 15.0):
        import torch
        qkv = self.host[0].view(torch.float16).float().numpy().reshape(self.t, -1)
        return oracle_attention_rate(qkv, self.t, self.h, threads, budget_s)


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

    def __init__(self, rank: int):
        import torch
        from beatlm_b200.model import Decoder, DecoderConfig, decoder_weights_random
        self.enc_wl = EncoderWorkload(rank)
        cfg = self.enc_wl.cfg
        self.dec = Decoder(cfg, DecoderConfig(), decoder_weights_random(cfg, DecoderConfig(),
                                                                        seed=rank))
        self.feats = self.enc_wl.enc.features(1)
        side = cfg.grid * cfg.patch
        self.depth_host = torch.empty((side, side), dtype=torch.float32).pin_memory()
        # ours in the head: 2 per convolution (im2col, GEMM), 3 per transposed
        # convolution, 1 per resampling: 24 reassembly, 40 fusion, 7 head
        self.launches_per_step = self.enc_wl.launches_per_step + 71
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

    def step_e2e(self, stream):
        self.enc_wl.buf.image.copy_(self.enc_wl.host, non_blocking=True)
        self.step(stream)
        self.depth_host.copy_(self.depth, non_blocking=True)

    def e2e_bytes(self):
        return self.enc_wl.host.numel() * 4, self.depth_host.numel() * 4

    def units(self):
        return 1

    def roofline(self, stream, avg_ms):
        return self.enc_wl.roofline(stream, avg_ms)

    def cpu_baseline(self, threads: int, budget_s: float = 15.0):
        """The encoder's CPU rate (its own bounded sample) and one run of the
        DPT head through the oracle at 518 px, combined per frame."""
        import numpy as np
        import oracle
        from beatlm_b200.model import DecoderConfig, decoder_weights_random
        enc = self.enc_wl.cpu_baseline(threads, budget_s)
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

    def __init__(self, rank: int):
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
        self.mid = torch.empty((px, c), dtype=torch.float32, device="cuda")
        self.out = torch.empty((px, c), dtype=torch.float32, device="cuda")
        self.host = self.x.cpu().pin_memory()
        self.out_host = torch.empty((px, c), dtype=torch.float32).pin_memory()
        mk = lambda src: N.Im2colArgs(input=src.data_ptr(), h=side, w=side, cin=c, ksize=3,
                                      stride=1, relu=1, out=self.cols.data_ptr(),
                                      out_dtype=N.BL_F16, k_pad=k_pad)
        self.i2c = [mk(self.x), mk(self.mid)]
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

    def step_e2e(self, stream):
        self.x.copy_(self.host, non_blocking=True)
        self.step(stream)
        self.out_host.copy_(self.out, non_blocking=True)

    def e2e_bytes(self):
        return self.host.numel() * 4, self.out_host.numel() * 4

    def units(self):
        return self.flops / 1e12

    def cpu_baseline(self, threads: int, budget_s: float = 15.0):
        fn, tflop, sample = self.reference_step(threads)
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < budget_s or n == 0:
            fn()
            n += 1
        dt = time.perf_counter() - t0
        return {"value": tflop * n / dt, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": "%s, %d repeats" % (sample, n)}


def oracle_attention_rate(qkv, t, h, threads, budget_s):
    """The reference's CPU path for one attention op (oracle/, a C restatement
    of reference.rs:437-494, f64 accumulation) timed on a bounded sample of
    query rows of every head, in TFLOP/s."""
    import oracle
    rows = 16
    t0 = time.perf_counter()
    oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
    dt = time.perf_counter() - t0
    rows = int(min(t, max(rows, rows * budget_s / max(dt, 1e-6) / 4)))
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < budget_s / 2 or n == 0:
        oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
        n += 1
    dt = time.perf_counter() - t0
    flops = 4.0 * rows * t * h * 64 * n
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": "%d of %d query rows x %d heads, %d repeats (f64 accumulation, "
                      "oracle/oracle.c)" % (rows, t, h, n)}


class EncoderWorkload:
    """Config 3: the Depth-Anything-V2-Small ViT-S/14 encoder at 518 px, 12
    blocks, bf16, random N(0, 0.02) weights (LayerNorm gamma 1 / beta 0,
    LayerScale 1), one frame per forward (batch 1), input U[0,1] normalised by
    the ImageNet mean/std. A step is one frame through a captured CUDA graph of
    the whole encoder (patch embedding, 12 blocks of 5 fused kernels, the four
    feature LayerNorms)."""

    name = "encoder"
    unit = "frames/s"
    dtype = "bf16 (weights, activations, Q/K); f16 V and P; f32 accumulate and residual"
    data = "synthetic: ImageNet-normalised U[0,1] 518x518x3 image, N(0,0.02) weights, seeded"
    workload_name = "da_v2_small_encoder_518 (config 3)"

    def roofline(self, stream, avg_ms):
        prof = self.slice_profile(stream)
        n, tot, avg_us = prof["attention"]
        steps = n / self.cfg.layers
        return {"achieved_tflops": self.attn_flops / (avg_us / 1e6) / 1e12,
                "kernel": "bl::attn::attention_fwd (%d launches per frame)" % self.cfg.layers,
                "how": "cudaEvent slice timer (bl_timer) around every kernel of 5 direct "
                       "(non-graph) encodes after the timed region, each queued behind a "
                       "20 ms stream hold so the kernels run back to back",
                "traffic": (None if self.large else
                            profiled_traffic("attention_fwd_encoder_vit_s_T1370_H6.md")),
                "kernels": {k: round(v[1] / steps, 2) for k, v in sorted(prof.items())}}

    large = False

    @classmethod
    def reference_step(cls, threads):
        """One encoder block of the oracle per step (1/layers of a frame; the
        patch embedding, under 1 % of a frame's arithmetic, is left out)."""
        import numpy as np
        import oracle
        from beatlm_b200.model import ViTConfig, block_weights_normal
        c = ViTConfig.large() if cls.large else ViTConfig.small()
        rng = np.random.default_rng(5)
        w = block_weights_normal(rng, c.dim, c.mlp)
        x = rng.standard_normal(c.tokens * c.dim, dtype=np.float32)
        fn = lambda: oracle.vit_block(x, w, c.tokens, c.heads, c.head_dim, c.mlp, c.eps,
                                      threads=threads)
        return fn, 1.0 / c.layers, ("one %s block (T=%d) per step = 1/%d frame, f64 oracle, "
                                    "patch embedding excluded"
                                    % ("ViT-L" if cls.large else "ViT-S", c.tokens, c.layers))

    scaling = "weak"

    def parallelism(self, world):
        return ("%d independent streams, one per GPU, no collective" % world if world > 1
                else "1 stream")

    def __init__(self, rank: int, frames: int = 1):
        import numpy as np
        import torch
        from beatlm_b200.model import Encoder, ViTConfig, block_weights_normal
        self.cfg = ViTConfig.large() if self.large else ViTConfig.small()
        cfg = self.cfg
        rng = np.random.default_rng(99 + rank)
        n = lambda *s: rng.standard_normal(int(np.prod(s)), dtype=np.float32) * 0.02
        w = {"blocks": [block_weights_normal(rng, cfg.dim, cfg.mlp) for _ in range(cfg.layers)],
             "patch_w": n(cfg.patch, cfg.patch, cfg.cin, cfg.dim), "patch_b": n(cfg.dim),
             "cls": n(cfg.dim), "pos": n(cfg.tokens, cfg.dim),
             "norm_g": np.ones(cfg.dim, np.float32), "norm_b": np.zeros(cfg.dim, np.float32)}
        self.frames = frames
        self.enc = Encoder(cfg, w, "bf16", planned_frames=frames)
        mean = np.array([0.485, 0.456, 0.406], np.float32)
        std = np.array([0.229, 0.224, 0.225], np.float32)
        img = ((rng.random((frames, cfg.side, cfg.side, cfg.cin), dtype=np.float32) - mean)
               / std).astype(np.float32)
        self.host = torch.from_numpy(img).pin_memory()
        self.buf = self.enc.buffers(frames)
        self.buf.image.copy_(self.host)
        self.prog = self.enc.program(frames)
        self.graph = None
        self.feats_host = [torch.empty(f.shape, dtype=f.dtype).pin_memory()
                           for f in self.enc.features(frames)]
        fl = cfg.flops_per_frame()
        self.flops = fl["total"] * frames
        self.attn_flops = 4.0 * cfg.tokens * cfg.tokens * cfg.dim * frames  # per layer launch
        self.launches_per_step = self.enc.launches_per_frame_batch(frames=frames)

    def config(self):
        c = self.cfg
        return {"workload": ("vit_l14_encoder (config 4)" if c.dim == 1024 else
                             "da_v2_small_encoder_518 (config 3)"),
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

    launch = "graph"  # or "direct": every kernel launched from the host each step

    def step(self, stream):
        if self.launch == "direct":
            self.prog.encode_all(stream)
            return
        if self.graph is None:
            self.graph = self.prog.capture(stream)
        self.graph.launch(stream)

    def step_e2e(self, stream):
        # Encoder.capture_host: image in, the encoder, each feature out on a
        # second stream once its LayerNorm has run (one graph per step)
        if getattr(self, "host_graph", None) is None:
            self.host_graph = self.enc.capture_host(self.frames, self.host, self.feats_host,
                                                    stream)
        self.host_graph.replay()

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

    def cpu_baseline(self, threads: int, budget_s: float = 15.0):
        """One encoder block through the oracle (reference.rs:520-544) on all
        host cores, scaled to a frame: 12 blocks plus the patch embedding."""
        import oracle
        from beatlm_b200.model import block_weights_normal
        import numpy as np
        c = self.cfg
        rng = np.random.default_rng(5)
        w = block_weights_normal(rng, c.dim, c.mlp)
        x = rng.standard_normal(c.tokens * c.dim, dtype=np.float32)
        t0 = time.perf_counter()
        oracle.vit_block(x, w, c.tokens, c.heads, c.head_dim, c.mlp, c.eps, threads=threads)
        t_block = time.perf_counter() - t0
        img = self.host[0].numpy().ravel()
        pw = rng.standard_normal(c.taps * c.dim, dtype=np.float32) * 0.02
        t0 = time.perf_counter()
        oracle.patch_embed(img, pw, None, c.grid, c.grid, c.patch, c.cin, c.dim, threads=threads)
        t_embed = time.perf_counter() - t0
        frame_s = c.layers * t_block + t_embed
        return {"value": 1.0 / frame_s, "unit": "frames/s", "cores": threads, "kind": "port",
                "sample": "1 block (%.2f s) x %d + patch embedding (%.2f s), f64 oracle, "
                          "%d threads" % (t_block, c.layers, t_embed, threads)}


class VitLWorkload(EncoderWorkload):
    """Config 4: a ViT-L/14-shaped encoder (24 blocks, dim 1024, 16 heads,
    MLP 4096, 1370 tokens), bf16, random N(0, 0.02) weights. Eight
    independent input streams shard one per GPU with no collective: each rank
    runs its own stream, one frame per step."""

    name = "vitl"
    large = True
    workload_name = "vit_l14_encoder (config 4)"
    data = "synthetic: ImageNet-normalised U[0,1] 518x518x3 image per stream, N(0,0.02) weights"


class HiresWorkload:
    """Config 5: the high-resolution ViT-L attention, T = 74*74 + 1 = 5477,
    16 heads x 64, bf16 Q/K (V f16), Q/K/V ~ N(0,1), batch 1. With g ranks
    each holds 16/g heads (made locally from the seed), computes their
    output slab and an NCCL all-gather assembles [T][1024] on every rank. A
    step is the whole op: the attention launch, the all-gather and the
    permute to heads side by side."""

    name = "hires"
    unit = "TFLOP/s"
    dtype = "bf16 Q/K, f16 V and P; f32 scores, softmax and accumulator; f16 output"
    data = "synthetic Q/K/V ~ N(0,1), seeded, each rank makes its own heads"
    workload_name = "hires_vit_l_attention_T5477 (config 5)"
    scaling = "strong"
    T, H = 5477, 16

    def parallelism(self, world):
        return ("heads/%d per GPU + NCCL all-gather of head outputs" % world if world > 1
                else "1 GPU, all heads")

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
        qkv = oracle.round_f16(cls._qkv(0, h)[0].reshape(t, -1))
        rows = 8
        t0 = time.perf_counter()
        oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
        per_row = (time.perf_counter() - t0) / rows
        rows = int(max(8, min(t, 2.0 / max(per_row, 1e-9))))
        fn = lambda: oracle.attention(qkv, t, h, 64, rows=(0, rows), threads=threads)
        return fn, 4.0 * rows * t * h * 64 / 1e12, (
            "%d of %d query rows x %d heads per step (oracle/oracle.c, f64)" % (rows, t, h))

    def __init__(self, rank: int, world: int = 1):
        import torch
        import beatlm_b200 as bl
        from beatlm_b200.parallel import HeadParallelAttention
        self.world = world
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
                "collective": "all_gather_into_tensor (NCCL) + permute" if self.world > 1
                              else "none",
                "l2": "flushed before every timed step (256 MiB write)"}

    def step(self, stream):
        self.op(self.dev, stream=stream)

    def step_e2e(self, stream):
        self.dev.copy_(self.host, non_blocking=True)
        self.step(stream)
        self.out_host.copy_(self.op.out, non_blocking=True)

    def e2e_bytes(self):
        return self.host.numel() * 2, self.out_host.numel() * 2

    def units(self):
        return self.op.flops() / self.world / 1e12  # this rank's share, TFLOP per step

    def roofline(self, stream, avg_ms, reps: int = 10):
        """This rank's attention launch alone, CUDA events on its stream."""
        import torch
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        ms = time_device(lambda s: self.op.compute(self.dev, stream=s), reps, 3, stream, flush)
        avg = sum(ms) / len(ms)
        return {"achieved_tflops": self.op.flops() / self.world / (avg / 1e3) / 1e12,
                "kernel": "bl::attn::attention_fwd (%d heads of %d on this GPU)"
                          % (self.op.local_heads, self.H),
                "how": "CUDA events around %d attention-only launches after the timed region, "
                       "L2 flushed between them" % reps,
                # one capture of the 16-head launch; a rank with fewer heads
                # reads that share of the Q/K/V
                "traffic": (lambda b: None if b is None else
                            int(b * self.op.local_heads / self.H))(
                    profiled_traffic("attention_fwd_hires_T5477_H16.md")),
                "attention_ms": round(avg, 5)}

    def cpu_baseline(self, threads: int, budget_s: float = 15.0):
        import oracle
        qkv = oracle.round_f16(self._qkv(0, self.H)[0].reshape(self.T, -1))
        return oracle_attention_rate(qkv, self.T, self.H, threads, budget_s)


WORKLOADS = {"attention": AttentionWorkload, "encoder": EncoderWorkload,
             "vitl": VitLWorkload, "hires": HiresWorkload, "decoder": DecoderWorkload,
             "depth": DepthWorkload}


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="encoder", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the cpu_baseline leg (profiling runs)")
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
    cls = WORKLOADS[args.workload]
    wl = cls(rank, world=world) if cls is HiresWorkload else cls(rank)
    if isinstance(wl, EncoderWorkload):
        wl.launch = args.launch
    stream = torch.cuda.Stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # device-resident timing
    barrier()
    with Clocks(local) as clk:
        times = time_device(wl.step, args.steps, args.warmup, stream, flush)
    barrier()
    total_ms = sum(times)
    # e2e through the public call with host buffers
    barrier()
    e2e_times = time_device(wl.step_e2e, args.steps, args.warmup, stream, flush)
    barrier()
    e2e_ms = sum(e2e_times)
    if world > 1:
        t = torch.tensor([total_ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = float(t[0]), float(t[1])
    value = wl.units() * args.steps * world / (total_ms / 1e3)
    e2e_value = wl.units() * args.steps * world / (e2e_ms / 1e3)
    extra = wl.roofline(stream, total_ms / args.steps)
    barrier()

    if rank == 0:
        pk = peaks()
        avg_ms = total_ms / args.steps
        achieved, kernels = extra["achieved_tflops"], extra.get("kernels")
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(avg_ms, 5),
            "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None,
            "dtype": wl.dtype, "data": wl.data,
            "config": dict(wl.config(), parallelism=wl.parallelism(world)),
            "e2e": {"value": round(e2e_value, 3), "unit": wl.unit,
                    "h2d_bytes_per_step": wl.e2e_bytes()[0],
                    "d2h_bytes_per_step": wl.e2e_bytes()[1]},
            "gpu_launches": wl.launches_per_step * args.steps,
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2),
                         "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(achieved / pk["bf16_tflops"], 4),
                         "peak_source": pk["source"] + " burst bf16 (MEASURED_PEAKS.json)",
                         "traffic": extra.get("traffic"), "kernel": extra["kernel"],
                         "how": extra["how"]},
            "clocks": clk.summary,
        }
        if kernels:
            line["kernels_us_per_step"] = kernels
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = wl.cpu_baseline(threads=os.cpu_count() or 1)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_reference(args, world, rank):
    """The reference's CPU implementation of the path: the oracle port (the
    Rust reference has no toolchain here), all host threads, rank 0 only; each
    step is a bounded sample of the workload (WORKLOADS[...].reference_step)."""
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    step, units_per_step, sample = wl.reference_step(threads)
    step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = units_per_step * args.steps / dt
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": wl.unit,
            "n_gpus": world, "steps": args.steps, "warmup": 1,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": wl.scaling,
            "vs_baseline": None, "dtype": "f64 accumulate, f32 storage",
            "data": "synthetic, seeded", "config": {"workload": wl.workload_name},
            "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
