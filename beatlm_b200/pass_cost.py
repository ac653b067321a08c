"""The pass-cost workload: what a launch costs on the GPU apart from the work
it dispatches, with and without its event pair. The reference's workload
(``crates/beatlm-host/src/pass_cost.rs:1-330``) with a CUDA launch as the
pass, a cudaEvent pair as its timestamp writes and a CUDA graph as "one
pass"; the frame itself is ``bl_pass_cost_frame_run``.

A run is every pairing (cell) of a variant with a pass count P. Frame n runs
cell n % cells (so clock drift lands on every cell alike), the first round is
untimed, one frame is in flight at a time, frames are paced at ``period_us``.
From the medians (nearest rank) of the cells' spans:

- ``per_pass_us`` (A, B, D) / ``per_dispatch_us`` (C):
  (span(P) - span(1)) / (P - 1) within one variant, trivial kernel only;
- ``over_one_pass_us``: (span_X(P) - span_C(P)) / (P - 1);
- ``over_ends_us`` (A): (span_A(P) - span_B(P)) / (P - 1);
- ``between_us`` (A): the span less the passes' own durations;
- ``encode_per_pass_us``: the host's enqueue time, derived like per_pass_us.

    python -m beatlm_b200.pass_cost [--kernels trivial|encoder] [--frames 100]
"""
from __future__ import annotations

import argparse
import ctypes
import dataclasses
import json
import time

from . import _native as N

DEFAULT_PASSES = (1, 8, 32, 128)  # pass_cost.rs:115
DEFAULT_EVERY = 8                 # pass_cost.rs:118
MAX_GROUPS = 65535                # pass_cost.rs:125

_CODES = {"per-pass": 0, "ends": 1, "one-pass": 2, "one-pass-pdl": 4}


@dataclasses.dataclass(frozen=True)
class Variant:
    """``Variant`` (pass_cost.rs:148): "per-pass", "ends", "one-pass" or
    "every" with its ``k``; "one-pass-pdl" (no reference counterpart) is the
    graph with programmatic dependent launch between its launches."""
    kind: str
    k: int = 0

    @staticmethod
    def parse(text: str) -> "Variant":
        if text in _CODES:
            return Variant(text)
        if not text.startswith("every:"):
            raise ValueError("%r is not one of per-pass, ends, one-pass, one-pass-pdl or "
                             "every:<k>" % text)
        k = text[len("every:"):]
        if not k.isdigit():
            raise ValueError("%r: %r is not a whole number" % (text, k))
        if int(k) == 0:
            raise ValueError("%r: k must be at least 1" % text)
        return Variant("every", int(k))

    @property
    def name(self) -> str:
        return "every:%d" % self.k if self.kind == "every" else self.kind

    @property
    def code(self) -> int:
        return 3 if self.kind == "every" else _CODES[self.kind]

    def times_pass(self, i: int, passes: int) -> bool:
        """Whether launch ``i`` carries its own event pair (pass_cost.rs:214)."""
        if self.kind == "per-pass":
            return True
        if self.kind == "every":
            return i % self.k == 0 or i + 1 == passes
        return False


DEFAULT_VARIANTS = (Variant("per-pass"), Variant("ends"), Variant("one-pass"),
                    Variant("every", DEFAULT_EVERY), Variant("one-pass-pdl"))


def nearest_rank(sorted_values, percent: int):
    """The ``percent``th percentile of an ascending list by nearest rank
    (stats.rs:75); None when empty."""
    if not sorted_values:
        return None
    rank = max(1, -(-len(sorted_values) * percent // 100))
    return sorted_values[rank - 1]


def median(values):
    return nearest_rank(sorted(values), 50)


@dataclasses.dataclass
class Frame:
    span_us: float
    passes_us: float
    encode_us: float
    pairs: int


def run_frame(variant: Variant, passes: int, *, stream, sink=None, groups: int = 1,
              kernels=None) -> Frame:
    """One frame of one cell (``bl_pass_cost_frame_run``)."""
    from .ops import _stream_ptr
    a = N.PassCostArgs(variant=variant.code, passes=passes, every=variant.k, groups=groups,
                       sink=None if sink is None else sink.data_ptr(),
                       kernels=None if kernels is None else kernels._h,
                       stream=_stream_ptr(stream))
    f = N.PassCostFrame()
    N.check(N.lib().bl_pass_cost_frame_run(ctypes.byref(a), ctypes.byref(f)))
    return Frame(f.span_us, f.passes_us, f.encode_us, f.pairs)


def run(passes=DEFAULT_PASSES, variants=DEFAULT_VARIANTS, *, frames_per_cell: int = 100,
        period_us: int = 16667, groups: int = 1, kernels=None, stream=None) -> dict:
    """Every cell, interleaved frame by frame after one untimed round; returns
    {(variant name, P): [Frame, ...]}."""
    import torch
    stream = stream or torch.cuda.Stream()
    if kernels is not None and max(passes) > len(kernels):
        raise ValueError("the program has %d kernels; a pass count of %d needs that many"
                         % (len(kernels), max(passes)))
    sink = None
    if kernels is None:
        if not 1 <= groups <= MAX_GROUPS:
            raise ValueError("groups must be in 1..=%d" % MAX_GROUPS)
        sink = torch.zeros(groups, dtype=torch.int32, device="cuda")
    cells = [(v, p) for v in variants for p in passes]
    out = {(v.name, p): [] for v, p in cells}
    start = time.perf_counter()
    for n in range(len(cells) * (frames_per_cell + 1)):
        if period_us > 0:
            wait = start + n * period_us * 1e-6 - time.perf_counter()
            if wait > 0:
                time.sleep(wait)
        v, p = cells[n % len(cells)]
        f = run_frame(v, p, stream=stream, sink=sink, groups=groups, kernels=kernels)
        if n >= len(cells):  # the first round pays for first use
            out[(v.name, p)].append(f)
    return out


def derive(frames: dict, trivial: bool = True) -> dict:
    """The derived figures of the module documentation, from the medians."""
    span = {c: median([f.span_us for f in fs]) for c, fs in frames.items() if fs}
    enc = {c: median([f.encode_us for f in fs]) for c, fs in frames.items() if fs}
    names = sorted({c[0] for c in span})
    counts = sorted({c[1] for c in span})
    d = {}
    for v in names:
        for p in counts:
            if p <= 1 or (v, p) not in span:
                continue
            row = {}
            if trivial and (v, 1) in span:
                key = "per_dispatch_us" if v.startswith("one-pass") else "per_pass_us"
                row[key] = (span[(v, p)] - span[(v, 1)]) / (p - 1)
                row["encode_per_pass_us"] = (enc[(v, p)] - enc[(v, 1)]) / (p - 1)
            if not v.startswith("one-pass") and ("one-pass", p) in span:
                row["over_one_pass_us"] = (span[(v, p)] - span[("one-pass", p)]) / (p - 1)
            if v == "per-pass" and ("ends", p) in span:
                row["over_ends_us"] = (span[(v, p)] - span[("ends", p)]) / (p - 1)
            if v == "per-pass":
                row["between_us"] = median([f.span_us - f.passes_us for f in frames[(v, p)]])
            d["[%s,%d]" % (v, p)] = row
    return {"span_us": {"[%s,%d]" % c: s for c, s in span.items()}, "derived": d}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--kernels", choices=["trivial", "encoder"], default="trivial")
    ap.add_argument("--passes", default=",".join(map(str, DEFAULT_PASSES)))
    ap.add_argument("--variants", default=",".join(v.name for v in DEFAULT_VARIANTS))
    ap.add_argument("--frames", type=int, default=100, help="timed frames per cell")
    ap.add_argument("--period-us", type=int, default=16667)
    ap.add_argument("--groups", type=int, default=1)
    a = ap.parse_args(argv)
    passes = [int(x) for x in a.passes.split(",")]
    variants = [Variant.parse(x) for x in a.variants.split(",")]
    kernels, config = None, {"kernels": a.kernels, "groups": a.groups}
    if a.kernels == "encoder":
        import numpy as np
        import torch
        from .model import Encoder, ViTConfig, block_weights_normal
        cfg = ViTConfig.small()
        rng = np.random.default_rng(0)
        n = lambda *s: rng.standard_normal(int(np.prod(s)), dtype=np.float32) * 0.02
        w = {"blocks": [block_weights_normal(rng, cfg.dim, cfg.mlp) for _ in range(cfg.layers)],
             "patch_w": n(cfg.patch, cfg.patch, cfg.cin, cfg.dim), "patch_b": n(cfg.dim),
             "cls": n(cfg.dim), "pos": n(cfg.tokens, cfg.dim),
             "norm_g": np.ones(cfg.dim, np.float32), "norm_b": np.zeros(cfg.dim, np.float32)}
        enc = Encoder(cfg, w, "bf16", planned_frames=1)
        buf = enc.buffers(1)
        buf.image.copy_(torch.from_numpy(rng.random(tuple(buf.image.shape), dtype=np.float32)))
        kernels = enc.program(1)
        config = {"kernels": "encoder ViT-S 518, 1 frame (first P of %d kernels)" % len(kernels)}
    res = run(passes, variants, frames_per_cell=a.frames, period_us=a.period_us,
              groups=a.groups, kernels=kernels)
    out = derive(res, trivial=a.kernels == "trivial")
    out["config"] = dict(config, passes=passes, variants=[v.name for v in variants],
                         frames_per_cell=a.frames, period_us=a.period_us)
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
