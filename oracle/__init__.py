"""CPU oracle for the ViT attention hot path: TEST INFRASTRUCTURE ONLY.

A C restatement (``oracle.c``) of the reference's f64-accumulating CPU
operations in ``crates/beatlm-bench/src/reference.rs`` of ynishi/beatlm, with
numpy wrappers. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``
(its ``cpu_baseline`` leg and ``--impl reference`` arm) import this package, as
the checker; the product library ``beatlm_b200`` never does.

Pinning: the reference is Rust and cannot be built here, so this restatement
is pinned by the reference's own known-answer tests (``reference.rs:723-837``),
transcribed in ``tests/golden/reference_kats.json``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "liboracle.so")
_lock = threading.Lock()
_lib = None

F32P = ctypes.POINTER(ctypes.c_float)


def build(force: bool = False) -> str:
    """Compiles ``oracle.c`` into ``liboracle.so`` beside it (gcc, OpenMP)."""
    src = os.path.join(_HERE, "oracle.c")
    if (not force and os.path.exists(_SO)
            and os.path.getmtime(_SO) >= max(os.path.getmtime(src),
                                             os.path.getmtime(os.path.join(_HERE, "oracle.h")))):
        return _SO
    tmp = _SO + ".tmp%d" % os.getpid()
    cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-fno-fast-math", "-o", tmp, src, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, _SO)
    return _SO


class BlockWeights(ctypes.Structure):
    _fields_ = [(n, F32P) for n in (
        "norm1_g", "norm1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "ls1",
        "norm2_g", "norm2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "ls2")]


ROUND_FN = ctypes.CFUNCTYPE(None, F32P, ctypes.c_size_t, ctypes.c_void_p)


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_SO)
            sz, f, i, d = ctypes.c_size_t, ctypes.c_float, ctypes.c_int, ctypes.c_double
            L.orc_uniform.argtypes = [ctypes.c_uint64, sz, f, f, F32P]
            L.orc_normal.argtypes = [ctypes.c_uint64, sz, f, f, F32P]
            L.orc_layernorm.argtypes = [F32P, F32P, F32P, sz, sz, f, i, F32P]
            L.orc_matmul.argtypes = [F32P, F32P, F32P, sz, sz, sz, i, F32P]
            L.orc_add.argtypes = [F32P, F32P, sz, F32P]
            L.orc_scale.argtypes = [F32P, sz, f, F32P]
            L.orc_erf.argtypes = [d]
            L.orc_erf.restype = d
            L.orc_gelu_erf.argtypes = [F32P, sz, F32P]
            L.orc_channel_scale.argtypes = [F32P, F32P, sz, sz, F32P]
            L.orc_patch_embed.argtypes = [F32P, F32P, F32P, sz, sz, sz, sz, sz, i, F32P]
            L.orc_prepend_token.argtypes = [F32P, F32P, sz, sz, F32P]
            L.orc_tokens_to_map.argtypes = [F32P, sz, sz, F32P]
            L.orc_attention_scores.argtypes = [F32P, sz, sz, sz, i, F32P]
            L.orc_softmax.argtypes = [F32P, sz, sz, i, F32P]
            L.orc_attention_values.argtypes = [F32P, F32P, sz, sz, sz, i, F32P]
            L.orc_attention_rows.argtypes = [F32P, sz, sz, sz, f, sz, sz, sz, sz, i, F32P]
            L.orc_vit_block.argtypes = [F32P, ctypes.POINTER(BlockWeights), sz, sz, sz, sz, f, i,
                                        ctypes.c_void_p, ctypes.c_void_p, F32P]
            L.orc_conv3x3.argtypes = [F32P, F32P, F32P, sz, sz, sz, sz, sz, i, F32P]
            L.orc_conv1x1.argtypes = [F32P, F32P, F32P, sz, sz, sz, i, F32P]
            L.orc_conv_transpose.argtypes = [F32P, F32P, F32P, sz, sz, sz, sz, sz, i, F32P]
            L.orc_resize_bilinear.argtypes = [F32P, sz, sz, sz, sz, sz, F32P]
            L.orc_round_f16.argtypes = [F32P, sz, ctypes.c_void_p]
            L.orc_round_bf16.argtypes = [F32P, sz, ctypes.c_void_p]
            L.orc_round_qkv_bf16.argtypes = [F32P, sz, ctypes.c_void_p]
            L.orc_round_qkv_f16.argtypes = [F32P, sz, ctypes.c_void_p]
            _lib = L
    return _lib


def _p(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(F32P)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def default_threads() -> int:
    return os.cpu_count() or 1


# ------------------------------------------------------------------ data

def uniform(seed: int, count: int, low: float, high: float) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib().orc_uniform(seed, count, low, high, _p(out))
    return out


def normal(seed: int, count: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib().orc_normal(seed, count, mean, std, _p(out))
    return out


# ------------------------------------------------------------------ ops

def layernorm(x, gamma, beta, eps, threads=None):
    x, gamma, beta = _f32(x), _f32(gamma), _f32(beta)
    c = gamma.size
    out = np.empty_like(x)
    lib().orc_layernorm(_p(x), _p(gamma), _p(beta), x.size // c, c, eps,
                        threads or default_threads(), _p(out))
    return out


def matmul(a, b, bias, m, k, n, threads=None):
    a, b = _f32(a), _f32(b)
    bias = None if bias is None else _f32(bias)
    out = np.empty(m * n, np.float32)
    lib().orc_matmul(_p(a), _p(b), _p(bias), m, k, n, threads or default_threads(), _p(out))
    return out


def add(a, b):
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    lib().orc_add(_p(a), _p(b), a.size, _p(out))
    return out


def scale(x, factor):
    x = _f32(x)
    out = np.empty_like(x)
    lib().orc_scale(_p(x), x.size, factor, _p(out))
    return out


def erf(x: float) -> float:
    return lib().orc_erf(x)


def gelu_erf(x):
    x = _f32(x)
    out = np.empty_like(x)
    lib().orc_gelu_erf(_p(x), x.size, _p(out))
    return out


def channel_scale(x, s):
    x, s = _f32(x), _f32(s)
    out = np.empty_like(x)
    lib().orc_channel_scale(_p(x), _p(s), x.size, s.size, _p(out))
    return out


def patch_embed(image, w, bias, gh, gw, p, cin, cout, threads=None):
    image, w = _f32(image), _f32(w)
    bias = None if bias is None else _f32(bias)
    out = np.empty(gh * gw * cout, np.float32)
    lib().orc_patch_embed(_p(image), _p(w), _p(bias), gh, gw, p, cin, cout,
                          threads or default_threads(), _p(out))
    return out


def prepend_token(token, tokens):
    token, tokens = _f32(token), _f32(tokens)
    c = token.size
    out = np.empty(token.size + tokens.size, np.float32)
    lib().orc_prepend_token(_p(token), _p(tokens), tokens.size // c, c, _p(out))
    return out


def tokens_to_map(x, channels):
    x = _f32(x)
    out = np.empty(x.size - channels, np.float32)
    lib().orc_tokens_to_map(_p(x), x.size // channels, channels, _p(out))
    return out


def attention_scores(qkv, t, h, d, threads=None):
    qkv = _f32(qkv)
    out = np.empty(t * h * t, np.float32)
    lib().orc_attention_scores(_p(qkv), t, h, d, threads or default_threads(), _p(out))
    return out


def softmax(x, cols, threads=None):
    x = _f32(x)
    out = np.empty_like(x)
    lib().orc_softmax(_p(x), x.size // cols, cols, threads or default_threads(), _p(out))
    return out


def attention_values(probs, qkv, t, h, d, threads=None):
    probs, qkv = _f32(probs), _f32(qkv)
    out = np.empty(t * h * d, np.float32)
    lib().orc_attention_values(_p(probs), _p(qkv), t, h, d, threads or default_threads(),
                               _p(out))
    return out


def attention(qkv, t, h, d, scale_=None, rows=None, heads=None, threads=None):
    """The scores -> scale -> softmax -> values chain, row-streamed.

    ``qkv`` is packed ``[t][3][h][d]``; the result is ``[rows][h * d]`` for
    query rows ``rows = (begin, end)`` (all by default); heads outside
    ``heads = (begin, end)`` are left zero."""
    qkv = _f32(qkv)
    r0, r1 = rows or (0, t)
    h0, h1 = heads or (0, h)
    if scale_ is None:
        scale_ = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    out = np.zeros((r1 - r0) * h * d, np.float32)
    lib().orc_attention_rows(_p(qkv), t, h, d, scale_, r0, r1, h0, h1,
                             threads or default_threads(), _p(out))
    return out


WEIGHT_NAMES = ("norm1_g", "norm1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "ls1",
                "norm2_g", "norm2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "ls2")


def vit_block(x, weights: dict, t, h, d, mlp, eps=1e-6, qkv_round=None, threads=None):
    """``reference.rs:520-544``. ``qkv_round`` models 16-bit storage of the
    packed projection that attention reads: None (f32, the reference), "f16" /
    "bf16" (all of it), "qk_bf16" / "qk_f16" (Q and K in that type, V in f16:
    the backend's packed layout)."""
    x = _f32(x)
    keep = {k: _f32(weights[k]) for k in WEIGHT_NAMES}
    bw = BlockWeights(**{k: _p(v) for k, v in keep.items()})
    out = np.empty_like(x)
    L = lib()
    width = ctypes.c_size_t(h * d)
    fn = {None: None, "f16": ctypes.cast(L.orc_round_f16, ctypes.c_void_p),
          "bf16": ctypes.cast(L.orc_round_bf16, ctypes.c_void_p),
          "qk_bf16": ctypes.cast(L.orc_round_qkv_bf16, ctypes.c_void_p),
          "qk_f16": ctypes.cast(L.orc_round_qkv_f16, ctypes.c_void_p)}[qkv_round]
    L.orc_vit_block(_p(x), ctypes.byref(bw), t, h, d, mlp, eps, threads or default_threads(),
                    fn, ctypes.cast(ctypes.byref(width), ctypes.c_void_p), _p(out))
    return out


def encoder_frame(image, w, grid, patch, cin, dim, heads, mlp, eps, out_indices, layers=None,
                  qkv_round=None, threads=None):
    """One frame of the DA-V2 ViT encoder graph
    (crates/beatlm/src/model/depth_anything_v2.rs:435-545) evaluated op by op
    in program order, as the reference's interpreter ``run``
    (crates/beatlm-bench/src/reference.rs:552-625) evaluates it: PatchEmbed,
    PrependToken (class token), Add (position embedding), the blocks
    (``vit_block``, reference.rs:520-544) and, after each block in
    ``out_indices``, the final LayerNorm and TokensToMap.

    ``image`` NHWC f32 [grid*patch][grid*patch][cin]; ``w``: ``patch_w``
    (HWIO), ``patch_b``, ``cls``, ``pos`` [tokens][dim], ``norm_g``/``norm_b``
    and ``blocks`` (per-block dicts of ``WEIGHT_NAMES``). Returns the feature
    maps, [grid*grid][dim] f32 each, in ``out_indices`` order."""
    layers = len(w["blocks"]) if layers is None else layers
    t = grid * grid + 1
    x = patch_embed(image, w["patch_w"], w["patch_b"], grid, grid, patch, cin, dim,
                    threads=threads)
    x = add(prepend_token(w["cls"], x), w["pos"])
    feats = []
    for i in range(layers):
        x = vit_block(x, w["blocks"][i], t, heads, dim // heads, mlp, eps, qkv_round=qkv_round,
                      threads=threads)
        if (i + 1) in out_indices:
            feats.append(tokens_to_map(layernorm(x, w["norm_g"], w["norm_b"], eps,
                                                 threads=threads), dim))
    return feats


def round_f16(x):
    x = np.array(x, dtype=np.float32, copy=True)
    lib().orc_round_f16(_p(x), x.size, None)
    return x


def round_bf16(x):
    x = np.array(x, dtype=np.float32, copy=True)
    lib().orc_round_bf16(_p(x), x.size, None)
    return x


# ------------------------------------------------------------- DPT decoder
# crates/beatlm-bench/src/reference.rs:25-230: NHWC maps, HWIO weights.

def conv3x3(x, w, bias, h, wd, cin, cout, stride=1, threads=None):
    x, w = _f32(x), _f32(w)
    bias = None if bias is None else _f32(bias)
    oh, ow = (h - 1) // stride + 1, (wd - 1) // stride + 1
    out = np.empty(oh * ow * cout, np.float32)
    lib().orc_conv3x3(_p(x), _p(w), _p(bias), h, wd, cin, cout, stride,
                      threads or default_threads(), _p(out))
    return out


def conv1x1(x, w, bias, pixels, cin, cout, threads=None):
    x, w = _f32(x), _f32(w)
    bias = None if bias is None else _f32(bias)
    out = np.empty(pixels * cout, np.float32)
    lib().orc_conv1x1(_p(x), _p(w), _p(bias), pixels, cin, cout, threads or default_threads(),
                      _p(out))
    return out


def conv_transpose(x, w, bias, h, wd, cin, cout, f, threads=None):
    x, w = _f32(x), _f32(w)
    bias = None if bias is None else _f32(bias)
    out = np.empty(h * f * wd * f * cout, np.float32)
    lib().orc_conv_transpose(_p(x), _p(w), _p(bias), h, wd, cin, cout, f,
                             threads or default_threads(), _p(out))
    return out


def resize_bilinear(x, ih, iw, oh, ow, c):
    x = _f32(x)
    out = np.empty(oh * ow * c, np.float32)
    lib().orc_resize_bilinear(_p(x), ih, iw, oh, ow, c, _p(out))
    return out


def relu(x):
    """reference.rs relu: max(x, 0) elementwise."""
    return np.maximum(_f32(x), np.float32(0))


def residual_unit(x, w1, b1, w2, b2, h, wd, c):
    """reference.rs:190-201: x + conv2(relu(conv1(relu(x))))."""
    first = conv3x3(relu(x), w1, b1, h, wd, c, c)
    second = conv3x3(relu(first), w2, b2, h, wd, c, c)
    return add(second, x)


def dpt_head(grid, patch, dim, neck, reassemble, fusion, head, w, feats, threads=None):
    """The DPT head of model/depth_anything_v2.rs:680-982 through the oracle's
    operations (f64 per op): reassembly (1x1, then ConvTranspose up / 3x3
    stride down / nothing), 3x3 to the fusion width without bias, fusion layers
    deepest first, the head. `w` holds HWIO weights by role (as
    beatlm_b200.model.decoder_weights_random makes them); returns the depth
    map [grid*patch]^2."""
    g, F = grid, fusion

    def unit(x, u, s):
        first = conv3x3(relu(x), u["w1"], u["b1"], s, s, F, F, threads=threads)
        return add(conv3x3(relu(first), u["w2"], u["b2"], s, s, F, F, threads=threads), x)

    maps = []
    for feat, c, rs, st in zip(feats, neck, reassemble, w["stages"]):
        x = conv1x1(feat, st["proj_w"], st["proj_b"], g * g, dim, c, threads=threads)
        side = g
        if rs[0] == "up":
            x = conv_transpose(x, st["resize_w"], st["resize_b"], g, g, c, c, rs[1], threads=threads)
            side = g * rs[1]
        elif rs[0] == "down":
            x = conv3x3(x, st["resize_w"], st["resize_b"], g, g, c, c, rs[1], threads=threads)
            side = (g - 1) // rs[1] + 1
        maps.append((conv3x3(x, st["neck_w"], None, side, side, c, F, threads=threads), side))
    fused, side = None, None
    for layer, (stage, s) in enumerate(reversed(maps)):
        nxt = len(maps) - 2 - layer
        out = maps[nxt][1] if nxt >= 0 else 2 * s
        f = w["fusion"][layer]
        x = stage if fused is None else add(unit(stage, f["unit1"], s), fused)
        x = unit(x, f["unit2"], s)
        x = resize_bilinear(x, s, s, out, out, F)
        fused = conv1x1(x, f["proj_w"], f["proj_b"], out * out, F, F, threads=threads)
        side = out
    h, o = w["head"], g * patch
    x = conv3x3(fused, h["w1"], h["b1"], side, side, F, F // 2, threads=threads)
    x = resize_bilinear(x, side, side, o, o, F // 2)
    x = relu(conv3x3(x, h["w2"], h["b2"], o, o, F // 2, head, threads=threads))
    return relu(conv1x1(x, h["w3"], h["b3"], o * o, head, 1, threads=threads))
