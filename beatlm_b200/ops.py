"""Host-side calls of the fused kernels on device buffers.

Torch tensors serve only as device memory and streams. Every op has two forms:
``*_args(...)`` packs the C-ABI argument struct (for a prebuilt program, see
``runtime.Kernels``), and the plain call packs and launches at once.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from . import _native as N

_TD = {"f32": N.BL_F32, "f16": N.BL_F16, "bf16": N.BL_BF16}
ACT = {None: 0, "none": 0, "relu": 1, "gelu_tanh": 2, "gelu_erf": 3}


def _stream_ptr(stream):
    """A cudaStream_t for the C ABI: a torch stream, a raw handle (int), or
    None for torch's current stream."""
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _dt(t):
    import torch
    return {torch.float32: N.BL_F32, torch.float16: N.BL_F16, torch.bfloat16: N.BL_BF16}[t.dtype]


def pack_qkv(qkv, qk_dtype: str = "f16", device="cuda"):
    """Packs f32 ``[..., tokens, 3, heads, head_dim]`` values into one 16-bit
    device buffer: the Q and K sections in ``qk_dtype`` ("f16" or "bf16"), the
    V section in f16, the layout the attention kernel reads."""
    import torch
    a = torch.as_tensor(np.ascontiguousarray(qkv, dtype=np.float32))
    qk = a[..., :2, :, :].to(torch.bfloat16 if qk_dtype == "bf16" else torch.float16)
    v = a[..., 2:, :, :].to(torch.float16)
    out = torch.empty(a.shape, dtype=torch.int16)
    out[..., :2, :, :] = qk.view(torch.int16)
    out[..., 2:, :, :] = v.view(torch.int16)
    return out.to(device)


# ------------------------------------------------------------------ attention

def attention_args(qkv, *, tokens, heads, out, head_dim=64, batch=1, qk_dtype="f16",
                   out_dtype=None, scale=None, rows=None, head_range=None, out_head_base=0,
                   qkv_row_stride=0, out_row_stride=None, workspace=None, kv_splits=0,
                   trace=None, query_tiles=0):
    """``kv_splits`` 0 picks the key-split count. Without ``workspace`` the
    splits of a query group combine in distributed shared memory (a cluster);
    with one (a zero-filled device buffer of at least
    ``attention_workspace_bytes`` bytes) they combine through it.
    ``query_tiles``: 128-row query tiles per CTA (1 or 2; 0 picks).
    ``trace``: optional int64 device buffer for 8 timestamps per CTA."""
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    r0, r1 = rows or (0, tokens)
    h0, h1 = head_range or (0, heads)
    odt = _TD[out_dtype] if out_dtype is not None else _dt(out)
    return N.AttentionArgs(batch=batch, tokens=tokens, heads=heads, head_dim=head_dim,
                           head_begin=h0, head_end=h1, row_begin=r0, row_end=r1, scale=scale,
                           qk_dtype=_TD[qk_dtype], v_dtype=N.BL_F16, out_dtype=odt,
                           qkv=qkv.data_ptr(), qkv_row_stride=qkv_row_stride,
                           out=out.data_ptr(),
                           out_row_stride=out.shape[-1] if out_row_stride is None
                           else out_row_stride, out_head_base=out_head_base,
                           kv_splits=kv_splits,
                           workspace=None if workspace is None else workspace.data_ptr(),
                           workspace_bytes=0 if workspace is None else workspace.numel(),
                           trace=None if trace is None else trace.data_ptr(),
                           query_tiles=query_tiles)


def attention_workspace_bytes(args) -> int:
    """Bytes of workspace ``bl_attention`` wants for these arguments (with
    ``kv_splits`` 0 it reports what the automatic choice would use)."""
    return N.lib().bl_attention_workspace_bytes(ctypes.byref(args))


def attention_choice(args) -> tuple[int, int, int]:
    """(query tiles per CTA, key splits, unsplit query groups) ``bl_attention``
    takes for ``args`` (the last nonzero for a mixed grid: that many groups
    unsplit, the rest split)."""
    qt, sp, un = ctypes.c_uint32(0), ctypes.c_uint32(0), ctypes.c_uint32(0)
    N.check(N.lib().bl_attention_choice(ctypes.byref(args), ctypes.byref(qt), ctypes.byref(sp),
                                        ctypes.byref(un)))
    return qt.value, sp.value, un.value


def attention_workspace(nbytes: int, device="cuda"):
    """A zero-filled, 256-byte-aligned device workspace (torch allocations are
    256-byte aligned)."""
    import torch
    return torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def attention(qkv, *, tokens: int, heads: int, head_dim: int = 64, batch: int = 1,
              qk_dtype: str = "f16", out=None, out_dtype: str = "f32", scale: float | None = None,
              rows: tuple[int, int] | None = None, head_range: tuple[int, int] | None = None,
              out_head_base: int = 0, stream=None, workspace=None, kv_splits: int = 0,
              query_tiles: int = 0):
    """The fused scores -> scale -> softmax -> values chain of one layer
    (reference kernel.rs:722-777) on packed ``[batch][tokens][3][heads][64]``
    16-bit ``qkv``; returns ``out`` ``[batch][tokens][heads * 64]``."""
    import torch
    h0, h1 = head_range or (0, heads)
    width = (h1 - out_head_base) * head_dim if head_range else heads * head_dim
    if out is None:
        tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[out_dtype]
        out = torch.zeros((batch, tokens, width), dtype=tdt, device=qkv.device)
        odt = None
    else:  # a float tensor's own type decides; a 16-bit container takes out_dtype
        odt = None if out.dtype.is_floating_point else out_dtype
    a = attention_args(qkv, tokens=tokens, heads=heads, out=out, head_dim=head_dim, batch=batch,
                       qk_dtype=qk_dtype, out_dtype=odt, scale=scale, rows=rows,
                       head_range=head_range, out_head_base=out_head_base,
                       workspace=workspace, kv_splits=kv_splits, query_tiles=query_tiles)
    N.check(N.lib().bl_attention(ctypes.byref(a), _stream_ptr(stream)))
    return out


# ------------------------------------------------------------------ linear

def gemm_args(w, *, a=None, ln=None, bias=None, act=None, scale=None, chan_scale=None,
              residual=None, res_period=0, out, out_dtype=None, out_split=None, m=None,
              out_row_offset=0, out_group=(0, 0), tile_n=0, stats_out=None, ln_stats=None,
              norm=None, norm_sync=None, weights_static=False, pair_tiles=0, split_k=0,
              stream_k=0, workspace=None, dot=None):
    """``stats_out``: a float32 ``[rows][parts][2]`` tensor the epilogue fills
    with per-slice (mean, M2) of each stored row (``parts`` = n / tile width).
    ``ln_stats``: such a tensor for ``ln``'s input, used instead of a pass
    over its rows. ``norm=(gamma, beta, eps, out)``: the epilogue also writes
    LayerNorm of every stored f32 row to the 16-bit ``out``; ``norm_sync`` is
    its zero-filled exchange buffer (``gemm_norm_sync_bytes``).
    ``weights_static``: ``w``, ``bias`` and ``chan_scale`` are not written by
    the kernel launched just before on the stream (model weights), so the
    GEMM may fetch them while that kernel finishes. ``pair_tiles=2``: 256-row
    tiles over CTA pairs (``bl_gemm_args.pair_tiles``); ``split_k``: the K
    split over a two-CTA cluster (0 automatic, 1 off, 2 on). ``stream_k=2``:
    tiles' k-stages cut into pieces dealt over the SMs (0 or 1: whole
    tiles); ``workspace``: its zero-filled device tensor of at least
    ``gemm_workspace_bytes(args)`` bytes, which each launch leaves
    zero-filled. ``dot=(w, bias, relu)``: each finished row reduced to
    one f32 value, relu(sum_c row[c] w[c] + bias) when relu, written to
    ``out`` (an f32 tensor of m values) in place of the row
    (``bl_gemm_args.dot_w``)."""
    import torch
    n, k = w.shape
    ab = {torch.float16: "f16", torch.bfloat16: "bf16"}[w.dtype]
    if ln is not None:
        x, gamma, beta, eps = ln
        m = x.shape[0] if m is None else m
    else:
        m = a.shape[0] if m is None else m
    odt = _TD[out_dtype] if out_dtype is not None else _dt(out)
    g = N.GemmArgs(m=m, n=n, k=k, ab_dtype=_TD[ab], a=_ptr(a),
                   lda=0 if a is None else a.stride(0), b=w.data_ptr(), ldb=w.stride(0),
                   act=ACT[act], scale=0.0 if scale is None else scale,
                   bias=_ptr(bias), chan_scale=_ptr(chan_scale), residual=_ptr(residual),
                   res_dtype=N.BL_F32 if residual is None else _dt(residual),
                   res_ld=0 if residual is None else residual.stride(0), res_period=res_period,
                   out=out.data_ptr(), out_dtype=odt, out_ld=out.stride(0),
                   out_row_offset=out_row_offset, out_group_rows=out_group[0],
                   out_group_gap=out_group[1], tile_n=tile_n,
                   weights_static=1 if weights_static else 0, pair_tiles=pair_tiles,
                   split_k=split_k, stream_k=stream_k)
    if dot is not None:
        dw, db, drelu = dot
        if (dw.dtype != torch.float32 or not dw.is_contiguous() or dw.numel() != n
                or out.dtype != torch.float32 or out.numel() != m or not out.is_contiguous()):
            raise ValueError("gemm_args: a row reduction takes f32 weights of n values and an "
                             "f32 output of m values")
        g.dot_w, g.dot_bias, g.dot_act = dw.data_ptr(), float(db), 1 if drelu else 0
        g.out_ld = 0  # m values, not rows
    if workspace is not None:
        g.workspace = workspace.data_ptr()
        g.workspace_bytes = workspace.numel() * workspace.element_size()
    if out_split is not None:
        g.split_col, g.out_dtype_hi = out_split[0], _TD[out_split[1]]
    if ln is not None:
        g.ln_x, g.ln_ldx, g.ln_gamma, g.ln_beta, g.ln_eps = (x.data_ptr(), x.stride(0),
                                                             gamma.data_ptr(), beta.data_ptr(),
                                                             eps)
    if stats_out is not None:
        g.stats_out, g.stats_parts = stats_out.data_ptr(), stats_out.shape[1]
    if ln_stats is not None:
        g.ln_stats, g.ln_stats_parts = ln_stats.data_ptr(), ln_stats.shape[1]
    if norm is not None:
        gamma, beta, eps, nout = norm
        g.norm_out, g.norm_out_dtype, g.norm_out_ld = nout.data_ptr(), _dt(nout), nout.stride(0)
        g.norm_gamma, g.norm_beta, g.norm_eps = gamma.data_ptr(), beta.data_ptr(), eps
        g.norm_sync, g.norm_sync_bytes = norm_sync.data_ptr(), norm_sync.numel()
    return g


def gemm_workspace_bytes(args) -> int:
    """Bytes of workspace the stream-K form needs for these ``gemm_args``
    (0 where the launch keeps whole tiles; ``bl_gemm_workspace_bytes``)."""
    return int(N.lib().bl_gemm_workspace_bytes(ctypes.byref(args)))


def gemm_norm_sync_bytes(m: int, n: int) -> int:
    """Bytes of the exchange buffer of an epilogue LayerNorm over m rows of
    n columns (``bl_gemm_norm_sync_bytes``)."""
    return int(N.lib().bl_gemm_norm_sync_bytes(ctypes.byref(N.GemmArgs(m=m, n=n))))


def linear(w, *, stream=None, **kw):
    """``out = epilogue(A . w^T)`` on the tensor cores (``bl_gemm``).

    ``w`` is the 16-bit weight ``[n][k]`` (f16 or bf16; A is converted to the
    same type); A is the 16-bit ``a`` ``[m][k]`` or, with
    ``ln=(x, gamma, beta, eps)``, LayerNorm of the f32 rows ``x`` computed
    inside the kernel. ``out_dtype`` defaults to ``out``'s own type;
    ``out_split=(col, dtype)`` stores columns from ``col`` on as ``dtype``
    (the f16 V part of packed Q|K|V rows). ``stats_out`` / ``ln_stats``:
    per-row partial LayerNorm statistics written by this GEMM's epilogue /
    consumed by its LayerNorm prologue (``gemm_args``)."""
    g = gemm_args(w, **kw)
    N.check(N.lib().bl_gemm(ctypes.byref(g), _stream_ptr(stream)))
    return kw["out"]


# ------------------------------------------------------------------ others

def layernorm_args(x, gamma, beta, eps, *, out, rows=None, in_row_offset=0, in_group=(0, 0)):
    rows = out.shape[0] if rows is None else rows
    return N.LayerNormArgs(rows=rows, cols=x.shape[1], x=x.data_ptr(), ldx=x.stride(0),
                           gamma=gamma.data_ptr(), beta=beta.data_ptr(), eps=eps,
                           out=out.data_ptr(), out_dtype=_dt(out), ldo=out.stride(0),
                           in_row_offset=in_row_offset, in_group_rows=in_group[0],
                           in_group_gap=in_group[1])


def layernorm(x, gamma, beta, eps, *, out, stream=None, **kw):
    a = layernorm_args(x, gamma, beta, eps, out=out, **kw)
    N.check(N.lib().bl_layernorm(ctypes.byref(a), _stream_ptr(stream)))
    return out


def patchify_args(image, *, frames, side, patch, cin, k_pad, a_out, a_dtype="bf16", cls=None,
                  pos=None, x=None):
    return N.PatchifyArgs(frames=frames, side=side, patch=patch, cin=cin, k_pad=k_pad,
                          dim=0 if cls is None else cls.numel(), image=image.data_ptr(),
                          a=a_out.data_ptr(), a_dtype=_TD[a_dtype], cls=_ptr(cls),
                          pos=_ptr(pos), x=_ptr(x))


def patchify(image, *, stream=None, **kw):
    a = patchify_args(image, **kw)
    N.check(N.lib().bl_patchify(ctypes.byref(a), _stream_ptr(stream)))
    return kw["a_out"]


# ------------------------------------------------------------------ DPT decoder
# The reference's Conv2d3x3 / Conv2d1x1 / ConvTranspose2d / ResizeBilinear main
# ops (crates/beatlm-core/src/kernel.rs:265-319, wgsl.rs:387-514; CPU
# definitions crates/beatlm-bench/src/reference.rs:25-175) on NHWC f32 maps:
# a convolution is bl_im2col into 16-bit rows then the tcgen05 GEMM.

def _round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


def conv_weights(hwio, ksize: int, cin: int, cout: int, dtype: str = "f16", device="cuda"):
    """HWIO weights [ks][ks][cin][cout] as the GEMM's [n_pad][k_pad] 16-bit
    matrix (row co holds column (ky ks + kx) cin + ci), zero-padded to a
    multiple of 32 rows and 64 columns."""
    import torch
    k = ksize * ksize * cin
    w = np.asarray(hwio, np.float32).reshape(k, cout).T
    m = np.zeros((_round_up(cout, 32), _round_up(k, 64)), np.float32)
    m[:cout, :k] = w
    td = torch.float16 if dtype == "f16" else torch.bfloat16
    return torch.from_numpy(m).to(td).to(device)


def im2col(x, h: int, w: int, cin: int, ksize: int = 3, stride: int = 1, relu: bool = False,
           k_pad: int | None = None, dtype: str = "f16", stream=None):
    """``bl_im2col``: the [oh * ow][k_pad] 16-bit rows of an NHWC map, f32 or
    already 16-bit of ``dtype`` (copied as it is)."""
    import torch
    pad = ksize // 2
    oh, ow = (h + 2 * pad - ksize) // stride + 1, (w + 2 * pad - ksize) // stride + 1
    k_pad = k_pad or _round_up(ksize * ksize * cin, 64)
    td = torch.float16 if dtype == "f16" else torch.bfloat16
    if x.dtype != torch.float32 and x.dtype != td:
        raise ValueError("im2col: the map is f32 or of the output dtype")
    out = torch.empty((oh * ow, k_pad), dtype=td, device=x.device)
    a = N.Im2colArgs(input=x.data_ptr(), h=h, w=w, cin=cin, ksize=ksize, stride=stride,
                     relu=1 if relu else 0, out=out.data_ptr(), out_dtype=_TD[dtype], k_pad=k_pad,
                     in_dtype=N.BL_F32 if x.dtype == torch.float32 else _TD[dtype])
    N.check(N.lib().bl_im2col(ctypes.byref(a), _stream_ptr(stream)))
    return out, oh, ow


def conv2d(x, weights, bias, h: int, w: int, cin: int, cout: int, *, ksize: int = 3,
           stride: int = 1, relu_input: bool = False, act=None, residual=None, stream=None,
           implicit: bool | None = None, split_k: int = 0, out_dtype: str = "f32",
           padded: bool = False, dot=None):
    """A 3x3 (zero padding 1) or 1x1 convolution of the NHWC f32 map ``x``:
    ``weights`` from ``conv_weights``, ``bias`` f32 [cout] or None, ``act``
    "relu" on the result, ``residual`` an f32 [oh * ow][cout] map added last
    (cout a multiple of 32). Returns f32 [oh * ow][cout]. ``x`` may also be a
    16-bit map of the weights' dtype (gathered without a rounding), and for a
    1x1 convolution the GEMM's 16-bit rows [h * w][k_pad]
    (``resize_bilinear_rows16``), multiplied as they are.

    ``implicit=True``: a 3x3 stride-1 convolution of a multiple of 32
    channels runs as an implicit GEMM (``bl_conv3x3``, the image read
    through the taps on chip, no gathered rows in memory; the same bits).
    By default the rows are gathered first (``bl_im2col``) and multiplied by
    the persistent ``bl_gemm``: measured faster on B200 at every DPT shape
    (148 x 148 x 64: 23 against 27 us; 518 x 518 x 32: 105 against 122 us),
    since the implicit kernel's f32 image tiles take about 1 us per TMA round
    trip, more than a three-stage ring hides, and are converted to 16 bits
    on chip for every tap. ``split_k``: as ``gemm_args`` (the gathered
    form's GEMM). ``out_dtype`` "f16" or "bf16": the result rounded once to
    16 bits in the epilogue (the bits a gather of the f32 result would
    store, for a map whose only reader is the next convolution). ``padded``:
    the result with all the weights' padded output channels (zeros), as
    [oh * ow][n_pad], which with 16 bits and n_pad = cout rounded up to 64 is
    the next 1x1 GEMM's rows. ``dot=(w, bias, relu)``: a 1x1 convolution to
    one channel after this one, in its epilogue (``w`` f32 [cout], cout at
    most 128 and a multiple of 32): returns f32 [oh * ow]."""
    import torch
    dt = "f16" if weights.dtype == torch.float16 else "bf16"
    rows16 = False
    if x.dtype in (torch.float16, torch.bfloat16):
        if x.dtype != weights.dtype or not x.is_contiguous() or implicit:
            raise ValueError("conv2d: a 16-bit map must be of the weights' dtype, contiguous, "
                             "and gathered (not implicit)")
        # the GEMM's rows already (resize_bilinear_rows16): a 1x1 convolution
        # of them is the GEMM alone; any other 16-bit map is gathered as it is
        rows16 = (ksize == 1 and stride == 1 and not relu_input
                  and tuple(x.shape) == (h * w, weights.shape[1]))
        if not rows16 and x.numel() != h * w * cin:
            raise ValueError("conv2d: a 16-bit map must be [h * w][cin], or for a 1x1 "
                             "convolution the GEMM's [h * w][k_pad] rows")
        implicit = False
    can = (ksize == 3 and stride == 1 and cin % 32 == 0 and x.dtype == torch.float32
           and x.is_contiguous() and x.data_ptr() % 16 == 0)
    if implicit is None:
        implicit = False
    elif implicit and not can:
        raise ValueError("conv2d: the implicit form takes 3x3, stride 1, channels a multiple of 32")
    if implicit:
        cols, oh, ow = None, h, w
    elif rows16:
        cols, oh, ow = x, h, w
    else:
        cols, oh, ow = im2col(x, h, w, cin, ksize, stride, relu_input, weights.shape[1], dt,
                              stream)
    n_pad = weights.shape[0]
    if residual is not None:
        if n_pad != cout:
            raise ValueError("conv2d: a residual needs cout a multiple of 32")
        residual = residual.reshape(oh * ow, cout)
    bias_pad = bias
    # The kernel reads the bias as n_pad f32 values of device memory: the
    # caller's tensor is used in place only when it is exactly that; anything
    # else (another dtype, a stride, host memory, cout padded) is copied into
    # a zero-padded f32 device vector.
    if bias is not None and not (bias.dtype == torch.float32 and bias.is_contiguous()
                                 and bias.device == x.device and bias.numel() == n_pad):
        bias_pad = torch.zeros(n_pad, dtype=torch.float32, device=x.device)
        bias_pad[:cout] = bias.reshape(-1)[:cout].to(device=x.device, dtype=torch.float32)
    otd = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[out_dtype]
    if dot is not None:
        if n_pad != cout or out_dtype != "f32":
            raise ValueError("conv2d: the one-channel 1x1 convolution after it takes cout a "
                             "multiple of 32 and an f32 result")
        out = torch.empty(oh * ow, dtype=torch.float32, device=x.device)
    else:
        out = torch.empty((oh * ow, n_pad), dtype=otd, device=x.device)
    g = gemm_args(weights, a=cols, m=oh * ow, bias=bias_pad, act=act, residual=residual,
                  out=out, split_k=split_k, dot=dot)
    if implicit:
        c = N.Conv3x3Args(input=x.data_ptr(), h=h, w=w, cin=cin, relu=1 if relu_input else 0)
        N.check(N.lib().bl_conv3x3(ctypes.byref(g), ctypes.byref(c), _stream_ptr(stream)))
    else:
        N.check(N.lib().bl_gemm(ctypes.byref(g), _stream_ptr(stream)))
    return out if n_pad == cout or padded or dot is not None else out[:, :cout].contiguous()


def conv_transpose_weights(hwio, cin: int, cout: int, f: int, dtype: str = "f16",
                           device="cuda"):
    """HWIO weights [f][f][cin][cout] of a transposed convolution as the GEMM's
    [(ky f + kx) cout + co][k_pad] 16-bit matrix (k_pad = cin rounded up to 64)."""
    import torch
    n = f * f * cout
    wt = np.asarray(hwio, np.float32).reshape(f * f, cin, cout).transpose(0, 2, 1).reshape(n, cin)
    m = np.zeros((n, _round_up(cin, 64)), np.float32)
    m[:, :cin] = wt
    td = torch.float16 if dtype == "f16" else torch.bfloat16
    return torch.from_numpy(m).to(td).to(device)


def conv_transpose(x, hwio, bias, h: int, w: int, cin: int, cout: int, f: int,
                   dtype: str = "f16", stream=None):
    """Transposed convolution of kernel = stride = f, no padding: one GEMM of
    each pixel by the [(ky f + kx) cout + co][ci] weights, then the f x f
    blocks scattered into the [h f][w f][cout] map with the bias. ``hwio`` is
    the HWIO array, or its device matrix from ``conv_transpose_weights``
    (which a CUDA graph capture needs: nothing then crosses from the host).
    ``x`` may also be 16-bit of ``dtype``: a map [h * w][cin] (gathered as it
    is), or the GEMM's rows [h * w][cin rounded up to 64] (used as they are,
    e.g. ``conv2d(..., out_dtype=dtype, padded=True)``)."""
    import torch
    n = f * f * cout
    if n % 32 != 0:
        raise ValueError("conv_transpose: f * f * cout must be a multiple of 32")
    k_pad = _round_up(cin, 64)
    if x.dtype != torch.float32 and tuple(x.shape) == (h * w, k_pad) and x.is_contiguous():
        if x.dtype != (torch.float16 if dtype == "f16" else torch.bfloat16):
            raise ValueError("conv_transpose: 16-bit rows must be of the weights' dtype")
        cols = x
    else:
        cols, _, _ = im2col(x, h, w, cin, 1, 1, False, None, dtype, stream)
    if isinstance(hwio, torch.Tensor) and hwio.dim() == 2:
        wdev = hwio
    else:
        wdev = conv_transpose_weights(hwio, cin, cout, f, dtype, x.device)
    blocks = torch.empty((h * w, n), dtype=torch.float32, device=x.device)
    g = gemm_args(wdev, a=cols, out=blocks)
    N.check(N.lib().bl_gemm(ctypes.byref(g), _stream_ptr(stream)))
    out = torch.empty((h * f * w * f, cout), dtype=torch.float32, device=x.device)
    N.check(N.lib().bl_blocks_to_map(blocks.data_ptr(), None if bias is None else bias.data_ptr(),
                                     out.data_ptr(), h, w, f, cout, _stream_ptr(stream)))
    return out


def conv1x1_one(x, w, bias: float, pixels: int, c: int, relu: bool = False, stream=None):
    """``bl_conv1x1_one``: one output channel of a 1x1 convolution of the
    NHWC f32 map ``x`` ([pixels][c]) by the f32 device vector ``w`` [c],
    plus ``bias``, ReLU when asked; returns f32 [pixels]."""
    import torch
    out = torch.empty(pixels, dtype=torch.float32, device=x.device)
    N.check(N.lib().bl_conv1x1_one(x.data_ptr(), w.data_ptr(), float(bias), out.data_ptr(),
                                   pixels, c, 1 if relu else 0, _stream_ptr(stream)))
    return out


def resize_bilinear(x, ih: int, iw: int, oh: int, ow: int, c: int, stream=None):
    """``bl_resize_bilinear``: corners aligned, f32 NHWC."""
    import torch
    out = torch.empty((oh * ow, c), dtype=torch.float32, device=x.device)
    N.check(N.lib().bl_resize_bilinear(x.data_ptr(), out.data_ptr(), ih, iw, oh, ow, c,
                                       _stream_ptr(stream)))
    return out


def resize_bilinear_rows16(x, ih: int, iw: int, oh: int, ow: int, c: int, ld: int | None = None,
                           dtype: str = "f16", stream=None):
    """``bl_resize_bilinear_rows16``: the resampling of ``resize_bilinear``
    written as 16-bit rows [oh * ow][ld] (channels past ``c`` zero), the
    operand ``conv2d`` takes for a 1x1 convolution without a gather."""
    import torch
    ld = c if ld is None else ld
    out = torch.empty((oh * ow, ld), dtype=torch.float16 if dtype == "f16" else torch.bfloat16,
                      device=x.device)
    N.check(N.lib().bl_resize_bilinear_rows16(x.data_ptr(), out.data_ptr(), ih, iw, oh, ow, c, ld,
                                              _TD[dtype], _stream_ptr(stream)))
    return out
