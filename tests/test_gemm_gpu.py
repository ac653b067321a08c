"""The tcgen05 GEMM (bl_gemm) against the oracle's matmul (reference.rs:273-298)
and its epilogue operations, through the C ABI.

The oracle receives the same 16-bit-rounded A and W values the tensor cores
read, so plain products differ only by f32 accumulation order: they must meet
the reference's own per-element tolerance |d| <= 1e-4 + 1e-4 |ref|
(reference.rs:17-24). With the LayerNorm prologue the normalised values are
computed in f32 on the GPU and in f64 in the oracle before both round to 16
bits, so a few elements round to neighbouring 16-bit values: there the bound
is relative L2 <= 1e-3 (bf16) / 2e-4 (f16)."""
import ctypes
import math

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

TOL_ABS, TOL_REL = 1e-4, 1e-4


def _dev(a, dtype):
    import torch
    td = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dtype]
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(td).cuda()


def _rnd(a, dtype):
    return oracle.round_bf16(a) if dtype == "bf16" else oracle.round_f16(a)


def _close(got, want, what):
    got = np.asarray(got, np.float32).ravel()
    want = np.asarray(want, np.float32).ravel()
    bad = np.abs(got - want) > TOL_ABS + TOL_REL * np.abs(want)
    assert not bad.any(), "%s: %d mismatches, first at %d: %r vs %r" % (
        what, bad.sum(), np.argmax(bad), got[np.argmax(bad)], want[np.argmax(bad)])


def _rel(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    return np.linalg.norm(got - want) / np.linalg.norm(want)


def _check_status():
    import beatlm_b200 as bl
    st = bl.status(reset=True)
    assert st.code == 0, hex(st.code)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("m,n,k,tile", [(1370, 1152, 384, 0), (1370, 384, 384, 32),
                                        (1370, 1536, 384, 128), (1370, 384, 1536, 32),
                                        (200, 192, 128, 96), (1, 64, 64, 64), (129, 128, 640, 64),
                                        (1370, 4096, 1024, 128), (2740, 1536, 384, 64),
                                        (1370, 3072, 1024, 256), (300, 512, 4096, 256),
                                        (1370, 4096, 1024, 0)])
def test_plain_gemm_with_bias(dtype, m, n, k, tile):
    """Shapes from one tile to several tiles per CTA of the persistent grid
    (1370 x 4096 at 128 columns: 352 tiles for 148 CTAs)."""
    import torch
    import beatlm_b200 as bl
    a = _rnd(oracle.normal(m + n, m * k), dtype)
    w = _rnd(oracle.uniform(k, k * n, -1 / math.sqrt(k), 1 / math.sqrt(k)), dtype)  # [in][out]
    b = oracle.uniform(n, n, -0.1, 0.1)
    out = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    bl.ops.linear(_dev(w.reshape(k, n).T, dtype), a=_dev(a.reshape(m, k), dtype),
                  bias=_dev(b, "f32"), out=out, tile_n=tile)
    torch.cuda.synchronize()
    _check_status()
    want = oracle.matmul(a, w, b, m, k, n)
    _close(out.cpu().numpy(), want, "gemm %dx%dx%d %s" % (m, n, k, dtype))


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("m,n,k,tile", [(1370, 384, 384, 0), (1370, 1024, 4096, 0),
                                        (1370, 1024, 1024, 256)])
def test_layerscale_residual_epilogue(dtype, m, n, k, tile):
    """x1 = x + ls * (A.W + b): ChannelScale then Add (reference.rs:379, 301),
    in place on the f32 residual stream (ViT-S proj; ViT-L fc2, more than one
    tile per CTA)."""
    import torch
    import beatlm_b200 as bl
    a = _rnd(oracle.normal(1, m * k), dtype)
    w = _rnd(oracle.uniform(2, k * n, -0.05, 0.05), dtype)
    b, ls = oracle.uniform(3, n, -0.1, 0.1), oracle.uniform(4, n, 0.1, 1.0)
    x = oracle.uniform(5, m * n, -2, 2)
    xd = _dev(x.reshape(m, n), "f32")
    bl.ops.linear(_dev(w.reshape(k, n).T, dtype), a=_dev(a.reshape(m, k), dtype),
                  bias=_dev(b, "f32"), chan_scale=_dev(ls, "f32"), residual=xd, out=xd,
                  tile_n=tile)
    torch.cuda.synchronize()
    _check_status()
    want = oracle.add(x, oracle.channel_scale(oracle.matmul(a, w, b, m, k, n), ls))
    _close(xd.cpu().numpy(), want, "layerscale+residual")


@pytest.mark.parametrize("tile", [0, 256])
def test_gelu_erf_epilogue_and_16bit_store(tile):
    import torch
    import beatlm_b200 as bl
    m, n, k = 300, 1536, 384
    a = _rnd(oracle.normal(6, m * k), "bf16")
    w = _rnd(oracle.uniform(7, k * n, -0.1, 0.1), "bf16")
    b = oracle.uniform(8, n, -0.1, 0.1)
    out = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    bl.ops.linear(_dev(w.reshape(k, n).T, "bf16"), a=_dev(a.reshape(m, k), "bf16"),
                  bias=_dev(b, "f32"), act="gelu_erf", out=out, tile_n=tile)
    torch.cuda.synchronize()
    _check_status()
    want = oracle.round_bf16(oracle.gelu_erf(oracle.matmul(a, w, b, m, k, n)))
    got = out.float().cpu().numpy().ravel()
    # one bf16 ulp of slack for values that sit on a rounding boundary
    assert np.all(np.abs(got - want) <= 2 ** -7 * np.abs(want) + 1e-4)
    assert _rel(got, want) < 2e-3


def test_gelu_erf_on_the_gpu_is_within_its_stated_error():
    """The reference's GPU test (vit.rs:175-199): GELU (erf) over [-10, 10] in
    steps of 2^-12 within GELU_ERF_MAX_ERROR = 5e-7 of GELU through f64 erf.
    The values enter as the bias of a zero product."""
    import torch
    import beatlm_b200 as bl
    grid = (-10.0 + np.arange(81921, dtype=np.float32) / np.float32(4096)).astype(np.float32)
    n = (grid.size + 127) // 128 * 128
    bias = np.zeros(n, np.float32)
    bias[:grid.size] = grid
    out = torch.zeros((1, n), dtype=torch.float32, device="cuda")
    bl.ops.linear(torch.zeros((n, 64), dtype=torch.float16, device="cuda"),
                  a=torch.zeros((1, 64), dtype=torch.float16, device="cuda"),
                  bias=_dev(bias, "f32"), act="gelu_erf", out=out, tile_n=128)
    torch.cuda.synchronize()
    got = out.cpu().numpy()[0, :grid.size].astype(np.float64)
    exact = np.array([0.5 * float(v) * (1.0 + oracle.erf(float(v) / math.sqrt(2.0)))
                      for v in grid])
    worst = float(np.max(np.abs(got - exact)))
    print("GELU (erf) on the GPU: max abs error %.3e" % worst)
    assert worst <= 5e-7


def _slice_stats(x, parts):
    """(mean, M2) of each of `parts` equal column slices of each row, f64."""
    m, d = x.shape
    xs = x.astype(np.float64).reshape(m, parts, d // parts)
    mean = xs.mean(axis=2)
    return np.stack([mean, ((xs - mean[:, :, None]) ** 2).sum(axis=2)], axis=2)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("d", [384, 1024])
@pytest.mark.parametrize("given_stats", [False, True])
def test_layernorm_prologue(dtype, d, given_stats):
    """QKV projection of LN(x): the LayerNorm (reference.rs:247-270) computed
    inside the GEMM, its row statistics either from a pass over the rows or
    given as per-slice (mean, M2) partials; Q|K stored in `dtype`, V in f16
    (split store)."""
    import torch
    import beatlm_b200 as bl
    m, n = 1370, 3 * d
    x = oracle.uniform(9, m * d, -2, 2) + np.float32(0.7)  # a non-zero mean
    g, be = oracle.uniform(10, d, 0.8, 1.2), oracle.uniform(11, d, -0.1, 0.1)
    w = _rnd(oracle.uniform(12, d * n, -1 / math.sqrt(d), 1 / math.sqrt(d)), dtype)
    b = oracle.uniform(13, n, -0.1, 0.1)
    out = torch.zeros((m, n), dtype=torch.int16, device="cuda")
    stats = (torch.from_numpy(_slice_stats(x.reshape(m, d), d // 32).astype(np.float32)).cuda()
             if given_stats else None)
    bl.ops.linear(_dev(w.reshape(d, n).T, dtype), ln=(_dev(x.reshape(m, d), "f32"),
                  _dev(g, "f32"), _dev(be, "f32"), 1e-6), bias=_dev(b, "f32"), out=out,
                  out_dtype=dtype, out_split=(2 * d, "f16"), ln_stats=stats)
    torch.cuda.synchronize()
    _check_status()
    o = out.cpu()
    qk = o[:, :2 * d].view(torch.bfloat16 if dtype == "bf16" else torch.float16).float().numpy()
    v = o[:, 2 * d:].view(torch.float16).float().numpy()
    a = _rnd(oracle.layernorm(x, g, be, 1e-6), dtype)
    want = oracle.matmul(a, w, b, m, d, n).reshape(m, n)
    # the stored values are 16-bit: compare with the oracle rounded the same way
    rel_qk = _rel(qk, _rnd(want[:, :2 * d], dtype))
    rel_v = _rel(v, oracle.round_f16(want[:, 2 * d:]))
    print("LN prologue %s D=%d: rel-L2 QK %.2e V %.2e" % (dtype, d, rel_qk, rel_v))
    assert rel_qk < 2e-4 and rel_v < 2e-4


@pytest.mark.parametrize("m,n,k", [(1370, 384, 384), (1370, 384, 1536), (300, 1024, 256)])
def test_row_statistics_of_the_stored_output(m, n, k):
    """A residual GEMM (x1 = x + ls * (A.W + b), f32) also writes each row's
    per-32-column (mean, M2) of the values it stored: checked against the
    stored output itself, and the LayerNorm prologue fed by them gives the
    same rows as a standalone LayerNorm of that output."""
    import torch
    import beatlm_b200 as bl
    a = _rnd(oracle.normal(21, m * k), "bf16")
    w = _rnd(oracle.uniform(22, k * n, -0.05, 0.05), "bf16")
    x = torch.from_numpy(oracle.uniform(23, m * n, -2, 2).reshape(m, n)).cuda()
    stats = torch.zeros((m, n // 32, 2), dtype=torch.float32, device="cuda")
    bl.ops.linear(_dev(w.reshape(k, n).T, "bf16"), a=_dev(a.reshape(m, k), "bf16"),
                  bias=_dev(oracle.uniform(24, n, -0.1, 0.1), "f32"),
                  chan_scale=_dev(oracle.uniform(25, n, 0.1, 1.0), "f32"), residual=x, out=x,
                  stats_out=stats)
    torch.cuda.synchronize()
    _check_status()
    want = _slice_stats(x.cpu().numpy(), n // 32)
    got = stats.cpu().numpy().astype(np.float64)
    assert np.allclose(got[..., 0], want[..., 0], rtol=1e-5, atol=1e-6)
    assert np.allclose(got[..., 1], want[..., 1], rtol=1e-4, atol=1e-5)
    # the consumer: LN(x) . W2 with the given statistics vs LN by its own kernel
    g, be = _dev(oracle.uniform(26, n, 0.8, 1.2), "f32"), _dev(oracle.uniform(27, n, -0.1, 0.1), "f32")
    w2 = _dev(_rnd(oracle.uniform(28, n * 64, -0.1, 0.1), "bf16").reshape(n, 64).T, "bf16")
    y1 = torch.zeros((m, 64), dtype=torch.float32, device="cuda")
    y2 = torch.zeros_like(y1)
    bl.ops.linear(w2, ln=(x, g, be, 1e-6), ln_stats=stats, out=y1)
    xn = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    bl.ops.layernorm(x, g, be, 1e-6, out=xn)
    bl.ops.linear(w2, a=xn, out=y2)
    torch.cuda.synchronize()
    _check_status()
    assert _rel(y1.cpu().numpy(), y2.cpu().numpy()) < 2e-3


@pytest.mark.parametrize("m", [1370, 300])
def test_layernorm_in_the_epilogue_matches_a_standalone_layernorm(m):
    """x1 = x + ls * (A.W + b) (f32, stored) and LayerNorm(x1) written by the
    same GEMM's epilogue: the normalised rows equal a standalone LayerNorm of
    the stored x1 to within a 16-bit rounding, and the exchange buffer is
    zero-filled again afterwards (a second launch gives the same rows)."""
    import torch
    import beatlm_b200 as bl
    n, k = 384, 1536
    a = _rnd(oracle.normal(31, m * k), "bf16")
    w = _rnd(oracle.uniform(32, k * n, -0.05, 0.05), "bf16")
    x0 = oracle.uniform(33, m * n, -2, 2).reshape(m, n)
    g = _dev(oracle.uniform(36, n, 0.8, 1.2), "f32")
    be = _dev(oracle.uniform(37, n, -0.1, 0.1), "f32")
    sync = torch.zeros(bl.ops.gemm_norm_sync_bytes(m, n), dtype=torch.uint8, device="cuda")
    outs = []
    for rep in range(2):
        x = torch.from_numpy(x0.copy()).cuda()
        xn = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
        bl.ops.linear(_dev(w.reshape(k, n).T, "bf16"), a=_dev(a.reshape(m, k), "bf16"),
                      bias=_dev(oracle.uniform(34, n, -0.1, 0.1), "f32"),
                      chan_scale=_dev(oracle.uniform(35, n, 0.1, 1.0), "f32"), residual=x, out=x,
                      norm=(g, be, 1e-6, xn), norm_sync=sync)
        torch.cuda.synchronize()
        _check_status()
        nctr = (8 * ((m + 127) // 128) + 15) // 16 * 16  # the counters, first in the buffer
        assert int(sync[:nctr].count_nonzero()) == 0
        want = torch.zeros_like(xn)
        bl.ops.layernorm(x, g, be, 1e-6, out=want)
        torch.cuda.synchronize()
        got, ref = xn.float().cpu().numpy(), want.float().cpu().numpy()
        assert np.all(np.abs(got - ref) <= 2 ** -7 * np.abs(ref) + 2e-3), np.max(np.abs(got - ref))
        outs.append(got)
    assert np.array_equal(outs[0], outs[1])


def test_layernorm_in_the_epilogue_is_refused_where_tiles_do_not_fit():
    import torch
    import beatlm_b200 as bl
    m, n = 128 * 40, 384  # 480 column tiles of 32
    w = torch.zeros((n, 64), dtype=torch.bfloat16, device="cuda")
    a = torch.zeros((m, 64), dtype=torch.bfloat16, device="cuda")
    x = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    xn = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    g = torch.ones(n, device="cuda")
    sync = torch.zeros(bl.ops.gemm_norm_sync_bytes(m, n), dtype=torch.uint8, device="cuda")
    with pytest.raises(bl.BackendError, match="resident"):
        bl.ops.linear(w, a=a, out=x, norm=(g, g, 1e-6, xn), norm_sync=sync)
    with pytest.raises(bl.BackendError, match="norm_sync"):
        bl.ops.linear(w, a=a[:128], out=x[:128], norm=(g, g, 1e-6, xn[:128]), norm_sync=sync[:64])


def test_statistics_arguments_are_checked():
    import torch
    import beatlm_b200 as bl
    w = torch.zeros((384, 384), dtype=torch.bfloat16, device="cuda")
    a = torch.zeros((128, 384), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(bl.BackendError, match="f32"):
        bl.ops.linear(w, a=a, out=torch.zeros((128, 384), dtype=torch.bfloat16, device="cuda"),
                      stats_out=torch.zeros((128, 12, 2), device="cuda"))
    with pytest.raises(bl.BackendError, match="parts"):
        bl.ops.linear(w, a=a, out=torch.zeros((128, 384), device="cuda"),
                      stats_out=torch.zeros((128, 7, 2), device="cuda"))


def test_patch_rows_land_after_the_class_token():
    """Output-row grouping (patch tokens after each frame's class token) and a
    periodic residual (the position embedding)."""
    import torch
    import beatlm_b200 as bl
    frames, t, n, k = 2, 10, 64, 64
    rows = frames * (t - 1)
    a = _rnd(oracle.normal(14, rows * k), "f16")
    w = _rnd(oracle.uniform(15, k * n, -0.1, 0.1), "f16")
    pos = oracle.uniform(16, t * n, -1, 1)
    out = torch.full((frames * t, n), 7.0, dtype=torch.float32, device="cuda")
    bl.ops.linear(_dev(w.reshape(k, n).T, "f16"), a=_dev(a.reshape(rows, k), "f16"),
                  residual=_dev(pos.reshape(t, n), "f32"), res_period=t, out=out,
                  out_row_offset=1, out_group=(t - 1, 1))
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(frames, t, n)
    prod = oracle.matmul(a, w, None, rows, k, n).reshape(frames, t - 1, n)
    want = prod + pos.reshape(t, n)[1:]
    assert np.all(got[:, 0] == 7.0)
    _close(got[:, 1:], want, "grouped rows")


def test_bad_shapes_are_errors():
    import torch
    import beatlm_b200 as bl
    w = torch.zeros((64, 60), dtype=torch.float16, device="cuda")
    with pytest.raises(bl.BackendError, match="multiple of 64"):
        bl.ops.linear(w, a=torch.zeros((4, 60), dtype=torch.float16, device="cuda"),
                      out=torch.zeros((4, 64), device="cuda"))
    w = torch.zeros((40, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(bl.BackendError, match="tile width"):
        bl.ops.linear(w, a=torch.zeros((4, 64), dtype=torch.float16, device="cuda"),
                      out=torch.zeros((4, 40), device="cuda"))


@pytest.mark.parametrize("m,n,k,tile,form", [
    (1370, 3072, 1024, 256, "bias"),      # ViT-L qkv
    (1370, 4096, 1024, 256, "gelu"),      # ViT-L fc1 (several tiles per pair)
    (1370, 1024, 1024, 128, "residual"),  # ViT-L proj
    (1370, 1024, 4096, 128, "residual"),  # ViT-L fc2
    (100, 256, 128, 256, "bias"),         # one pair tile, the odd CTA's rows all past M
    (700, 384, 384, 128, "generic"),      # generic epilogue (scale), f16
])
def test_cta_pair_tiles_equal_one_cta_tiles(m, n, k, tile, form):
    """256-row tiles over CTA pairs (cta_group::2 MMAs reading both CTAs'
    operands) give the same bits as 128-row tiles of one CTA with the same
    epilogue, and meet the oracle."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    dtype = "f16" if form == "generic" else "bf16"
    a = _rnd(oracle.normal(7 * m + n, m * k), dtype)
    w = _rnd(oracle.uniform(k + 1, k * n, -1 / math.sqrt(k), 1 / math.sqrt(k)), dtype)
    b = oracle.uniform(n + 2, n, -0.1, 0.1)
    wd, ad, bd = _dev(w.reshape(k, n).T, dtype), _dev(a.reshape(m, k), dtype), _dev(b, "f32")
    x0 = oracle.uniform(n + 3, m * n, -1.0, 1.0).reshape(m, n)
    ls = oracle.uniform(n + 4, n, 0.1, 1.0)
    outs = []
    for pair in (0, 2):
        kw = dict(bias=bd, tile_n=tile, weights_static=True, pair_tiles=pair)
        if form == "residual":
            x = _dev(x0, "f32")
            kw.update(chan_scale=_dev(ls, "f32"), residual=x, out=x)
        elif form == "gelu":
            kw.update(act="gelu_erf", out=torch.zeros((m, n), dtype=torch.bfloat16, device="cuda"))
        elif form == "generic":
            kw.update(scale=0.5, out=torch.zeros((m, n), dtype=torch.float32, device="cuda"))
        else:
            kw.update(out=torch.zeros((m, n), dtype=torch.bfloat16, device="cuda"))
        g = ops.gemm_args(wd, a=ad, **kw)
        N = bl.ops.N
        N.check(N.lib().bl_gemm(ctypes.byref(g), None))
        torch.cuda.synchronize()
        _check_status()
        outs.append(kw["out"].float().cpu().numpy())
    assert np.array_equal(outs[0], outs[1]), form
    want = oracle.matmul(a, w, b, m, k, n)
    if form == "residual":
        want = x0.ravel() + want * np.tile(ls, m)
        _close(outs[1], want, "pair residual")
    elif form == "generic":
        _close(outs[1], 0.5 * want, "pair generic")
    else:
        if form == "gelu":
            want = oracle.gelu_erf(want)
        assert _rel(outs[1], want) <= 4e-3


def test_cta_pairs_reject_row_parts_and_prologues():
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    m, n, k = 512, 256, 128
    w = torch.zeros((n, k), dtype=torch.bfloat16, device="cuda")
    a = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    g = ops.gemm_args(w, a=a, out=out, pair_tiles=3)
    with pytest.raises(bl.BackendError, match="pair_tiles"):
        bl.ops.N.check(bl.ops.N.lib().bl_gemm(ctypes.byref(g), None))
    g = ops.gemm_args(w, a=a, out=out, pair_tiles=2, tile_n=64)
    with pytest.raises(bl.BackendError, match="CTA pairs"):
        bl.ops.N.check(bl.ops.N.lib().bl_gemm(ctypes.byref(g), None))


@pytest.mark.parametrize("m,n,k,form", [
    (1370, 384, 1536, "residual"),  # ViT-S fc2 (the automatic choice)
    (1370, 384, 1024, "bias"),
    (129, 128, 256, "gelu"),        # the shortest K the split takes: two stages per CTA
    (300, 64, 3456, "bias"),        # a single column tile, K of the DPT neck convolution
    (1370, 512, 1600, "generic"),   # K / 64 = 25: unequal halves
])
def test_k_split_over_a_cluster_meets_the_oracle(m, n, k, form):
    """The K range split over two CTAs of a cluster, each adding the other's
    partial sums for its half of the columns (distributed shared memory)
    before the epilogue: within the reference's GEMM tolerance of the oracle,
    and close to the unsplit kernel (which sums K in one chain)."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    dtype = "bf16"
    a = _rnd(oracle.normal(11 * m + k, m * k), dtype)
    w = _rnd(oracle.uniform(k + 5, k * n, -1 / math.sqrt(k), 1 / math.sqrt(k)), dtype)
    b = oracle.uniform(n + 6, n, -0.1, 0.1)
    wd, ad, bd = _dev(w.reshape(k, n).T, dtype), _dev(a.reshape(m, k), dtype), _dev(b, "f32")
    x0 = oracle.uniform(n + 7, m * n, -1.0, 1.0).reshape(m, n)
    ls = oracle.uniform(n + 8, n, 0.1, 1.0)
    outs = []
    for split in (1, 2):
        kw = dict(bias=bd, weights_static=True, split_k=split)
        if form == "residual":
            x = _dev(x0, "f32")
            kw.update(chan_scale=_dev(ls, "f32"), residual=x, out=x)
        elif form == "gelu":
            kw.update(act="gelu_erf", out=torch.zeros((m, n), dtype=torch.float32, device="cuda"))
        elif form == "generic":
            kw.update(scale=0.25, out=torch.zeros((m, n), dtype=torch.float32, device="cuda"))
        else:
            kw.update(out=torch.zeros((m, n), dtype=torch.float32, device="cuda"))
        g = ops.gemm_args(wd, a=ad, **kw)
        bl.ops.N.check(bl.ops.N.lib().bl_gemm(ctypes.byref(g), None))
        torch.cuda.synchronize()
        _check_status()
        outs.append(kw["out"].float().cpu().numpy())
    want = oracle.matmul(a, w, b, m, k, n)
    if form == "residual":
        want = x0.ravel() + want * np.tile(ls, m)
    elif form == "gelu":
        want = oracle.gelu_erf(want)
    elif form == "generic":
        want = 0.25 * want
    _close(outs[1], want, "K split %s" % form)
    # two f32 partial sums added instead of one chain: a few ulps over long K
    assert _rel(outs[1], outs[0]) < 1e-5


def test_k_split_rejects_what_it_cannot_take():
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    w = torch.zeros((96, 1024), dtype=torch.bfloat16, device="cuda")
    a = torch.zeros((256, 1024), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((256, 96), dtype=torch.float32, device="cuda")
    for bad, match in ((dict(split_k=3), "split_k"), (dict(split_k=2), "K split")):
        g = ops.gemm_args(w, a=a, out=out, **bad)
        with pytest.raises(bl.BackendError, match=match):
            bl.ops.N.check(bl.ops.N.lib().bl_gemm(ctypes.byref(g), None))


def _sk_case(m, n, k, form, seed, tile_n=0):
    """Operands, host expectation and a kwargs builder for a stream-K case."""
    import torch
    dtype = "bf16"
    a = _rnd(oracle.normal(13 * m + k + seed, m * k), dtype)
    w = _rnd(oracle.uniform(k + 9 + seed, k * n, -1 / math.sqrt(k), 1 / math.sqrt(k)), dtype)
    b = oracle.uniform(n + 10 + seed, n, -0.1, 0.1)
    wd, ad, bd = _dev(w.reshape(k, n).T, dtype), _dev(a.reshape(m, k), dtype), _dev(b, "f32")
    x0 = oracle.uniform(n + 11 + seed, m * n, -1.0, 1.0).reshape(m, n)
    ls = oracle.uniform(n + 12 + seed, n, 0.1, 1.0)

    def kwargs():
        kw = dict(a=ad, bias=bd, weights_static=True, split_k=1, tile_n=tile_n)
        if form == "residual":
            x = _dev(x0, "f32")
            kw.update(chan_scale=_dev(ls, "f32"), residual=x, out=x)
        elif form == "gelu":
            kw.update(act="gelu_erf", out=torch.zeros((m, n), dtype=torch.float32, device="cuda"))
        elif form == "generic":
            kw.update(scale=0.25, out=torch.zeros((m, n), dtype=torch.float32, device="cuda"))
        else:
            kw.update(out=torch.zeros((m, n), dtype=torch.float32, device="cuda"))
        return kw

    want = oracle.matmul(a, w, b, m, k, n)
    if form == "residual":
        want = x0.ravel() + want * np.tile(ls, m)
    elif form == "gelu":
        want = oracle.gelu_erf(want)
    elif form == "generic":
        want = 0.25 * want
    return wd, kwargs, want


def _sk_flag_bytes(m, n, args):
    """The flag area at the head of a stream-K workspace: one word per
    (tile, piece) slot padded to 256 bytes; tiles and pieces follow from the
    workspace size, whose rest is 128 x bn f32 per slot."""
    from beatlm_b200 import ops
    total = ops.gemm_workspace_bytes(args)
    for bn in (128, 256):
        for pieces in (2, 3):
            slots = ((m + 127) // 128) * (n // bn) * pieces
            flags = (4 * slots + 255) // 256 * 256
            if n % bn == 0 and flags + 4 * 128 * bn * slots == total:
                return flags
    raise AssertionError("no (tile width, pieces) gives %d bytes" % total)


@pytest.mark.parametrize("m,n,k,form,tile", [
    (1370, 1024, 4096, "residual", 0),  # ViT-L fc2 (128-column tiles, three pieces)
    (300, 1024, 2048, "generic", 128),  # ragged last row tile
    (129, 256, 1024, "gelu", 256),      # 256-column tiles, one row past a tile
    (384, 512, 2048, "bias", 128),
])
def test_stream_k_meets_the_oracle(m, n, k, form, tile):
    """Stream-K (stream_k 2): every tile's k-stages cut into pieces dealt
    over the SMs, each accumulated on its own and added in piece order by the
    CTA holding the last piece. Within the reference's GEMM tolerance of the
    oracle, close to whole tiles (a few partial sums instead of one chain),
    the same bits on a second launch through the same workspace, whose flags
    the launches leave at zero."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    mode = 2
    wd, kwargs, want = _sk_case(m, n, k, form, 0, tile)
    whole_kw = kwargs()
    g = ops.gemm_args(wd, stream_k=1, **whole_kw)
    bl.ops.N.check(bl.ops.N.lib().bl_gemm(ctypes.byref(g), None))
    probe_kw = kwargs()
    probe = ops.gemm_args(wd, stream_k=mode, **probe_kw)
    nbytes = ops.gemm_workspace_bytes(probe)
    assert nbytes > 0, "stream-K not taken"
    flags = _sk_flag_bytes(m, n, probe)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(2):
        kw = kwargs()
        g = ops.gemm_args(wd, stream_k=mode, workspace=ws, **kw)
        bl.ops.N.check(bl.ops.N.lib().bl_gemm(ctypes.byref(g), None))
        torch.cuda.synchronize()
        _check_status()
        assert int(ws[:flags].count_nonzero()) == 0, "flags left set"
        outs.append(kw["out"].float().cpu().numpy())
    torch.cuda.synchronize()
    whole = whole_kw["out"].float().cpu().numpy()
    _close(outs[0], want, "stream-K %s" % form)
    assert np.array_equal(outs[0], outs[1])
    assert _rel(outs[0], whole) < 1e-5


def test_stream_k_row_parts_compute_as_the_whole_launch():
    """The pieces come from the whole launch's shape, so a program that
    splits the GEMM into row parts (each a launch of its own) gives the same
    bits as the unsplit launch."""
    import torch
    from beatlm_b200 import ops
    from beatlm_b200.runtime import Kernels, Spec
    m, n, k = 1370, 1024, 4096
    wd, kwargs, _ = _sk_case(m, n, k, "residual", 3)
    res = []
    for parts in (1, 3, 5):
        kw = kwargs()
        probe = ops.gemm_args(wd, stream_k=2, **kw)
        ws = torch.zeros(ops.gemm_workspace_bytes(probe), dtype=torch.uint8, device="cuda")
        assert ws.numel() > 0
        prog = Kernels([Spec(ops.gemm_args(wd, stream_k=2, workspace=ws, **kw), "fc2", parts)])
        prog.encode_all(None)
        torch.cuda.synchronize()
        _check_status()
        res.append(kw["out"].cpu())
        prog.close()
    assert torch.equal(res[0], res[1]) and torch.equal(res[0], res[2])


def test_stream_k_workspace_query_and_rejects():
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops

    def args(m, n, k, **kw):
        w = torch.zeros((n, k), dtype=torch.bfloat16, device="cuda")
        a = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
        out = torch.zeros((m, n), dtype=torch.float32, device="cuda")
        return ops.gemm_args(w, a=a, out=out, **kw), (w, a, out)

    # only on request: 0 and 1 keep whole tiles and need no workspace
    for mode in (0, 1):
        g, keep = args(1370, 1024, 4096, stream_k=mode)
        assert ops.gemm_workspace_bytes(g) == 0
    # ViT-L fc2: 88 tiles of 32 stages in three pieces, a 128 x 128 slot each
    g, keep = args(1370, 1024, 4096, stream_k=2)
    slots = 88 * 3
    assert ops.gemm_workspace_bytes(g) == (4 * slots + 255) // 256 * 256 + slots * 128 * 128 * 4
    for bad, match in ((dict(stream_k=3), "stream_k"),
                       (dict(stream_k=2), "workspace"),
                       (dict(stream_k=2, tile_n=32), "stream-K takes"),
                       (dict(stream_k=2, split_k=2), "stream-K takes")):
        g, keep = args(1370, 1024, 4096, **bad)
        with pytest.raises(bl.BackendError, match=match):
            bl.ops.N.check(bl.ops.N.lib().bl_gemm(ctypes.byref(g), None))
