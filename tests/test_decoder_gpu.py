"""The DPT decoder's convolutions and resampling on the GPU (bl_im2col +
the tcgen05 GEMM, bl_blocks_to_map, bl_resize_bilinear and its 16-bit rows
form, bl_conv1x1_one and the GEMM's row reduction) against the oracle
restatement of the reference's CPU definitions
(crates/beatlm-bench/src/reference.rs:25-230), at DPT-S shapes on the 37 x 37
patch grid. f16 operands, f32 accumulation: relative L2 <= 1e-3 against the
f32 oracle, and <= 1e-5 against the oracle fed the same f16-rounded
operands."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

REL = 1e-3
REL_ROUNDED = 1e-5


def _rel(got, want):
    got, want = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def _data(seed, n, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)


@pytest.mark.parametrize("h,w,cin,cout,stride,relu", [
    (37, 37, 64, 64, 1, True),     # a fusion residual unit's convolution
    (37, 37, 384, 64, 1, False),   # the neck's 3x3 to the fusion width
    (37, 37, 48, 48, 2, False),    # K = 432 padded to 448, cout 48 padded to 64
    (19, 19, 192, 384, 2, False),  # the deepest stage's strided convolution
    (20, 23, 3, 32, 1, True),      # cin not a multiple of 8: the per-column gather
])
def test_conv3x3_matches_the_reference(h, w, cin, cout, stride, relu):
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    x = _data(1, h * w * cin)
    wt = _data(2, 9 * cin * cout, 1.0 / np.sqrt(9 * cin))
    b = _data(3, cout, 0.1)
    dev = torch.from_numpy(x).cuda()
    got = ops.conv2d(dev, ops.conv_weights(wt, 3, cin, cout), torch.from_numpy(b).cuda(), h, w,
                     cin, cout, stride=stride, relu_input=relu).cpu().numpy()
    assert bl.status(reset=True).code == 0
    xin = oracle.relu(x) if relu else x
    want = oracle.conv3x3(xin, wt, b, h, w, cin, cout, stride)
    assert got.size == want.size
    rel = _rel(got, want)
    rounded = oracle.conv3x3(oracle.round_f16(xin), oracle.round_f16(wt), b, h, w, cin, cout,
                             stride)
    rel_r = _rel(got, rounded)
    print("conv3x3 %dx%dx%d->%d s%d: rel-L2 %.2e (f32 oracle), %.2e (rounded operands)"
          % (h, w, cin, cout, stride, rel, rel_r))
    assert rel <= REL and rel_r <= REL_ROUNDED


@pytest.mark.parametrize("pixels,cin,cout,act", [(1369, 384, 96, None), (1369, 64, 64, "relu"),
                                                 (5476, 64, 32, "relu")])
def test_conv1x1_matches_the_reference(pixels, cin, cout, act):
    import torch
    from beatlm_b200 import ops
    x, wt, b = _data(4, pixels * cin), _data(5, cin * cout, 1 / np.sqrt(cin)), _data(6, cout, 0.1)
    got = ops.conv2d(torch.from_numpy(x).cuda(), ops.conv_weights(wt, 1, cin, cout),
                     torch.from_numpy(b).cuda(), pixels, 1, cin, cout, ksize=1,
                     act=act).cpu().numpy()
    want = oracle.conv1x1(x, wt, b, pixels, cin, cout)
    if act == "relu":
        want = oracle.relu(want)
    assert _rel(got, want) <= REL


def test_a_residual_unit_matches_the_reference():
    """x + conv2(relu(conv1(relu(x)))) (reference.rs:190-201) with the ReLU
    applied on the way into each im2col and the residual added by the second
    GEMM's epilogue."""
    import torch
    from beatlm_b200 import ops
    h = w = 37
    c = 64
    x = _data(7, h * w * c)
    w1, w2 = _data(8, 9 * c * c, 1 / 24), _data(9, 9 * c * c, 1 / 24)
    b1, b2 = _data(10, c, 0.1), _data(11, c, 0.1)
    dev = torch.from_numpy(x).cuda()
    first = ops.conv2d(dev, ops.conv_weights(w1, 3, c, c), torch.from_numpy(b1).cuda(), h, w,
                       c, c, relu_input=True)
    got = ops.conv2d(first, ops.conv_weights(w2, 3, c, c), torch.from_numpy(b2).cuda(), h, w,
                     c, c, relu_input=True, residual=dev).cpu().numpy()
    want = oracle.residual_unit(x, w1, b1, w2, b2, h, w, c)
    rel = _rel(got, want)
    print("residual unit: rel-L2 %.2e" % rel)
    assert rel <= REL


@pytest.mark.parametrize("h,w,cin,cout,f", [(37, 37, 48, 48, 4), (37, 37, 96, 96, 2),
                                            (3, 5, 64, 8, 2)])
def test_conv_transpose_matches_the_reference(h, w, cin, cout, f):
    import torch
    from beatlm_b200 import ops
    x, wt, b = _data(12, h * w * cin), _data(13, f * f * cin * cout, 1 / np.sqrt(cin)), \
        _data(14, cout, 0.1)
    got = ops.conv_transpose(torch.from_numpy(x).cuda(), wt, torch.from_numpy(b).cuda(), h, w,
                             cin, cout, f).cpu().numpy()
    want = oracle.conv_transpose(x, wt, b, h, w, cin, cout, f)
    assert got.size == want.size and _rel(got, want) <= REL


@pytest.mark.parametrize("ih,iw,oh,ow,c", [(37, 37, 74, 74, 64), (19, 19, 37, 37, 64),
                                           (2, 2, 3, 3, 1), (1, 4, 1, 7, 1), (2, 1, 1, 1, 1)])
def test_resize_bilinear_matches_the_reference(ih, iw, oh, ow, c):
    import torch
    from beatlm_b200 import ops
    x = _data(15, ih * iw * c)
    got = ops.resize_bilinear(torch.from_numpy(x).cuda(), ih, iw, oh, ow, c).cpu().numpy()
    want = oracle.resize_bilinear(x, ih, iw, oh, ow, c)
    assert np.abs(got.ravel() - want).max() <= 1e-5 * max(1.0, np.abs(want).max())


def _oracle_decoder(cfg, dcfg, w, feats):
    return oracle.dpt_head(cfg.grid, cfg.patch, cfg.dim, dcfg.neck, dcfg.reassemble,
                           dcfg.fusion, dcfg.head, w, feats)


def test_the_dpt_head_matches_the_reference_chain():
    """The whole DPT head of Depth-Anything-V2-Small at 266 px (grid 19:
    stages 76, 38, 19 and 10 a side, fusion to 152, depth at 266 x 266) from
    random features, against the oracle chain of the reference's decoder. Some
    20 convolutions in f16 operands each add their rounding: relative L2
    <= 3e-3 for the depth map."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.model import Decoder, DecoderConfig, ViTConfig, decoder_weights_random
    cfg, dcfg = ViTConfig.small(side=266), DecoderConfig()
    w = decoder_weights_random(cfg, dcfg, seed=5)
    feats = [_data(40 + i, cfg.grid * cfg.grid * cfg.dim) for i in range(4)]
    dec = Decoder(cfg, dcfg, w)
    depth = dec.forward([torch.from_numpy(f).cuda() for f in feats]).cpu().numpy()
    assert bl.status(reset=True).code == 0
    want = _oracle_decoder(cfg, dcfg, w, feats)
    assert depth.shape == (266, 266)
    rel = _rel(depth, want)
    print("DPT head at 266 px: rel-L2 %.2e, max-abs %.2e" % (rel, np.abs(depth.ravel() - want).max()))
    assert rel <= 3e-3


def test_the_captured_head_replays_the_direct_pass():
    """Decoder.capture: the same kernels on the same features as forward(),
    so the replayed depth equals the direct one bit for bit, and a replay
    after the features change follows them."""
    import torch
    from beatlm_b200.model import Decoder, DecoderConfig, ViTConfig, decoder_weights_random
    cfg, dcfg = ViTConfig.small(side=266), DecoderConfig()
    dec = Decoder(cfg, dcfg, decoder_weights_random(cfg, dcfg, seed=6))
    feats = [torch.from_numpy(_data(60 + i, cfg.grid * cfg.grid * cfg.dim)).cuda()
             for i in range(4)]
    want = dec.forward(feats).clone()
    s = torch.cuda.Stream()
    g, depth = dec.capture(feats, s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(depth, want)
    for i, f in enumerate(feats):
        f.copy_(torch.from_numpy(_data(70 + i, f.numel())))
    want2 = dec.forward(feats).clone()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(depth, want2) and not torch.equal(want, want2)


def test_the_head_on_a_side_stream_equals_the_current_stream():
    """Decoder.forward(stream=s) with s not the current stream: every
    convolution, resampling, temporary and add of the head runs on s, so the
    depth equals the pass on the current stream bit for bit."""
    import torch
    from beatlm_b200.model import Decoder, DecoderConfig, ViTConfig, decoder_weights_random
    cfg, dcfg = ViTConfig.small(side=266), DecoderConfig()
    dec = Decoder(cfg, dcfg, decoder_weights_random(cfg, dcfg, seed=8))
    feats = [torch.from_numpy(_data(80 + i, cfg.grid * cfg.grid * cfg.dim)).cuda()
             for i in range(4)]
    want = dec.forward(feats).clone()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    got = dec.forward(feats, stream=side)
    side.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("h,w,f,cout,bias", [(5, 3, 2, 6, True), (4, 7, 3, 8, True),
                                             (37, 37, 4, 48, False)])
def test_blocks_to_map_scatters_every_block(h, w, f, cout, bias):
    """bl_blocks_to_map, both forms (4-channel vectors when cout is a multiple
    of 4, else per element): out[y f + ky][x f + kx][co] = blocks[y w + x]
    [(ky f + kx) cout + co] + bias[co], exactly."""
    import ctypes
    import torch
    from beatlm_b200 import _native as N
    blocks = _data(20, h * w * f * f * cout)
    b = _data(21, cout, 0.1)
    dev_b = torch.from_numpy(b).cuda() if bias else None
    dev = torch.from_numpy(blocks).cuda()
    out = torch.full((h * f, w * f, cout), float("nan"), device="cuda")
    N.check(N.lib().bl_blocks_to_map(dev.data_ptr(), None if dev_b is None else dev_b.data_ptr(),
                                     out.data_ptr(), h, w, f, cout, None))
    torch.cuda.synchronize()
    want = blocks.reshape(h, w, f, f, cout).transpose(0, 2, 1, 3, 4).reshape(h * f, w * f, cout)
    if bias:
        want = want + b
    assert np.array_equal(out.cpu().numpy(), want.astype(np.float32))


@pytest.mark.parametrize("h,w,cin,cout,relu,act,res", [
    (37, 37, 64, 64, True, None, True),     # a fusion unit's second convolution
    (148, 148, 64, 32, False, None, False),  # the head's first convolution
    (74, 74, 96, 64, False, "relu", False),  # k-blocks straddling taps (96 channels)
    (23, 1, 32, 32, True, None, False),      # one column: both side taps outside
    (1, 40, 32, 64, False, None, True),      # one row: the vertical taps outside
    (5, 7, 192, 128, True, "relu", False),   # fewer pixels than one tile
    (518, 518, 32, 32, False, "relu", False),  # the depth head's full-resolution convolution
])
def test_implicit_conv3x3_equals_the_gathered_one(h, w, cin, cout, relu, act, res):
    """bl_conv3x3 (the image read through the taps on chip) against im2col +
    bl_gemm with K in one chain (split_k 1): the same 16-bit A values, the
    same k-block order and the same epilogue, so the same bits; and both
    against the oracle."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    x = _data(40 + cin, h * w * cin)
    wt = _data(41, 9 * cin * cout, 1.0 / np.sqrt(9 * cin))
    b = torch.from_numpy(_data(42, cout, 0.1)).cuda()
    dev = torch.from_numpy(x).cuda()
    r = torch.from_numpy(_data(43, h * w * cout)).cuda().reshape(h * w, cout) if res else None
    wdev = ops.conv_weights(wt, 3, cin, cout)
    run = lambda implicit: ops.conv2d(dev, wdev, b, h, w, cin, cout, relu_input=relu, act=act,
                                      residual=r, implicit=implicit, split_k=1)
    got, gathered = run(True), run(False)
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    assert torch.equal(got, gathered)
    if h * w <= 40000:
        xin = oracle.relu(x) if relu else x
        want = oracle.conv3x3(xin, wt, b.cpu().numpy(), h, w, cin, cout, 1)
        if act == "relu":
            want = oracle.relu(want)
        if res:
            want = want + r.cpu().numpy().ravel()
        assert _rel(got.cpu().numpy(), want) <= REL


def _im2col_host(x, h, w, cin, ks, stride, relu, k_pad, dtype):
    """The reference's im2col order (K = taps x cin, tap = ky * ks + kx), zero
    border, ReLU on the way in, rounded to the 16-bit type."""
    pad = ks // 2
    oh, ow = (h + 2 * pad - ks) // stride + 1, (w + 2 * pad - ks) // stride + 1
    img = x.reshape(h, w, cin)
    if relu:
        img = np.maximum(img, 0.0)
    padded = np.zeros((h + 2 * pad, w + 2 * pad, cin), np.float32)
    padded[pad:pad + h, pad:pad + w] = img
    out = np.zeros((oh, ow, k_pad), np.float32)
    for ky in range(ks):
        for kx in range(ks):
            t = (ky * ks + kx) * cin
            out[:, :, t:t + cin] = padded[ky:ky + stride * oh:stride, kx:kx + stride * ow:stride]
    out = out.reshape(oh * ow, k_pad)
    return oracle.round_f16(out) if dtype == "f16" else oracle.round_bf16(out)


@pytest.mark.parametrize("h,w,cin,ks,stride,relu,dtype", [
    (37, 37, 64, 3, 1, True, "f16"),      # a fusion unit at 37 px
    (148, 148, 64, 3, 1, False, "f16"),
    (518, 518, 32, 3, 1, True, "f16"),    # the head's full-resolution convolution
    (74, 74, 96, 3, 2, False, "bf16"),    # stride 2, 96 channels: vectors straddle taps
    (23, 1, 32, 3, 1, True, "f16"),       # one column
    (5, 7, 384, 3, 1, False, "f16"),      # K = 3456 (the neck's widest)
    (300, 11, 40, 1, 1, True, "bf16"),    # 1x1, K padded from 40 to 64
])
def test_im2col_gathers_the_reference_order(h, w, cin, ks, stride, relu, dtype):
    """bl_im2col's vector path (each block's tap table, each thread's
    (pixel, vector) stepped by the grid stride with carries) against a host
    gather of the same map: the same 16-bit values in every column, the
    padding columns zero."""
    import torch
    from beatlm_b200 import ops
    x = _data(70 + cin + h, h * w * cin)
    got, oh, ow = ops.im2col(torch.from_numpy(x).cuda(), h, w, cin, ksize=ks, stride=stride,
                             relu=relu, dtype=dtype)
    torch.cuda.synchronize()
    k_pad = got.shape[1]
    want = _im2col_host(x, h, w, cin, ks, stride, relu, k_pad, dtype)
    assert np.array_equal(got.float().cpu().numpy(), want)


@pytest.mark.parametrize("pixels,c,relu", [
    (518 * 518, 32, True),  # the depth head's last convolution
    (1001, 4, False),       # pixels not a multiple of a warp step
    (37, 64, True),
    (17, 256, False),
    (5, 1024, True),        # the widest row it takes
])
def test_conv1x1_one_matches_the_oracle(pixels, c, relu):
    """bl_conv1x1_one (one output channel of a 1x1 convolution, summed in f32
    by a fixed shuffle order) against the oracle's conv1x1 with one output
    channel (f64 sums): within 1e-5 relative L2, and two calls give the same
    bits."""
    import torch
    from beatlm_b200 import ops
    x = _data(90 + c, pixels * c)
    w = _data(91 + c, c, 1.0 / np.sqrt(c))
    b = 0.05
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    got = ops.conv1x1_one(xd, wd, b, pixels, c, relu=relu)
    again = ops.conv1x1_one(xd, wd, b, pixels, c, relu=relu)
    torch.cuda.synchronize()
    want = oracle.conv1x1(x, w.reshape(c, 1), np.array([b], np.float32), pixels, c, 1)
    if relu:
        want = np.maximum(want, 0.0)
    got = got.cpu().numpy()
    assert np.array_equal(got, again.cpu().numpy())
    assert _rel(got, want) < 1e-5
    if relu:
        assert (got >= 0).all()


@pytest.mark.parametrize("ih,iw,oh,ow,c,ld", [
    (148, 148, 296, 296, 64, 64),  # the last fusion layer's resampling before its projection
    (19, 19, 37, 37, 64, 64),      # the deepest layer's
    (37, 37, 74, 74, 48, 64),      # channels padded to the row width with zeros
    (2, 3, 5, 4, 8, 16),
    (1, 1, 1, 1, 8, 8),
])
@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_resize_rows16_is_the_rounded_f32_resampling(ih, iw, oh, ow, c, ld, dt):
    """bl_resize_bilinear_rows16 writes exactly the f32 resampling of
    bl_resize_bilinear rounded once to 16 bits (to nearest even), zeros in the
    padded channels, and stays within the oracle's tolerance."""
    import torch
    from beatlm_b200 import ops
    x = _data(70 + c, ih * iw * c)
    xd = torch.from_numpy(x).cuda()
    got = ops.resize_bilinear_rows16(xd, ih, iw, oh, ow, c, ld, dt)
    f32 = ops.resize_bilinear(xd, ih, iw, oh, ow, c)
    torch.cuda.synchronize()
    td = torch.float16 if dt == "f16" else torch.bfloat16
    assert got.dtype == td and tuple(got.shape) == (oh * ow, ld)
    want = f32.to(td)
    assert torch.equal(got[:, :c].view(torch.int16), want.view(torch.int16))
    assert not got[:, c:].float().abs().sum().item()
    ref = oracle.resize_bilinear(x, ih, iw, oh, ow, c)
    rel16 = 1e-2 if dt == "bf16" else 1e-3
    assert np.abs(got[:, :c].float().cpu().numpy().ravel() - ref).max() <= \
        rel16 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("side,out_side,c", [(74, 148, 64), (148, 296, 64)])
def test_projection_of_the_16bit_resampling_equals_the_gathered_one(side, out_side, c):
    """A fusion layer's resampling + 1x1 projection + the next stage map:
    from the 16-bit rows of bl_resize_bilinear_rows16 the GEMM alone gives
    the same bits as the f32 resampling followed by the 1x1 gather."""
    import torch
    from beatlm_b200 import ops
    x = torch.from_numpy(_data(80, side * side * c)).cuda()
    w = ops.conv_weights(_data(81, c * c, 1.0 / np.sqrt(c)), 1, c, c)
    b = torch.from_numpy(_data(82, c, 0.1)).cuda()
    res = torch.from_numpy(_data(83, out_side * out_side * c)).cuda().reshape(-1, c)
    rows = ops.resize_bilinear_rows16(x, side, side, out_side, out_side, c, w.shape[1])
    got = ops.conv2d(rows, w, b, out_side, out_side, c, c, ksize=1, residual=res)
    mid = ops.resize_bilinear(x, side, side, out_side, out_side, c)
    want = ops.conv2d(mid, w, b, out_side, out_side, c, c, ksize=1, residual=res)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    with pytest.raises(ValueError):
        ops.conv2d(rows[:-1], w, b, out_side, out_side, c, c, ksize=1)
    with pytest.raises(ValueError):
        ops.conv2d(rows, w, b, out_side, out_side, c, c, ksize=1, implicit=True)


@pytest.mark.parametrize("side,c,relu,dt", [(518, 32, False, "f16"), (74, 64, True, "f16"),
                                            (37, 48, True, "bf16"), (9, 8, False, "bf16")])
def test_gather_of_a_16bit_map_equals_the_gather_of_its_f32_map(side, c, relu, dt):
    """bl_im2col of a 16-bit map (the head's resampling written by
    bl_resize_bilinear_rows16) gives the same bits as the gather of the same
    values in f32, ReLU included, and so the same 3x3 convolution."""
    import torch
    from beatlm_b200 import ops
    td = torch.float16 if dt == "f16" else torch.bfloat16
    m16 = torch.from_numpy(_data(84, side * side * c)).cuda().to(td).reshape(-1, c)
    m32 = m16.float()
    got, _, _ = ops.im2col(m16, side, side, c, 3, 1, relu, dtype=dt)
    want, _, _ = ops.im2col(m32, side, side, c, 3, 1, relu, dtype=dt)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    wt = ops.conv_weights(_data(85, 9 * c * 32, 1.0 / np.sqrt(9 * c)), 3, c, 32, dtype=dt)
    b = torch.from_numpy(_data(86, 32, 0.1)).cuda()
    y16 = ops.conv2d(m16, wt, b, side, side, c, 32, relu_input=relu, act="relu")
    y32 = ops.conv2d(m32, wt, b, side, side, c, 32, relu_input=relu, act="relu")
    torch.cuda.synchronize()
    assert torch.equal(y16, y32)


@pytest.mark.parametrize("side,cin,cout,dt", [(148, 64, 64, "f16"), (37, 64, 48, "bf16")])
def test_conv_16bit_output_is_the_rounded_f32_output(side, cin, cout, dt):
    """conv2d(out_dtype=16-bit) (a fusion unit's first convolution, whose only
    reader is the next gather) stores the f32 result rounded once to nearest
    even: the bits the gather of the f32 map would store."""
    import torch
    from beatlm_b200 import ops
    td = torch.float16 if dt == "f16" else torch.bfloat16
    x = torch.from_numpy(_data(87, side * side * cin)).cuda()
    wt = ops.conv_weights(_data(88, 9 * cin * cout, 1.0 / np.sqrt(9 * cin)), 3, cin, cout,
                          dtype=dt)
    b = torch.from_numpy(_data(89, cout, 0.1)).cuda()
    got = ops.conv2d(x, wt, b, side, side, cin, cout, relu_input=True, out_dtype=dt)
    want = ops.conv2d(x, wt, b, side, side, cin, cout, relu_input=True)
    torch.cuda.synchronize()
    assert got.dtype == td and tuple(got.shape) == (side * side, cout)
    assert torch.equal(got.view(torch.int16), want.to(td).view(torch.int16))


@pytest.mark.parametrize("c,f", [(48, 4), (96, 2)])
def test_reassembly_in_16_bits_equals_the_f32_chain(c, f):
    """A reassembly stage (1x1 projection, then the transposed convolution):
    the projection's map stored in f16 with its padded channels (48 -> the
    64-column GEMM rows, used as they are) or as a 16-bit map (96, gathered as
    it is) gives the same bits as the f32 map narrowed and gathered."""
    import torch
    from beatlm_b200 import ops
    g, dim = 37, 384
    feat = torch.from_numpy(_data(92, g * g * dim)).cuda()
    pw = ops.conv_weights(_data(93, dim * c, 1.0 / np.sqrt(dim)), 1, dim, c)
    pb = torch.zeros(pw.shape[0], dtype=torch.float32, device="cuda")
    pb[:c] = torch.from_numpy(_data(94, c, 0.1)).cuda()
    tw = ops.conv_transpose_weights(_data(95, f * f * c * c, 1.0 / np.sqrt(c)), c, c, f)
    tb = torch.from_numpy(_data(96, c, 0.1)).cuda()
    x16 = ops.conv2d(feat, pw, pb, g, g, dim, c, ksize=1, out_dtype="f16", padded=True)
    x32 = ops.conv2d(feat, pw, pb, g, g, dim, c, ksize=1)
    got = ops.conv_transpose(x16, tw, tb, g, g, c, c, f)
    want = ops.conv_transpose(x32, tw, tb, g, g, c, c, f)
    torch.cuda.synchronize()
    assert tuple(x16.shape) == (g * g, pw.shape[0]) and tuple(x32.shape) == (g * g, c)
    assert not x16[:, c:].float().abs().sum().item()
    assert torch.equal(got, want)


@pytest.mark.parametrize("side,cin,cout,relu", [(518, 32, 32, True), (37, 64, 64, False),
                                                (20, 32, 96, True), (5, 64, 128, True)])
def test_one_channel_1x1_in_the_epilogue_matches_the_oracle(side, cin, cout, relu):
    """The head's last two convolutions as one GEMM (bl_gemm_args.dot_w: the
    3x3 convolution with ReLU, each finished row reduced to one channel in
    the epilogue) against the 3x3 convolution followed by bl_conv1x1_one and
    against the oracle's 1x1 convolution of the same map: within 1e-5
    relative L2 (the sums run in another order); two launches give the same
    bits."""
    import torch
    from beatlm_b200 import ops
    x = torch.from_numpy(_data(97, side * side * cin)).cuda()
    wt = ops.conv_weights(_data(98, 9 * cin * cout, 1.0 / np.sqrt(9 * cin)), 3, cin, cout)
    b = torch.from_numpy(_data(99, cout, 0.1)).cuda()
    w3 = _data(100, cout, 1.0 / np.sqrt(cout))
    w3d, b3 = torch.from_numpy(w3).cuda(), 0.05
    got = ops.conv2d(x, wt, b, side, side, cin, cout, act="relu", dot=(w3d, b3, relu))
    again = ops.conv2d(x, wt, b, side, side, cin, cout, act="relu", dot=(w3d, b3, relu))
    mid = ops.conv2d(x, wt, b, side, side, cin, cout, act="relu")
    two = ops.conv1x1_one(mid, w3d, b3, side * side, cout, relu=relu)
    torch.cuda.synchronize()
    assert got.shape == (side * side,) and torch.equal(got, again)
    assert _rel(got.cpu().numpy(), two.cpu().numpy()) < 1e-5
    want = oracle.conv1x1(mid.cpu().numpy(), w3.reshape(cout, 1), np.array([b3], np.float32),
                          side * side, cout, 1)
    if relu:
        want = np.maximum(want, 0.0)
    assert _rel(got.cpu().numpy(), want) < 1e-5
    with pytest.raises(ValueError):  # an f32 reduction only
        ops.conv2d(x, wt, b, side, side, cin, cout, out_dtype="f16", dot=(w3d, b3, relu))
