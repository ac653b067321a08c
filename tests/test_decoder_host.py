"""Host-side structure of the DPT head (model.Decoder) without a GPU: the
launch count the bench reports for the depth model."""
import torch

from beatlm_b200 import model


def test_head_launch_count_follows_its_structure():
    """DPT-S (neck 48/96/192/384): projections and necks 16, the transposed
    convolutions 2 (48 channels, from the projection's rows) and 3 (96), the
    strided one 2; fusion 6 + 3 x 10; head 5: 64 launches."""
    dc = model.DecoderConfig()
    d = model.Decoder.__new__(model.Decoder)
    d.dcfg = dc
    d.stages = [{"c": c, "resample": rs, "proj": (torch.empty((-(-c // 32) * 32, 64)),)}
                for c, rs in zip(dc.neck, dc.reassemble)]
    d.fusion = [None] * len(dc.neck)
    assert d.launches_per_frame() == 64


def test_16bit_map_arguments_are_checked_before_any_launch():
    """Malformed 16-bit maps are errors on the host (no device needed): a map
    of another dtype than the weights, rows of the wrong shape, a 16-bit map
    for the implicit convolution, and a gather of a map of a third dtype."""
    import pytest
    from beatlm_b200 import ops
    w = torch.zeros((64, 64), dtype=torch.float16)  # 1x1, 64 -> 64, k_pad 64
    with pytest.raises(ValueError):
        ops.conv2d(torch.zeros((16, 64), dtype=torch.bfloat16), w, None, 4, 4, 64, 64, ksize=1)
    with pytest.raises(ValueError):
        ops.conv2d(torch.zeros((15, 64), dtype=torch.float16), w, None, 4, 4, 64, 64, ksize=1)
    with pytest.raises(ValueError):
        ops.conv2d(torch.zeros((16, 64), dtype=torch.float16), w, None, 4, 4, 64, 64, ksize=1,
                   implicit=True)
    with pytest.raises(ValueError):
        ops.im2col(torch.zeros((16, 64), dtype=torch.bfloat16), 4, 4, 64, 3, dtype="f16")
    with pytest.raises(ValueError):
        ops.conv_transpose(torch.zeros((16, 64), dtype=torch.bfloat16),
                           torch.zeros((16 * 48, 64), dtype=torch.float16), None, 4, 4, 48, 48, 4)


def test_row_reduction_arguments_are_checked_on_the_host():
    """gemm_args(dot=...) takes f32 weights of n values and an f32 output of m
    values; anything else is an error before any launch, and a valid one
    sets the reduction's fields with out_ld left to the library."""
    import pytest
    from beatlm_b200 import ops
    w = torch.zeros((32, 64), dtype=torch.float16)  # n = 32, k = 64
    a = torch.zeros((10, 64), dtype=torch.float16)
    out = torch.zeros(10, dtype=torch.float32)
    dw = torch.ones(32)
    g = ops.gemm_args(w, a=a, out=out, dot=(dw, 0.5, True))
    assert g.dot_w == dw.data_ptr()
    assert g.dot_bias == 0.5 and g.dot_act == 1 and g.out_ld == 0
    with pytest.raises(ValueError):
        ops.gemm_args(w, a=a, out=out, dot=(torch.ones(31), 0.0, False))
    with pytest.raises(ValueError):
        ops.gemm_args(w, a=a, out=torch.zeros(9), dot=(torch.ones(32), 0.0, False))
    with pytest.raises(ValueError):
        ops.gemm_args(w, a=a, out=out, dot=(torch.ones(32, dtype=torch.float16), 0.0, False))


def test_head_launch_count_equals_the_launches_a_pass_makes(monkeypatch):
    """One DPT-S head pass at 518 px with the library replaced by a recorder
    (CPU tensors, nothing computed): the kernel entry points it calls are
    exactly launches_per_frame(), the figure the bench reports."""
    import ctypes
    import functools
    from beatlm_b200 import _native, ops
    launching = {"bl_im2col", "bl_gemm", "bl_blocks_to_map", "bl_resize_bilinear",
                 "bl_resize_bilinear_rows16", "bl_conv1x1_one", "bl_conv3x3"}
    calls = []

    class Recorder:
        def __getattr__(self, name):
            def call(*args):
                calls.append(name)
                return 0
            return call

    monkeypatch.setattr(_native, "lib", lambda: Recorder())
    monkeypatch.setattr(ops, "_stream_ptr", lambda stream: ctypes.c_void_p(0))
    monkeypatch.setattr(ops, "conv_weights", functools.partial(ops.conv_weights, device="cpu"))
    cfg, dc = model.ViTConfig.small(), model.DecoderConfig()
    d = model.Decoder(cfg, dc, model.decoder_weights_random(cfg, dc, seed=0), device="cpu")
    feats = [torch.zeros((cfg.grid * cfg.grid, cfg.dim)) for _ in dc.neck]
    depth = d.forward(feats)
    side = cfg.grid * cfg.patch
    assert tuple(depth.shape) == (side, side)
    assert sum(1 for c in calls if c in launching) == d.launches_per_frame() == 64
    assert "bl_conv1x1_one" not in calls  # the last 1x1 runs in the GEMM epilogue
