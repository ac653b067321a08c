"""bl_attention_noalloc: the attention entry point for callers that cannot
allocate device memory (a host whose device memory is fixed by a static plan
and that must not allocate in its frame loop, or an FFI host without a CUDA
allocator). It keeps the split-key scratch in a static array inside the
library instead of a caller-owned workspace.

Called through the C ABI twice in a row (the array keeps the previous call's
contents, so the second call checks that the counters are cleared) and
compared with bl_attention given a workspace, within the attention tolerance
used everywhere else (relative L2 <= 1e-3). This file sorts last so a run that
stops at the first failure has run every other test; it also passes alone in
a fresh process."""
import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3


def _rel(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    return float(np.linalg.norm(got - want) / np.linalg.norm(want))


@pytest.mark.parametrize("kv_splits", [4, 0])
def test_no_alloc_attention_matches_the_workspace_entry_point(kv_splits):
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import _native as N
    from beatlm_b200 import ops
    t, h = 1370, 6
    qkv = oracle.normal(77, t * 3 * h * 64).reshape(1, t, 3, h, 64)
    dev = bl.pack_qkv(qkv, "bf16")
    want = torch.zeros((1, t, h * 64), dtype=torch.float32, device="cuda")
    args = ops.attention_args(dev, tokens=t, heads=h, out=want, qk_dtype="bf16",
                              kv_splits=kv_splits)
    assert ops.attention_workspace_bytes(args) > 0  # this case splits the keys
    ws = ops.attention_workspace(ops.attention_workspace_bytes(args))
    bl.attention(dev, tokens=t, heads=h, qk_dtype="bf16", out=want, workspace=ws,
                 kv_splits=kv_splits)
    torch.cuda.synchronize()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        got = torch.full((1, t, h * 64), float("nan"), dtype=torch.float32, device="cuda")
        a = ops.attention_args(dev, tokens=t, heads=h, out=got, qk_dtype="bf16",
                               kv_splits=kv_splits)
        N.check(N.lib().bl_attention_noalloc(ctypes.byref(a), stream))
        torch.cuda.synchronize()
        assert bl.status(reset=True).code == 0
        rel = _rel(got.cpu().numpy(), want.cpu().numpy())
        print("no-alloc call %d (kv_splits=%d): rel-L2 vs workspace entry %.3e" % (
            call, kv_splits, rel))
        assert np.isfinite(got.cpu().numpy()).all()
        assert rel <= REL_L2


def test_no_alloc_rejects_scratch_beyond_its_maximum():
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import _native as N
    from beatlm_b200 import ops
    t, h, batch = 1370, 6, 4
    dev = torch.zeros((batch, t, 3 * h * 64), dtype=torch.int16, device="cuda")
    out = torch.zeros((batch, t, h * 64), dtype=torch.float32, device="cuda")
    a = ops.attention_args(dev, tokens=t, heads=h, batch=batch, out=out, kv_splits=11)
    with pytest.raises(bl.BackendError, match="static scratch"):
        N.check(N.lib().bl_attention_noalloc(ctypes.byref(a), None))
