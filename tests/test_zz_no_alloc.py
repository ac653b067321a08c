"""bl_attention_noalloc: the attention entry point for callers that cannot
allocate device memory (a host whose device memory is fixed by a static plan
and that must not allocate in its frame loop, or an FFI host without a CUDA
allocator). It keeps the split-key scratch in a static array inside the
library instead of a caller-owned workspace.

Called through the C ABI twice in a row (the array keeps the previous call's
contents, so the second call checks that the counters are cleared) and
compared with bl_attention given a workspace: the same kernel, split count and
combine formula, so the two agree to relative L2 <= 1e-6 (a stale counter or a
stale partial on the second call would show far above that). Both are also
held to the attention tolerance against the oracle (relative L2 <= 1e-3), and
the second call must leave the device's free memory and torch's allocator
untouched. This file sorts last so a run that stops at the first failure has
run every other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

REL_SAME = 1e-6   # against bl_attention with a workspace: same kernel and formula
REL_L2 = 1e-3     # against the oracle: the attention tolerance


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
    want_host = want.cpu().numpy()
    # the oracle reads the same 16-bit values the kernel reads
    ref_in = qkv.copy()
    ref_in[:, :, :2] = oracle.round_bf16(ref_in[:, :, :2])
    ref_in[:, :, 2:] = oracle.round_f16(ref_in[:, :, 2:])
    ref = oracle.attention(ref_in.reshape(t, -1), t, h, 64)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    outs = [torch.full((1, t, h * 64), float("nan"), dtype=torch.float32, device="cuda")
            for _ in range(2)]
    torch.cuda.synchronize()
    for call, got in enumerate(outs):
        a = ops.attention_args(dev, tokens=t, heads=h, out=got, qk_dtype="bf16",
                               kv_splits=kv_splits)
        if call == 1:  # after the first call's set-up: nothing may be allocated
            free0, _ = torch.cuda.mem_get_info()
            alloc0 = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        N.check(N.lib().bl_attention_noalloc(ctypes.byref(a), stream))
        torch.cuda.synchronize()
        if call == 1:
            free1, _ = torch.cuda.mem_get_info()
            alloc1 = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
            assert free1 == free0, "the second call changed free device memory by %d bytes" % (
                free0 - free1)
            assert alloc1 == alloc0
        assert bl.status(reset=True).code == 0
        host = got.cpu().numpy()
        assert np.isfinite(host).all()
        rel = _rel(host, want_host)
        rel_ref = _rel(host, ref)
        print("no-alloc call %d (kv_splits=%d): rel-L2 %.3e vs workspace entry, %.3e vs oracle"
              % (call, kv_splits, rel, rel_ref))
        assert rel <= REL_SAME
        assert rel_ref <= REL_L2


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
