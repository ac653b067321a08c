"""The fused attention kernel (through the C ABI) against the CPU oracle's
scores -> scale -> softmax -> values chain (reference.rs:437-494).

Tolerance (stated by the task): relative L2 <= 1e-3 against the oracle's f32
result; max-abs is reported. The oracle reads the same 16-bit-rounded Q/K/V
values the kernel reads (Q/K in f16 or bf16, V in f16), so the comparison
measures the kernel's arithmetic, not input quantisation."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3


def _rounded(qkv, qk_dtype):
    q = qkv.copy()
    rnd = oracle.round_bf16 if qk_dtype == "bf16" else oracle.round_f16
    q[..., :2, :, :] = rnd(q[..., :2, :, :])
    q[..., 2, :, :] = oracle.round_f16(q[..., 2, :, :])
    return q


def _errors(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    return rel, float(np.max(np.abs(got - want)))


def _run(t, h, seed, qk_dtype="f16", out_dtype="f32", batch=1, std=1.0, rows=None,
         head_range=None):
    import torch
    import beatlm_b200 as bl
    qkv = oracle.normal(seed, batch * t * 3 * h * 64, 0.0, std).reshape(batch, t, 3, h, 64)
    dev = bl.pack_qkv(qkv, qk_dtype)
    out = bl.attention(dev, tokens=t, heads=h, batch=batch, qk_dtype=qk_dtype,
                       out_dtype=out_dtype, rows=rows, head_range=head_range)
    torch.cuda.synchronize()
    st = bl.status(reset=True)
    assert st.code == 0, (hex(st.code), st.block, st.where)
    return _rounded(qkv, qk_dtype), out.float().cpu().numpy()


@pytest.mark.parametrize("t", [1, 17, 64, 128, 129, 300, 1370])
@pytest.mark.parametrize("qk_dtype", ["f16", "bf16"])
def test_attention_matches_the_oracle(t, qk_dtype):
    h = 6
    ref_in, got = _run(t, h, seed=100 + t, qk_dtype=qk_dtype)
    want = oracle.attention(ref_in[0].reshape(t, 3 * h * 64), t, h, 64)
    rel, mx = _errors(got[0], want)
    print("T=%d %s: rel-L2 %.3e max-abs %.3e" % (t, qk_dtype, rel, mx))
    assert rel <= REL_L2 and mx < 5e-3


@pytest.mark.parametrize("t,splits,qt", [(300, 2, 2), (1370, 3, 2), (1370, 0, 2), (1370, 11, 2),
                                         (129, 2, 2), (5477, 0, 2), (1370, 3, 1), (1370, 0, 1),
                                         (5477, 0, 1)])
def test_key_splits_match_the_oracle(t, splits, qt):
    """Keys split across CTAs, combined by the last CTA of each tile group
    through a caller-owned workspace; repeated calls reuse it (its counters
    return to zero). ``qt`` query tiles of 128 rows per CTA."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    h = 6
    qkv = oracle.normal(300 + t, t * 3 * h * 64).reshape(1, t, 3, h, 64)
    dev = bl.pack_qkv(qkv, "bf16")
    out = torch.zeros((1, t, h * 64), dtype=torch.float32, device="cuda")
    args = ops.attention_args(dev, tokens=t, heads=h, out=out, qk_dtype="bf16",
                              kv_splits=splits, query_tiles=qt)
    nbytes = ops.attention_workspace_bytes(args)
    ws = ops.attention_workspace(nbytes)
    for _ in range(2):
        out.zero_()
        bl.attention(dev, tokens=t, heads=h, qk_dtype="bf16", out=out, workspace=ws,
                     kv_splits=splits, query_tiles=qt)
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    units = h * -(-t // (128 * qt))  # one counter per (head, query group), at the end
    assert nbytes == 0 or not ws[nbytes - 4 * units:nbytes].any()  # counters back at zero
    rows = (0, t) if t < 2000 else (1000, 1130)
    want = oracle.attention(_rounded(qkv, "bf16")[0].reshape(t, -1), t, h, 64, rows=rows)
    rel, mx = _errors(out.cpu().numpy()[0][rows[0]:rows[1]], want)
    print("T=%d splits=%d (workspace %d B): rel-L2 %.3e" % (t, splits, nbytes, rel))
    assert rel <= REL_L2


def test_split_workspace_too_small_is_an_error():
    import torch
    import beatlm_b200 as bl
    t, h = 1370, 6
    dev = bl.pack_qkv(np.zeros((1, t, 3, h, 64), np.float32), "f16")
    ws = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(bl.BackendError, match="workspace"):
        bl.attention(dev, tokens=t, heads=h, workspace=ws, kv_splits=4)


@pytest.mark.parametrize("out_dtype", ["f16", "bf16"])
def test_16bit_outputs(out_dtype):
    t, h = 257, 2
    ref_in, got = _run(t, h, seed=7, out_dtype=out_dtype)
    want = oracle.attention(ref_in[0].reshape(t, -1), t, h, 64)
    rel, mx = _errors(got[0], want)
    assert rel <= (4e-3 if out_dtype == "bf16" else REL_L2), rel


def test_batch_and_head_range():
    t, h, b = 200, 4, 3
    ref_in, got = _run(t, h, seed=21, batch=b, head_range=(1, 3))
    for i in range(b):
        want = oracle.attention(ref_in[i].reshape(t, -1), t, h, 64).reshape(t, h, 64)
        g = got[i].reshape(t, 3, 64)   # heads 1..2 at columns 64.. (out_head_base 0)
        rel, _ = _errors(g[:, 1:3], want[:, 1:3])
        assert rel <= REL_L2
        assert not g[:, 0].any()


def test_large_scores_stay_finite_and_match():
    """Scores of spread ~16 (x4 inputs): the lazy rescale path runs."""
    t, h = 700, 2
    ref_in, got = _run(t, h, seed=33, std=2.0)
    want = oracle.attention(ref_in[0].reshape(t, -1), t, h, 64)
    assert np.isfinite(got).all()
    rel, mx = _errors(got[0], want)
    assert rel <= REL_L2, rel


def test_row_parts_cover_the_output_and_equal_the_whole():
    """Program::split (kernel.rs:2384): parts over query rows, each computed by
    its own launch, together equal the whole kernel's result."""
    import torch
    import beatlm_b200 as bl
    t, h = 1370, 6
    qkv = oracle.normal(5, t * 3 * h * 64).reshape(1, t, 3, h, 64)
    dev = bl.pack_qkv(qkv, "f16")
    for splits in (1, 3):  # unsplit, and keys split over a cluster of 3
        whole = bl.attention(dev, tokens=t, heads=h, kv_splits=splits)
        for parts in (3, 7, 22, 200):
            bounds = [round(i * t / min(parts, t)) for i in range(min(parts, t) + 1)]
            out = torch.zeros_like(whole)
            for r0, r1 in zip(bounds[:-1], bounds[1:]):
                if r1 > r0:
                    bl.attention(dev, tokens=t, heads=h, out=out, rows=(r0, r1),
                                 kv_splits=splits)
            torch.cuda.synchronize()
            assert torch.equal(out, whole), (splits, parts)
    assert bl.status(reset=True).code == 0


@pytest.mark.parametrize("splits", [2, 3, 4, 8])
def test_cluster_combine_equals_the_workspace_combine(splits):
    """Without a workspace the key splits of a query group form a thread-block
    cluster and combine in distributed shared memory; with one they combine
    through it. Same partials, same formula: the results agree, and both meet
    the oracle."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    t, h = 1370, 6
    qkv = oracle.normal(600 + splits, t * 3 * h * 64).reshape(1, t, 3, h, 64)
    dev = bl.pack_qkv(qkv, "bf16")
    clus = bl.attention(dev, tokens=t, heads=h, qk_dtype="bf16", kv_splits=splits)
    a = ops.attention_args(dev, tokens=t, heads=h, out=clus, qk_dtype="bf16", kv_splits=splits)
    ws = ops.attention_workspace(ops.attention_workspace_bytes(a))
    glob = bl.attention(dev, tokens=t, heads=h, qk_dtype="bf16", kv_splits=splits, workspace=ws)
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    rel, mx = _errors(clus.cpu().numpy(), glob.cpu().numpy())
    assert rel < 1e-6, rel
    want = oracle.attention(_rounded(qkv, "bf16")[0].reshape(t, -1), t, h, 64)
    rel, mx = _errors(clus.cpu().numpy()[0], want)
    assert rel <= REL_L2


def test_hires_rows_sample():
    """Config 5 shape (T=5477, H=16) on a sample of query rows."""
    t, h = 5477, 16
    ref_in, got = _run(t, h, seed=55, rows=(2048, 2048 + 130))
    want = oracle.attention(ref_in[0].reshape(t, -1), t, h, 64, rows=(2048, 2048 + 130))
    rel, mx = _errors(got[0][2048:2048 + 130], want)
    assert rel <= REL_L2, rel


@pytest.mark.parametrize("t,splits,std,out_dtype", [
    (1, 1, 1.0, "f32"), (129, 1, 1.0, "f32"), (300, 2, 1.0, "bf16"), (700, 1, 2.0, "f32"),
    (1370, 1, 1.0, "f32"), (1370, 2, 1.0, "bf16"), (1370, 3, 1.0, "f16"), (1370, 8, 1.0, "f32")])
def test_one_query_tile_per_cta_equals_two(t, splits, std, out_dtype):
    """One 128-row query tile per CTA (8 warps, two S buffers) against two
    (12 warps, three S buffers): a row's arithmetic depends on the key splits
    only, so with the same splits the outputs are the same bits, in both
    combine forms; and the one-tile kernel meets the oracle."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    h = 6
    qkv = oracle.normal(900 + t + splits, t * 3 * h * 64, 0.0, std).reshape(1, t, 3, h, 64)
    dev = bl.pack_qkv(qkv, "bf16")
    run = lambda qt, ws=None: bl.attention(dev, tokens=t, heads=h, qk_dtype="bf16",
                                           out_dtype=out_dtype, kv_splits=splits,
                                           query_tiles=qt, workspace=ws)
    two, one = run(2), run(1)
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    assert torch.equal(one, two)
    if splits > 1:
        a = ops.attention_args(dev, tokens=t, heads=h, out=one, qk_dtype="bf16",
                               kv_splits=splits, query_tiles=1)
        one_ws = run(1, ops.attention_workspace(ops.attention_workspace_bytes(a)))
        torch.cuda.synchronize()
        assert bl.status(reset=True).code == 0
        assert torch.equal(one_ws, one)
    want = oracle.attention(_rounded(qkv, "bf16")[0].reshape(t, -1), t, h, 64)
    rel, mx = _errors(one.float().cpu().numpy()[0], want)
    print("T=%d splits=%d std=%g %s: QT=1 rel-L2 %.3e max-abs %.3e" % (t, splits, std, out_dtype,
                                                                      rel, mx))
    assert rel <= (4e-3 if out_dtype == "bf16" else REL_L2), rel


def test_query_tiles_beyond_two_are_rejected():
    import beatlm_b200 as bl
    dev = bl.pack_qkv(np.zeros((1, 64, 3, 2, 64), np.float32), "f16")
    with pytest.raises(bl.BackendError, match="query tiles"):
        bl.attention(dev, tokens=64, heads=2, query_tiles=3)


def test_mixed_grid_rows_equal_their_uniform_launches():
    """Config 5's shape (T=5477, H=16): the automatic choice is a mixed grid
    (the query groups that fill whole waves of clusters unsplit, the rest
    split), so the last wave is short. Each row must then equal, bit for bit,
    the uniform launch with its own group's split count (1 or the tail's),
    and the output meets the oracle on sampled rows of both kinds."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import ops
    t, h = 5477, 16
    qkv = oracle.normal(4242, t * 3 * h * 64).reshape(1, t, 3, h, 64)
    dev = bl.pack_qkv(qkv, "bf16")
    out = torch.zeros((1, t, h * 64), dtype=torch.float32, device="cuda")
    qt, splits, unsplit = ops.attention_choice(
        ops.attention_args(dev, tokens=t, heads=h, out=out, qk_dtype="bf16"))
    print("T=%d H=%d: %d query tiles per CTA, %d groups unsplit, the rest split %d ways"
          % (t, h, qt, unsplit, splits))
    assert unsplit > 0 and splits > 1  # the tail of 352 groups on 148 SMs
    mixed = bl.attention(dev, tokens=t, heads=h, qk_dtype="bf16", out=out)
    one = bl.attention(dev, tokens=t, heads=h, qk_dtype="bf16", kv_splits=1, query_tiles=qt)
    many = bl.attention(dev, tokens=t, heads=h, qk_dtype="bf16", kv_splits=splits,
                        query_tiles=qt)
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    rows = 128 * qt
    groups = -(-t // rows)
    got = mixed.view(t, h, 64)
    for u in range(groups * h):
        head, g = divmod(u, groups)
        r0, r1 = g * rows, min(t, (g + 1) * rows)
        want = (one if u < unsplit else many).view(t, h, 64)[r0:r1, head]
        assert torch.equal(got[r0:r1, head], want), u
    first_split_head, g = divmod(unsplit, groups)  # the first split group
    for head, (r0, r1) in ((0, (0, 64)), (first_split_head, (g * rows, g * rows + 64))):
        ref = oracle.attention(_rounded(qkv, "bf16")[0].reshape(t, -1), t, h, 64, rows=(r0, r1))
        rel, _ = _errors(got[r0:r1, head].cpu().numpy(),
                         ref.reshape(r1 - r0, h, 64)[:, head])
        assert rel <= REL_L2, (head, rel)
