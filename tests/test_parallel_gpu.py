"""Config 5 split by heads (T=5477, 16 heads): every rank's slab computed
through the C ABI, assembled heads side by side, against the whole op and
the oracle. With one GPU the ranks run one after another on it (no
collective); with two or more GPUs two NCCL processes run the real
all-gather."""
import os
import socket

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

T, H = 5477, 16
ROWS = (2000, 2100)  # oracle sample of query rows (the whole op is ~123 GFLOP in f64)


def _qkv(seed=11):
    return oracle.normal(seed, T * 3 * H * 64).reshape(1, T, 3, H, 64)


def _rounded(qkv):
    q = qkv.copy()
    q[..., :2, :, :] = oracle.round_bf16(q[..., :2, :, :])
    q[..., 2, :, :] = oracle.round_f16(q[..., 2, :, :])
    return q


def _rel(got, want):
    got, want = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
    return float(np.linalg.norm(got - want) / np.linalg.norm(want))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_slabs_assemble_to_the_whole_op(world):
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.parallel import HeadParallelAttention
    qkv = _qkv()
    whole = bl.attention(bl.pack_qkv(qkv, "bf16"), tokens=T, heads=H, qk_dtype="bf16",
                         out_dtype="f16")[0]
    ops = [HeadParallelAttention(T, H, r, world, out_dtype="f16") for r in range(world)]
    stacked = torch.empty_like(ops[0].stacked)
    for r, op in enumerate(ops):
        local = np.ascontiguousarray(qkv[:, :, :, op.h0:op.h1])
        stacked[r].copy_(op.compute(bl.pack_qkv(local, "bf16")))
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    out = stacked.permute(1, 0, 2).reshape(T, H * 64)
    assert _rel(out.float().cpu(), whole.float().cpu()) < 1e-3
    want = oracle.attention(_rounded(qkv)[0].reshape(T, -1), T, H, 64, rows=ROWS)
    rel = _rel(out[ROWS[0]:ROWS[1]].float().cpu(), want)
    print("world %d: rel-L2 vs oracle %.3e" % (world, rel))
    assert rel <= 1e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    import beatlm_b200 as bl
    from beatlm_b200.parallel import HeadParallelAttention
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        qkv = _qkv()
        op = HeadParallelAttention(T, H, rank, world, out_dtype="f16")
        local = np.ascontiguousarray(qkv[:, :, :, op.h0:op.h1])
        for _ in range(2):  # twice: the slots are overwritten, not accumulated
            out = op(bl.pack_qkv(local, "bf16"))
        torch.cuda.synchronize()
        st = bl.status(reset=True).code
        res = out.cpu().float().numpy()
        if rank == 0:
            whole = bl.attention(bl.pack_qkv(qkv, "bf16"), tokens=T, heads=H, qk_dtype="bf16",
                                 out_dtype="f16")[0].float().cpu().numpy()
            q.put((rank, st, _rel(res, whole), res[ROWS[0]:ROWS[1]]))
        else:
            q.put((rank, st, None, None))
    finally:
        dist.destroy_process_group()


def test_head_parallel_all_gather_over_nccl():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, st, rel, rows = q.get(timeout=300)
        res[r] = (st, rel, rows)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    assert res[0][0] == 0 and res[1][0] == 0
    assert res[0][1] < 1e-3
    want = oracle.attention(_rounded(_qkv())[0].reshape(T, -1), T, H, 64, rows=ROWS)
    assert _rel(res[0][2], want) <= 1e-3
