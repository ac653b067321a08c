"""Config 5 split by heads (T=5477, 16 heads): every rank's slab computed
through the C ABI and assembled heads side by side, against the whole op and
the oracle.

With one GPU no two launches ever wait on each other: the ranks' slabs run
one after another with no exchange, and the fused exchange
(bl_attention_peers) runs as rank 0 of two with rank 1's buffer attached
from local memory and rank 1's arrival written by the host, so the single
launch's wait is satisfied (or, in the expiry case, left unsatisfied until
its bounded wait gives up). With two or more GPUs two NCCL processes run the
real exchange, both the fused form and the NCCL all-gather form, and the C
ABI's non-blocking communicator (bl_comm) over real NCCL."""
import ctypes
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
    ops = [HeadParallelAttention(T, H, r, world, out_dtype="f16", exchange="nccl")
           for r in range(world)]
    stacked = torch.empty_like(ops[0].stacked)
    for r, op in enumerate(ops):
        local = np.ascontiguousarray(qkv[:, :, :, op.h0:op.h1])
        stacked[r].copy_(op.compute_local(bl.pack_qkv(local, "bf16")))
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    out = stacked.permute(1, 0, 2).reshape(T, H * 64)
    assert _rel(out.float().cpu(), whole.float().cpu()) < 1e-3
    want = oracle.attention(_rounded(qkv)[0].reshape(T, -1), T, H, 64, rows=ROWS)
    rel = _rel(out[ROWS[0]:ROWS[1]].float().cpu(), want)
    print("world %d: rel-L2 vs oracle %.3e" % (world, rel))
    assert rel <= 1e-3


def test_fused_exchange_stores_into_every_rank_and_bounds_its_wait():
    """bl_attention_peers as rank 0 of 2 (heads 0-7), rank 1's buffer a local
    zeroed buffer attached in its place.

    1. Rank 1's arrival for launch 1 is written by the host first: the launch
       completes; its rows land in both buffers' slot 1 (this rank's columns
       0-511 of [T][1024]), bit-equal to bl_attention of the same 8 heads and
       within 1e-3 of the oracle; its flag reached rank 1's header and its
       own.
    2. Launch 2 with no arrival from rank 1 and a 1 ms wait limit: the kernel
       returns by itself, the status word says peer timeout (0x60) for rank 1,
       and the context stays usable.
    3. Launch 3 with rank 1's arrival written: complete and correct again."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import _native as N
    from beatlm_b200 import ops
    from beatlm_b200.parallel import PeerBuffers, device_view
    L = N.lib()
    qkv = _qkv(seed=21)
    whole = bl.attention(bl.pack_qkv(qkv, "bf16"), tokens=T, heads=H, qk_dtype="bf16",
                         out_dtype="f16")[0]
    local = bl.pack_qkv(np.ascontiguousarray(qkv[:, :, :, :8]), "bf16")
    # the same 8 heads through bl_attention: the same grid and key splits, so
    # the rows the exchange stores must be these bits
    same = bl.attention(local, tokens=T, heads=8, qk_dtype="bf16", out_dtype="f16")[0]
    slot_bytes = T * H * 64 * 2
    peers = PeerBuffers(0, 2, slot_bytes)
    other = torch.zeros(PeerBuffers.buffer_bytes(slot_bytes), dtype=torch.uint8, device="cuda")
    peers.attach(1, other)
    mine = L.bl_peers_slot(peers._h, 0) - 256  # this rank's header
    stride = (slot_bytes + 255) // 256 * 256
    flags = device_view(mine, (64,), torch.float16).view(torch.int32)  # 256-byte header
    dummy = torch.empty((T, H * 64), dtype=torch.float16, device="cuda")
    a = ops.attention_args(local, tokens=T, heads=8, out=dummy, qk_dtype="bf16",
                           out_dtype="f16", out_row_stride=H * 64)
    slot = ctypes.c_uint32()
    try:
        for launch in (1, 2, 3):
            assert peers.next_epoch() == launch
            arrives = launch != 2
            if arrives:
                flags[1] = launch  # rank 1 "arrived" for this launch
            else:
                N.check(L.bl_set_wait_limit(2_000_000))  # ~1 ms of SM clock
            torch.cuda.synchronize()
            N.check(L.bl_attention_peers(ctypes.byref(a), peers._h, 0, ctypes.byref(slot), None))
            torch.cuda.synchronize()
            N.check(L.bl_set_wait_limit(0))
            st = bl.status(reset=True)
            assert slot.value == launch % 2
            if not arrives:
                assert st.code == 0x60 and st.where == 1, (hex(st.code), st.where)
                continue
            assert st.code == 0, hex(st.code)
            out = peers.slot(slot.value, (T, H * 64), torch.float16)
            theirs = device_view(other.data_ptr() + 256 + slot.value * stride, (T, H * 64),
                                 torch.float16)
            assert torch.equal(out[:, :512], theirs[:, :512])
            assert torch.equal(out[:, :512], same)
            rel = _rel(out[:, :512].float().cpu(), whole[:, :512].float().cpu())
            assert rel < 1e-3, rel  # the 16-head launch splits its keys differently
            want = oracle.attention(_rounded(qkv)[0].reshape(T, -1), T, H, 64, rows=ROWS)
            want = want.reshape(ROWS[1] - ROWS[0], H * 64)[:, :512]
            rel_o = _rel(out[ROWS[0]:ROWS[1], :512].float().cpu(), want)
            print("fused exchange launch %d: rel-L2 vs whole %.2e, vs oracle %.2e"
                  % (launch, rel, rel_o))
            assert rel_o <= 1e-3
            theirs_flags = device_view(other.data_ptr(), (64,), torch.float16).view(torch.int32)
            assert int(theirs_flags[0]) == launch  # this rank's arrival reached rank 1
            assert int(flags[0]) == launch  # and its own
    finally:
        L.bl_set_wait_limit(0)
        torch.cuda.synchronize()
        peers.close()


def test_peer_attention_rejects_what_it_cannot_do():
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import _native as N
    from beatlm_b200 import ops
    from beatlm_b200.parallel import PeerBuffers
    L = N.lib()
    peers = PeerBuffers(0, 2, 1370 * 384 * 2)
    qkv = torch.zeros((1370, 3 * 6 * 64), dtype=torch.int16, device="cuda")
    out = torch.zeros((1370, 384), dtype=torch.float16, device="cuda")
    a = ops.attention_args(qkv, tokens=1370, heads=6, out=out, out_dtype="f16")
    try:
        with pytest.raises(bl.BackendError, match="not mapped"):
            N.check(L.bl_attention_peers(ctypes.byref(a), peers._h, 0, None, None))
        peers.attach(1, torch.zeros(PeerBuffers.buffer_bytes(1370 * 384 * 2), dtype=torch.uint8,
                                    device="cuda"))
        a.out_dtype = N.BL_F32
        with pytest.raises(bl.BackendError, match="16-bit"):
            N.check(L.bl_attention_peers(ctypes.byref(a), peers._h, 0, None, None))
        a.out_dtype = N.BL_F16
        with pytest.raises(bl.BackendError, match="column"):
            N.check(L.bl_attention_peers(ctypes.byref(a), peers._h, 64, None, None))
        assert peers.next_epoch() == 1  # nothing was launched
    finally:
        peers.close()


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
        res = {}
        for exchange in ("peers", "nccl"):
            op = HeadParallelAttention(T, H, rank, world, out_dtype="f16", exchange=exchange)
            local = bl.pack_qkv(np.ascontiguousarray(qkv[:, :, :, op.h0:op.h1]), "bf16")
            for _ in range(3):  # both slots, then the first again: overwritten, not accumulated
                out = op(local)
            torch.cuda.synchronize()
            res[exchange] = (bl.status(reset=True).code,
                             out.reshape(T, H * 64).cpu().float().numpy())
            dist.barrier()
            op.close()
        # the C ABI's own non-blocking communicator over real NCCL: an
        # all-gather of device bytes, once directly and once as a kernel spec
        from beatlm_b200 import comm as C
        from beatlm_b200.parallel import exchange_handles
        from beatlm_b200.runtime import Kernels, Spec
        uid = exchange_handles(C.unique_id() if rank == 0 else bytes(128), world)[:128]
        c = C.Comm(uid, world, rank, timeout_ms=30000)
        send = torch.full((4096,), rank + 1, dtype=torch.uint8, device="cuda")
        recv = torch.zeros(world * 4096, dtype=torch.uint8, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        c.all_gather(send.data_ptr(), recv.data_ptr(), 4096, stream=stream)
        torch.cuda.synchronize()
        comm_ok = all(bool((recv[r * 4096:(r + 1) * 4096] == r + 1).all()) for r in range(world))
        recv.zero_()
        k = Kernels([Spec(c.args(send.data_ptr(), recv.data_ptr(), 4096), "exchange")])
        k.encode(0, stream=stream)
        torch.cuda.synchronize()
        comm_ok = comm_ok and all(bool((recv[r * 4096:(r + 1) * 4096] == r + 1).all())
                                  for r in range(world))
        k.close()
        c.close()
        res["comm"] = (0 if comm_ok else 1, None)
        if rank == 0:
            whole = bl.attention(bl.pack_qkv(qkv, "bf16"), tokens=T, heads=H, qk_dtype="bf16",
                                 out_dtype="f16")[0].float().cpu().numpy()
            q.put((rank, {k: (st, None if o is None else _rel(o, whole),
                              None if o is None else o[ROWS[0]:ROWS[1]])
                          for k, (st, o) in res.items()}))
        else:
            q.put((rank, {k: (st, None, None) for k, (st, o) in res.items()}))
    finally:
        dist.destroy_process_group()


def test_head_parallel_exchange_over_nvlink():
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
        r, d = q.get(timeout=300)
        res[r] = d
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    assert res[0]["comm"][0] == 0 and res[1]["comm"][0] == 0  # bl_comm all-gathers
    want = oracle.attention(_rounded(_qkv())[0].reshape(T, -1), T, H, 64, rows=ROWS)
    for exchange in ("peers", "nccl"):
        assert res[0][exchange][0] == 0 and res[1][exchange][0] == 0, exchange
        assert res[0][exchange][1] < 1e-3, exchange
        rel = _rel(res[0][exchange][2], want)
        print("%s exchange over 2 GPUs: rel-L2 vs oracle %.3e" % (exchange, rel))
        assert rel <= 1e-3
