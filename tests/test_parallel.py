"""Host logic of the multi-GPU paths, on CPU: the head partition of config 5
and the frame sharding of configs 3-4; with two gloo ranks (world size 2,
127.0.0.1) the exchange of peer-buffer handles and the NCCL-form head
all-gather."""
import os
import socket

import numpy as np
import pytest

from beatlm_b200.parallel import exchange_handles, gather_heads, head_slab, shard_frames


@pytest.mark.parametrize("world", [1, 2, 4, 8, 16])
def test_head_slabs_cover_every_head_once(world):
    heads = 16
    seen = []
    for r in range(world):
        h0, h1 = head_slab(r, world, heads)
        assert h1 - h0 == heads // world
        seen += list(range(h0, h1))
    assert seen == list(range(heads))


def test_head_slab_rejects_uneven_and_bad_ranks():
    with pytest.raises(ValueError, match="divide"):
        head_slab(0, 3, 16)
    with pytest.raises(ValueError):
        head_slab(2, 2, 16)
    with pytest.raises(ValueError):
        head_slab(0, 0, 16)


@pytest.mark.parametrize("frames,world", [(8, 8), (8, 1), (8, 3), (3, 8), (0, 2)])
def test_frame_shards_partition_the_streams(frames, world):
    got = [list(shard_frames(frames, r, world)) for r in range(world)]
    assert sum(got, []) == list(range(frames))
    if frames == world:
        assert all(len(g) == 1 for g in got)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_rank(rank, world, port, t, heads, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = torch.arange(t * heads * 64, dtype=torch.float32).reshape(t, heads, 64)
        h0, h1 = head_slab(rank, world, heads)
        stacked = torch.full((world, t, (h1 - h0) * 64), -1.0)
        stacked[rank].copy_(full[:, h0:h1].reshape(t, -1))  # this rank's heads only
        view = gather_heads(stacked, rank, world)  # [t][world][w], no copy
        ok = view.data_ptr() == stacked.data_ptr() and torch.equal(view.reshape(t, -1),
                                                                    full.reshape(t, -1))
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_head_all_gather_assembles_heads_side_by_side_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_gather_rank, args=(r, world, port, 37, 16, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    results = dict(q.get(timeout=10) for _ in range(world))
    assert results == {0: True, 1: True}


def test_gather_heads_checks_shapes():
    import torch
    with pytest.raises(ValueError):
        gather_heads(torch.zeros(3, 4, 64), 0, 2)


def _handles_rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = bytes((rank * 64 + i) % 251 for i in range(64))  # a 64-byte IPC handle's size
        q.put((rank, exchange_handles(mine, world)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_peer_handles_are_exchanged_in_rank_order_gloo(world):
    """Every rank ends with every rank's handle, rank order, as
    bl_peers_open wants them."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_handles_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    want = b"".join(bytes((r * 64 + i) % 251 for i in range(64)) for r in range(world))
    assert all(got[r] == want for r in range(world))


def test_a_single_rank_exchanges_nothing():
    assert exchange_handles(b"x" * 64, 1) == b"x" * 64
