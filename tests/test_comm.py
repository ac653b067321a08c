"""The communicator's failure handling (bl_comm_*), on CPU with fake ranks:
host processes that load a stand-in NCCL (tests/fake_nccl.c) through
BEATLM_B200_NCCL and meet through files in a shared directory. No GPU is
touched: the buffers are host memory.

Covered: the communicator is created non-blocking (the fake refuses a
blocking one); ranks that all join gather each other's bytes, directly and
as a BL_OP_ALLGATHER kernel spec encoded from a program; a rank that never
joins makes init time out and abort; a peer that leaves after joining makes
the next all-gather time out and abort, after which the communicator refuses
work; an error NCCL reports asynchronously aborts too."""
import ctypes
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def fake_nccl(tmp_path_factory):
    out = tmp_path_factory.mktemp("fake_nccl") / "libfakenccl.so"
    subprocess.run(["gcc", "-O1", "-shared", "-fPIC", "-o", str(out),
                    os.path.join(HERE, "fake_nccl.c")], check=True)
    return str(out)


def _rank(rank, world, uid, workdir, lib, script, q):
    os.environ["BEATLM_B200_NCCL"] = lib
    os.environ["FAKE_NCCL_DIR"] = workdir
    for k, v in script.get("env", {}).items():
        os.environ[k] = v
    from beatlm_b200 import _native as N
    from beatlm_b200.comm import Comm
    out = {"rank": rank}
    try:
        if script.get("skip_rank") == rank:  # this rank never joins
            q.put(out)
            return
        c = Comm(uid, world, rank, timeout_ms=script.get("timeout_ms", 5000))
        out["joined"] = True
        if script.get("leave_rank") == rank:  # joins, then goes away
            q.put(out)
            return
        send = (ctypes.c_uint8 * 16)(*[(rank * 16 + i) % 256 for i in range(16)])
        recv = (ctypes.c_uint8 * (16 * world))()
        try:
            if script.get("as_spec"):
                # binding set 1 sends from `other` and receives into `recv2`
                from beatlm_b200.runtime import Kernels, Spec
                other = (ctypes.c_uint8 * 16)(*[(rank * 16 + i + 7) % 256 for i in range(16)])
                recv2 = (ctypes.c_uint8 * (16 * world))()
                k = Kernels([Spec(c.args(ctypes.addressof(send), ctypes.addressof(recv), 16),
                                  "exchange")],
                            sets=[[], [(ctypes.addressof(send), ctypes.addressof(other), 16),
                                       (ctypes.addressof(recv), ctypes.addressof(recv2),
                                        16 * world)]])
                out["len"] = len(k)
                k.encode(0, stream=0)
                k.encode(0, stream=0, set=1)
                out["recv2"] = bytes(recv2)
            else:
                c.all_gather(ctypes.addressof(send), ctypes.addressof(recv), 16)
            out["recv"] = bytes(recv)
        except N.BackendError as e:
            out["error"] = (e.code, str(e))
            out["aborted"] = c.aborted
            try:
                c.all_gather(ctypes.addressof(send), ctypes.addressof(recv), 16)
            except N.BackendError as e2:
                out["after"] = e2.code
        c.close()
    except N.BackendError as e:
        out["error"] = (e.code, str(e))
    q.put(out)


_IDS = [0]


def _run(world, lib, tmp_path, script):
    import torch.multiprocessing as mp
    # the fake's unique id is a token naming its files (made here, so this
    # process never loads the stand-in library)
    _IDS[0] += 1
    uid = ("fake%d_%d" % (os.getpid(), _IDS[0])).encode().ljust(128, b"\0")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, str(tmp_path), lib, script, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        d = q.get(timeout=120)
        res[d["rank"]] = d
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    return res, uid


def _files(tmp_path, uid, what):
    token = uid.split(b"\0")[0].decode()
    return sorted(f for f in os.listdir(tmp_path) if f.startswith(token + "." + what))


def _want(world):
    return bytes((r * 16 + i) % 256 for r in range(world) for i in range(16))


@pytest.mark.parametrize("world", [2, 3])
def test_ranks_that_join_gather_each_others_bytes(fake_nccl, tmp_path, world):
    res, uid = _run(world, fake_nccl, tmp_path, {})
    for r in range(world):
        assert res[r].get("recv") == _want(world), res[r]
    assert _files(tmp_path, uid, "abort") == []
    assert len(_files(tmp_path, uid, "destroy")) == world


def test_the_all_gather_encodes_as_a_kernel_spec(fake_nccl, tmp_path):
    """Set 0 as built; set 1 (a binding set) swaps both buffers."""
    res, _ = _run(2, fake_nccl, tmp_path, {"as_spec": True})
    want2 = bytes((r * 16 + i + 7) % 256 for r in range(2) for i in range(16))
    for r in range(2):
        assert res[r]["len"] == 1 and res[r].get("recv") == _want(2), res[r]
        assert res[r]["recv2"] == want2


def test_a_rank_that_never_joins_times_out_and_aborts(fake_nccl, tmp_path):
    from beatlm_b200 import _native as N
    res, uid = _run(2, fake_nccl, tmp_path, {"skip_rank": 1, "timeout_ms": 300})
    code, msg = res[0]["error"]
    assert code == N.BL_ERR_TIMEOUT and "init" in msg and "aborted" in msg
    assert _files(tmp_path, uid, "abort") == [uid.split(b"\0")[0].decode() + ".abort.0"]


def test_a_peer_that_leaves_times_out_the_next_collective(fake_nccl, tmp_path):
    from beatlm_b200 import _native as N
    res, uid = _run(2, fake_nccl, tmp_path, {"leave_rank": 1, "timeout_ms": 400})
    assert res[1]["joined"]
    code, msg = res[0]["error"]
    assert code == N.BL_ERR_TIMEOUT and "all-gather" in msg
    assert res[0]["aborted"] is True
    assert res[0]["after"] == N.BL_ERR_COMM  # an aborted communicator refuses work
    assert len(_files(tmp_path, uid, "abort")) == 1


def test_an_asynchronous_nccl_error_aborts(fake_nccl, tmp_path):
    from beatlm_b200 import _native as N
    res, uid = _run(2, fake_nccl, tmp_path, {"env": {"FAKE_NCCL_ASYNC_ERROR": "6"}})
    for r in range(2):
        code, msg = res[r]["error"]
        assert code == N.BL_ERR_COMM and "remote process" in msg
    assert len(_files(tmp_path, uid, "abort")) == 2


def test_without_nccl_the_calls_say_so(tmp_path):
    """A library path that does not load: bl_comm_available is 0 and the
    calls return BL_ERR_UNSUPPORTED (in a child process: NCCL is looked up
    once per process)."""
    code = ("import os; os.environ['BEATLM_B200_NCCL'] = %r\n"
            "from beatlm_b200 import _native as N, comm\n"
            "assert not comm.available()\n"
            "try:\n    comm.unique_id()\nexcept N.BackendError as e:\n"
            "    assert e.code == 2 and 'not loadable' in str(e), e\n    print('ok')\n"
            % str(tmp_path / "missing.so"))
    r = subprocess.run(["python", "-c", code], capture_output=True, text=True,
                       cwd=os.path.dirname(HERE))
    assert r.stdout.strip() == "ok", r.stdout + r.stderr
