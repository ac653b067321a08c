"""The non-blocking NCCL communicator of the C ABI (``bl_comm_*``): every wait
bounded by the communicator's timeout, the communicator aborted when it runs
out. A host without another runtime drives collectives through it; the
unique id travels between ranks by any host channel."""
from __future__ import annotations

import ctypes

from . import _native as N


def available() -> bool:
    return bool(N.lib().bl_comm_available())


def unique_id() -> bytes:
    buf = (ctypes.c_uint8 * N.COMM_ID_BYTES)()
    N.check(N.lib().bl_comm_unique_id(buf))
    return bytes(buf)


class Comm:
    """Rank `rank` of `world`; ``timeout_ms`` bounds every wait."""

    def __init__(self, uid: bytes, world: int, rank: int, timeout_ms: int = 60000):
        if len(uid) != N.COMM_ID_BYTES:
            raise ValueError("a unique id has %d bytes" % N.COMM_ID_BYTES)
        h = ctypes.c_void_p()
        buf = (ctypes.c_uint8 * len(uid)).from_buffer_copy(uid)
        N.check(N.lib().bl_comm_init(buf, world, rank, timeout_ms, ctypes.byref(h)))
        self._h, self.world, self.rank = h, world, rank

    def all_gather(self, send_ptr: int, recv_ptr: int, nbytes: int, stream=None):
        """recv[r * nbytes:(r + 1) * nbytes] = rank r's send, enqueued on
        `stream` (a raw cudaStream_t or None)."""
        N.check(N.lib().bl_comm_all_gather(self._h, send_ptr, recv_ptr, nbytes, stream))

    def args(self, send_ptr: int, recv_ptr: int, nbytes: int) -> "N.AllGatherArgs":
        """The all-gather as a kernel spec's arguments (runtime.Spec)."""
        return N.AllGatherArgs(comm=self._h, send=send_ptr, recv=recv_ptr, bytes=nbytes)

    def check(self):
        N.check(N.lib().bl_comm_check(self._h))

    @property
    def aborted(self) -> bool:
        return bool(N.lib().bl_comm_aborted(self._h))

    def abort(self):
        N.check(N.lib().bl_comm_abort(self._h))

    def close(self):
        if self._h:
            h, self._h = self._h, None
            N.check(N.lib().bl_comm_destroy(h))
