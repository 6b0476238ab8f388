"""NCCL communicator of the data-parallel step, over the library's C ABI (mfb_comm_*).

The reference's only collective is the psum of (loss, count, gradient tree)
over the 1-D ``"data"`` mesh (src/minifield_training/engine/step.py:36-78,
psum at :62). Here each process drives one GPU and one ``Communicator``:
rank 0 draws an NCCL unique id, the host hands it to the other ranks (a
file, a store, any side channel: ``unique_id_via_file`` is one), and every
rank builds the communicator with it. Collectives take device arrays and a
stream and are enqueued like kernels. Every call is bounded by the
communicator's timeout; an NCCL error or a missed deadline aborts the
communicator and raises ``CommError`` (the host learns of a failed peer
instead of waiting forever).
"""

import ctypes
import glob
import os
import sys
import time

from . import _lib
from .device import DeviceArray

P = ctypes.c_void_p

F32, F64, BF16, U8, I32 = range(5)
SUM, MAX, MIN = range(3)
_DTYPES = {"float32": F32, "bfloat16": BF16, "uint8": U8, "int32": I32}


class CommError(RuntimeError):
    """A collective failed or passed its deadline; the communicator is aborted."""


def _call(name, *args):
    status = getattr(_lib.lib(), name)(*args)
    if status == _lib.ERR_COMM:
        raise CommError(f"{name}: {_lib.last_error()}")
    _lib.check(status, name)


def nccl_library() -> str:
    """Path of the NCCL to load: MFB_NCCL_LIBRARY if set, else the NCCL wheel next to the interpreter's
    packages (the copy other CUDA frameworks in this environment load, so one process holds one NCCL),
    else the system's ``libnccl.so.2``."""
    env = os.environ.get("MFB_NCCL_LIBRARY")
    if env:
        return env
    for base in sys.path:
        hits = glob.glob(os.path.join(base, "nvidia", "nccl", "lib", "libnccl.so.2"))
        if hits:
            return hits[0]
    return "libnccl.so.2"


_VERSION = None


def load() -> int:
    """Load NCCL once; returns its version code (e.g. 22803 for 2.28.3)."""
    global _VERSION
    if _VERSION is None:
        v = ctypes.c_int()
        _call("mfb_comm_load", nccl_library().encode(), ctypes.byref(v))
        _VERSION = v.value
    return _VERSION


def unique_id() -> bytes:
    """A fresh NCCL unique id (drawn by rank 0 and handed to every rank)."""
    load()
    n = _lib.lib().mfb_comm_unique_id_bytes()
    buf = ctypes.create_string_buffer(n)
    _call("mfb_comm_unique_id", buf, n)
    return buf.raw


def unique_id_via_file(path: str, rank: int, timeout_s: float = 120.0) -> bytes:
    """Rank 0 draws the id and writes it to ``path`` (atomically); the other ranks wait for the file."""
    if rank == 0:
        uid = unique_id()
        tmp = f"{path}.{os.getpid()}.tmp"
        with open(tmp, "wb") as fh:
            fh.write(uid)
        os.replace(tmp, path)
        return uid
    load()
    n = _lib.lib().mfb_comm_unique_id_bytes()
    deadline = time.monotonic() + timeout_s
    while True:
        try:
            with open(path, "rb") as fh:
                data = fh.read()
            if len(data) == n:
                return data
        except FileNotFoundError:
            pass
        if time.monotonic() > deadline:
            raise CommError(f"no NCCL unique id at {path} after {timeout_s} s")
        time.sleep(0.01)


def _ptr_count(a, count=None):
    if isinstance(a, DeviceArray):
        return a.ptr, a.size if count is None else count, _DTYPES[a.dtype]
    raise TypeError("collectives take DeviceArray buffers")


class Communicator:
    """One rank of a NCCL communicator over ``world`` processes (one GPU each)."""

    def __init__(self, world: int, rank: int, uid: bytes, timeout_s: float = 300.0):
        load()
        self.world, self.rank, self.timeout_s = int(world), int(rank), float(timeout_s)
        h = P()
        _call("mfb_comm_init", uid, len(uid), self.world, self.rank, ctypes.c_double(self.timeout_s), ctypes.byref(h))
        self.handle = h

    def allreduce(self, buf: DeviceArray, op: int = SUM, stream=None, out: DeviceArray = None):
        """In place (or into ``out``) reduction of ``buf`` over the ranks."""
        ptr, n, dt = _ptr_count(buf)
        dst = out.ptr if out is not None else ptr
        _call("mfb_comm_allreduce", self.handle, P(ptr), P(dst), n, dt, op, stream)

    def allreduce_f64(self, ptr: int, count: int, op: int = SUM, stream=None):
        """In-place reduction of ``count`` doubles at device address ``ptr``."""
        _call("mfb_comm_allreduce", self.handle, P(ptr), P(ptr), count, F64, op, stream)

    def reduce_scatter(self, send: DeviceArray, recv: DeviceArray, op: int = SUM, stream=None):
        ptr, n, dt = _ptr_count(recv)
        if send.size != n * self.world or send.dtype != recv.dtype:
            raise ValueError("reduce_scatter: send must hold world x recv elements of recv's type")
        _call("mfb_comm_reduce_scatter", self.handle, P(send.ptr), P(ptr), n, dt, op, stream)

    def all_gather(self, send: DeviceArray, recv: DeviceArray, stream=None):
        ptr, n, dt = _ptr_count(send)
        if recv.size != n * self.world or send.dtype != recv.dtype:
            raise ValueError("all_gather: recv must hold world x send elements of send's type")
        _call("mfb_comm_allgather", self.handle, P(ptr), P(recv.ptr), n, dt, stream)

    def reduce(self, buf: DeviceArray, root: int, op: int = SUM, stream=None):
        """In-place reduction of ``buf`` over the ranks into rank ``root``'s copy (others unchanged)."""
        ptr, n, dt = _ptr_count(buf)
        _call("mfb_comm_reduce", self.handle, P(ptr), P(ptr), n, dt, op, int(root), stream)

    def broadcast(self, buf: DeviceArray, root: int, stream=None):
        """In-place broadcast of rank ``root``'s ``buf`` to every rank."""
        ptr, n, dt = _ptr_count(buf)
        _call("mfb_comm_broadcast", self.handle, P(ptr), P(ptr), n, dt, int(root), stream)

    def wait(self, stream=None, timeout_s: float = None):
        """Wait for ``stream`` while watching the communicator (raises CommError on failure or timeout)."""
        _call("mfb_comm_wait", self.handle, stream, ctypes.c_double(timeout_s or self.timeout_s))

    def abort(self):
        if self.handle is not None:
            _call("mfb_comm_abort", self.handle)

    def close(self):
        h, self.handle = self.handle, None
        if h is not None:
            _call("mfb_comm_destroy", h)

    def __del__(self):
        try:
            if getattr(self, "handle", None) is not None and _lib._lib is not None:
                _lib.lib().mfb_comm_destroy(self.handle)
                self.handle = None
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
