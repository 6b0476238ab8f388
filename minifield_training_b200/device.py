"""Device arrays, streams and workspaces over the library's runtime helpers.

``DeviceArray`` is the array type of this package's functional API: a typed
device buffer (pointer, shape, dtype) that plays the role a ``jax.Array``
plays in the reference. Host NumPy arrays passed to the API are uploaded
(cast to the kernel dtype) on the way in; results stay on the device until
``.numpy()`` is called.
"""

import ctypes

import ml_dtypes
import numpy as np

from . import _lib

DTYPES = {
    "bfloat16": np.dtype(ml_dtypes.bfloat16),
    "float32": np.dtype(np.float32),
    "int32": np.dtype(np.int32),
    "int8": np.dtype(np.int8),
    "uint8": np.dtype(np.uint8),
}


def _canon(dtype) -> str:
    if isinstance(dtype, str) and dtype in DTYPES:
        return dtype
    d = np.dtype(dtype)
    for name, nd in DTYPES.items():
        if nd == d:
            return name
    if d == np.bool_:
        return "int32"
    raise TypeError(f"unsupported dtype {dtype}")


class DeviceArray:
    """A contiguous device buffer with a shape and a dtype."""

    __slots__ = ("ptr", "shape", "dtype", "_owner", "_base", "__weakref__")

    def __init__(self, shape, dtype, ptr=None, owner=True):
        self.shape = tuple(int(s) for s in shape)
        self.dtype = _canon(dtype)
        self._owner = owner and ptr is None
        self._base = None
        if ptr is None:
            p = ctypes.c_void_p()
            _lib.call("mfb_malloc", ctypes.byref(p), max(self.nbytes, 1))
            ptr = p.value
        self.ptr = ptr

    @property
    def size(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64))

    @property
    def itemsize(self) -> int:
        return DTYPES[self.dtype].itemsize

    @property
    def nbytes(self) -> int:
        return self.size * self.itemsize

    @property
    def ndim(self) -> int:
        return len(self.shape)

    def __repr__(self):
        return f"DeviceArray(shape={self.shape}, dtype={self.dtype})"

    def __del__(self):
        if getattr(self, "_owner", False) and self.ptr and _lib._lib is not None:
            try:
                _lib.lib().mfb_free(ctypes.c_void_p(self.ptr))
            except Exception:
                pass
            self.ptr = None

    @classmethod
    def empty(cls, shape, dtype):
        return cls(shape, dtype)

    @classmethod
    def zeros(cls, shape, dtype, stream=None):
        a = cls(shape, dtype)
        _lib.call("mfb_memset", ctypes.c_void_p(a.ptr), 0, a.nbytes, stream)
        return a

    @classmethod
    def from_numpy(cls, host, dtype=None, stream=None):
        host = np.asarray(host)
        name = _canon(dtype if dtype is not None else host.dtype)
        data = np.ascontiguousarray(host.astype(DTYPES[name], copy=False))
        a = cls(host.shape, name)
        _lib.call("mfb_memcpy_h2d", ctypes.c_void_p(a.ptr), data.ctypes.data_as(ctypes.c_void_p), a.nbytes, stream)
        if stream is not None:
            sync(stream)
        return a

    def numpy(self, stream=None) -> np.ndarray:
        out = np.empty(self.shape, DTYPES[self.dtype])
        _lib.call("mfb_memcpy_d2h", out.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(self.ptr), self.nbytes, stream)
        sync(stream)
        return out

    def float32(self) -> np.ndarray:
        return self.numpy().astype(np.float32)

    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        shape = list(shape)
        if -1 in shape:
            known = int(np.prod([s for s in shape if s != -1]))
            shape[shape.index(-1)] = self.size // known
        if int(np.prod(shape)) != self.size:
            raise ValueError(f"cannot reshape {self.shape} to {tuple(shape)}")
        view = DeviceArray(shape, self.dtype, ptr=self.ptr, owner=False)
        view._base = self  # a view keeps its owner alive
        return view

    def view(self, offset: int, shape, dtype=None):
        """A view of ``shape`` starting ``offset`` elements (of this dtype) in."""
        dtype = _canon(dtype or self.dtype)
        shape = tuple(int(x) for x in ((shape,) if np.isscalar(shape) else shape))
        nbytes = int(np.prod(shape, dtype=np.int64)) * DTYPES[dtype].itemsize
        start = int(offset) * self.itemsize
        if offset < 0 or start + nbytes > self.nbytes:
            raise ValueError(f"view [{start}, {start + nbytes}) bytes outside a {self.nbytes}-byte array")
        v = DeviceArray(shape, dtype, ptr=self.ptr + start, owner=False)
        v._base = self
        return v

    def copy_(self, other: "DeviceArray", stream=None):
        if other.nbytes != self.nbytes:
            raise ValueError("size mismatch")
        _lib.call("mfb_memcpy_d2d", ctypes.c_void_p(self.ptr), ctypes.c_void_p(other.ptr), self.nbytes, stream)
        return self


def as_device(x, dtype, stream=None) -> DeviceArray:
    """Return ``x`` as a DeviceArray of ``dtype`` (uploading host arrays)."""
    if isinstance(x, DeviceArray):
        if x.dtype != _canon(dtype):
            raise TypeError(f"expected {dtype} device array, got {x.dtype}")
        return x
    return DeviceArray.from_numpy(np.asarray(x), dtype, stream)


def sync(stream=None):
    if stream is None:
        _lib.call("mfb_device_sync")
    else:
        _lib.call("mfb_stream_sync", stream)


def set_device(index: int):
    _lib.call("mfb_set_device", int(index))


def device_count() -> int:
    n = ctypes.c_int()
    _lib.call("mfb_device_count", ctypes.byref(n))
    return n.value


def sm_version(index: int = 0):
    a, b = ctypes.c_int(), ctypes.c_int()
    _lib.call("mfb_device_sm_version", int(index), ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


def require_b200(index: int = 0):
    """Raise unless device ``index`` is an sm_100 (B200-class) GPU."""
    major, minor = sm_version(index)
    if (major, minor) != (10, 0):
        raise RuntimeError(f"the b200 backend needs an sm_100 device, found sm_{major}{minor}")


class Workspace:
    """Grow-only scratch buffer handed to kernels that take a workspace."""

    def __init__(self):
        self.buf = None

    def get(self, nbytes: int) -> DeviceArray:
        if self.buf is None or self.buf.nbytes < nbytes:
            self.buf = DeviceArray((max(int(nbytes), 256),), "uint8")
        return self.buf


_WORKSPACES = {}


def workspace(tag: str, nbytes: int) -> DeviceArray:
    ws = _WORKSPACES.setdefault(tag, Workspace())
    return ws.get(nbytes)


class Event:
    def __init__(self):
        p = ctypes.c_void_p()
        _lib.call("mfb_event_create", ctypes.byref(p))
        self.ptr = p

    def record(self, stream=None):
        _lib.call("mfb_event_record", self.ptr, stream)

    def wait_on(self, stream):
        """Make later work on ``stream`` wait for this event's most recent record."""
        _lib.call("mfb_stream_wait_event", stream, self.ptr)

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float()
        _lib.call("mfb_event_elapsed_ms", self.ptr, end.ptr, ctypes.byref(ms))
        return ms.value

    def __del__(self):
        try:
            _lib.lib().mfb_event_destroy(self.ptr)
        except Exception:
            pass


class HostBuffer:
    """Pinned host memory viewed as a NumPy array (for end-to-end timing)."""

    def __init__(self, shape, dtype):
        self.dtype = np.dtype(dtype)
        self.shape = tuple(shape)
        nbytes = int(np.prod(self.shape)) * self.dtype.itemsize
        p = ctypes.c_void_p()
        _lib.call("mfb_host_alloc", ctypes.byref(p), max(nbytes, 1))
        self.ptr = p
        buf = (ctypes.c_uint8 * max(nbytes, 1)).from_address(p.value)
        self.array = np.frombuffer(buf, dtype=self.dtype, count=int(np.prod(self.shape))).reshape(self.shape)

    def __del__(self):
        try:
            _lib.lib().mfb_host_free(self.ptr)
        except Exception:
            pass


def h2d(dst: DeviceArray, src_ptr, nbytes: int, stream=None):
    _lib.call("mfb_memcpy_h2d", ctypes.c_void_p(dst.ptr), src_ptr, nbytes, stream)


def d2h(dst_ptr, src: DeviceArray, nbytes: int, stream=None):
    _lib.call("mfb_memcpy_d2h", dst_ptr, ctypes.c_void_p(src.ptr), nbytes, stream)
