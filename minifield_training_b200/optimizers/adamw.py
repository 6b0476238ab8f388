"""Transactional full-weight AdamW over device arenas.

Mirrors src/minifield_training/optimizers/adamw.py: ``CommitCode`` (:30-39),
``AdamWConfig`` and its validation (:42-110), ``CommitResult`` (:113-122),
``initialize_state`` (:300-322) and ``make_transaction(inventory, config)`` ->
``transition(state, gradients, active_loss, accumulation_valid)`` (:384-571).
The inventory mirrors ``core/parameters.py:12-57`` (name, shape, trainable,
decayed). The update itself is ``mfb_adamw_commit`` in libmfb200.so.

Layout: a ``State`` keeps params, m and v in three FP32 device arenas ordered
[decayed trainable | undecayed trainable | frozen] (names sorted inside each
group), plus a grads arena over the trainable prefix and an int32 device step.
``state["params"][name]`` etc. are views into the arenas. The transaction
updates the arenas in place only when it commits (the reference's donated
transaction, adamw.py:574-591); a rejected update leaves them untouched, so
``result.state`` is the same object either way.
"""

import ctypes
import dataclasses
import enum
import hashlib
import json
import math

import numpy as np

from .. import _lib
from ..device import DeviceArray

_INT32_MAX = np.iinfo(np.int32).max


class CommitCode(enum.IntEnum):
    """Result codes, as adamw.py:30-39."""

    COMMITTED = 0
    ACCUMULATION_INVALID = 1
    NONFINITE_LOSS = 2
    INVALID_STATE = 3
    NONFINITE_GRADIENT = 4
    STEP_OVERFLOW = 5
    CANDIDATE_INVALID = 6


_F32_MAX = float(np.finfo(np.float32).max)
_F32_TINY = float(np.finfo(np.float32).tiny)

# Admission of one setting as a float32 scalar: (test on the Python value,
# what the value must be). The first failing test names the error, so the
# order is the precedence of the messages (adamw.py:53-93 of the reference).
_SCALAR_RULES = (
    (lambda x: not isinstance(x, bool) and isinstance(x, (int, float)), "a non-boolean finite number"),
    (lambda x: math.isfinite(float(x)) and abs(float(x)) <= _F32_MAX, "a finite float32 scalar"),
    (lambda x: not float(x) or float(np.float32(x)) != 0, "representable in float32"),
    (lambda x: not float(np.float32(x)) or abs(float(np.float32(x))) >= _F32_TINY,
     "zero or a normal float32 scalar"),
)

# Range of each setting once rounded to float32, checked only after every
# setting passed the scalar rules; fields in declaration order.
_RANGE_RULES = {
    "learning_rate": (lambda x: x > 0, "positive"),
    "beta1": (lambda x: 0 <= x < 1, "in [0, 1)"),
    "beta2": (lambda x: 0 <= x < 1, "in [0, 1)"),
    "epsilon": (lambda x: x > 0, "positive"),
    "weight_decay": (lambda x: x >= 0, "nonnegative"),
    "clip_norm": (lambda x: x > 0, "positive"),
}


def _first_broken(rules, value):
    """The requirement text of the first rule ``value`` fails, or None."""
    return next((what for test, what in rules if not test(value)), None)


@dataclasses.dataclass(frozen=True)
class AdamWConfig:
    """Validated float32 settings (adamw.py:42-92).

    Every setting is stored as the float32 value the update uses. A bad
    setting raises the reference's ``ValueError`` text ("<name> must be ...");
    scalar problems of any field are reported before range problems.
    """

    learning_rate: float
    beta1: float = 0.9
    beta2: float = 0.95
    epsilon: float = 1e-8
    weight_decay: float = 0.01
    clip_norm: float = 1.0

    def __post_init__(self):
        raw = {name: getattr(self, name) for name in _RANGE_RULES}
        problems = ((name, _first_broken(_SCALAR_RULES, value)) for name, value in raw.items())
        problems = [(name, what) for name, what in problems if what is not None]
        if problems:
            name, what = problems[0]
            raise ValueError(f"{name} must be {what}")
        rounded = {name: float(np.float32(value)) for name, value in raw.items()}
        for name, (test, what) in _RANGE_RULES.items():
            if not test(rounded[name]):
                raise ValueError(f"{name} must be {what}")
        for name, value in rounded.items():
            object.__setattr__(self, name, value)


@dataclasses.dataclass(frozen=True)
class ParameterSpec:
    """One stored leaf (core/parameters.py:11-21)."""

    name: str
    shape: tuple
    trainable: bool
    decayed: bool
    source_dtype: str = "bfloat16"
    master_dtype: str = "float32"
    quantized: bool = False


@dataclasses.dataclass(frozen=True)
class Inventory:
    """Leaf metadata with the derived membership views (core/parameters.py:24-55).

    ``sha256`` identifies the inventory the way the reference does: SHA-256 of
    the canonical JSON of (format, dtypes, quantization profile, specs), so a
    checkpoint manifest written here names the same inventory hash as one
    written by the reference for the same build_inventory arguments.
    """

    specs: tuple
    parameter_count: int = 0
    source_dtype: str = "bfloat16"
    master_dtype: str = "float32"
    quantization_profile: object = None
    sha256: str = ""

    @property
    def names(self):
        return tuple(s.name for s in self.specs)

    @property
    def trainable_names(self):
        return tuple(s.name for s in self.specs if s.trainable)

    @property
    def frozen_names(self):
        return tuple(s.name for s in self.specs if not s.trainable)


def canonical_json(value) -> str:
    """Deterministic JSON text, non-finite numbers rejected (core/json_io.py:18-26)."""
    return json.dumps(value, ensure_ascii=False, sort_keys=True, separators=(",", ":"), allow_nan=False)


def build_inventory(shapes, *, decayed_names=frozenset(), frozen_names=frozenset(),
                    format_id="minifield_training_b200/1", source_dtype="bfloat16", master_dtype="float32",
                    quantization_profile=None, quantized_names=frozenset()) -> Inventory:
    """Inventory over ``shapes`` (name -> shape) (core/parameters.py:58-152).

    Frozen leaves cannot decay; a quantized leaf needs a named quantization
    profile. Leaves are ordered by name.
    """
    if source_dtype not in {"bfloat16", "float16", "float32"}:
        raise ValueError("Unsupported checkpoint source dtype")
    if master_dtype != "float32":
        raise ValueError("Full-weight masters must be float32")
    if quantization_profile is None and quantized_names:
        raise ValueError("Quantized leaves require a declared QAT profile")
    if quantization_profile is not None and not quantization_profile:
        raise ValueError("Quantization profile cannot be empty")
    unknown = (set(decayed_names) | set(frozen_names) | set(quantized_names)) - set(shapes)
    if unknown:
        raise ValueError(f"Inventory names are not parameters: {sorted(unknown)}")
    if set(decayed_names) & set(frozen_names):
        raise ValueError("Frozen parameters cannot be decayed")
    specs = tuple(
        ParameterSpec(name, tuple(int(x) for x in shapes[name]), name not in frozen_names, name in decayed_names,
                      source_dtype, master_dtype, name in quantized_names)
        for name in sorted(shapes))
    if not specs:
        raise ValueError("Full-weight inventory must not be empty")
    payload = {
        "format": format_id,
        "source_dtype": source_dtype,
        "master_dtype": master_dtype,
        "quantization_profile": quantization_profile,
        "specs": [{"name": sp.name, "shape": list(sp.shape), "source_dtype": sp.source_dtype,
                   "master_dtype": sp.master_dtype, "trainable": sp.trainable, "decayed": sp.decayed,
                   "quantized": sp.quantized} for sp in specs],
    }
    return Inventory(specs, parameter_count=sum(int(np.prod(sp.shape)) for sp in specs), source_dtype=source_dtype,
                     master_dtype=master_dtype, quantization_profile=quantization_profile,
                     sha256=hashlib.sha256(canonical_json(payload).encode("utf-8")).hexdigest())


class Layout:
    """Arena offsets: [decayed trainable | undecayed trainable | frozen].

    Inside each group leaves follow ``order`` (names, default sorted), so a
    caller can make leaves that one kernel writes together adjacent.
    """

    def __init__(self, inventory: Inventory, order=None):
        rank = {n: i for i, n in enumerate(order if order is not None else sorted(inventory.names))}
        if set(rank) != set(inventory.names):
            raise ValueError("arena order must list every inventory name once")
        specs = sorted(inventory.specs, key=lambda s: rank[s.name])
        groups = ([s for s in specs if s.trainable and s.decayed],
                  [s for s in specs if s.trainable and not s.decayed],
                  [s for s in specs if not s.trainable])
        self.specs = {s.name: s for s in inventory.specs}
        self.offsets = {}
        off = 0
        sizes = []
        for group in groups:
            for s in group:
                # 4-element (16-byte) alignment for every leaf keeps vector access aligned.
                self.offsets[s.name] = off
                off += _round4(int(np.prod(s.shape, dtype=np.int64)))
            sizes.append(off)
        self.n_decayed, self.n_train, self.n_total = sizes
        self.trainable = tuple(s.name for s in groups[0] + groups[1])

    def size(self, name):
        return int(np.prod(self.specs[name].shape, dtype=np.int64))

    def views(self, arena: DeviceArray, names):
        return {n: arena.view(self.offsets[n], self.specs[n].shape) for n in names}


def _round4(n):
    return (n + 3) // 4 * 4


class State(dict):
    """``{"params", "m", "v", "step"}`` (optimizers/state.py:11-17) backed by arenas."""

    def __init__(self, layout: Layout, arenas):
        self.layout = layout
        self.arenas = arenas  # params, m, v, grads, step
        names = list(layout.specs)
        super().__init__(params=layout.views(arenas["params"], names), m=layout.views(arenas["m"], names),
                         v=layout.views(arenas["v"], names), step=arenas["step"])

    def gradient_tree(self):
        """Views of the grads arena for the trainable leaves (the transition's input layout)."""
        return self.layout.views(self.arenas["grads"], self.layout.trainable)


def initialize_state(parameters, inventory: Inventory, *, order=None, grads=None, params=None) -> State:
    """Zero-moment FP32 state (adamw.py:300-322); rejects non-finite masters.

    ``order`` sets the arena order (see Layout); ``grads`` / ``params``
    optionally supply the gradient arena (FP32, at least n_train elements) and
    the master arena (FP32, zeroed, at least n_total elements), both 16-byte
    aligned, e.g. buffers that a collective library also addresses.
    """
    layout = Layout(inventory, order)
    if set(parameters) != set(layout.specs):
        raise ValueError("Full-weight parameter tree mismatch")
    arenas = {k: DeviceArray.zeros((max(layout.n_total, 4),), "float32") for k in ("m", "v")}
    if params is not None:
        if params.dtype != "float32" or params.size < layout.n_total or params.ptr % 16:
            raise ValueError("master arena must be 16-byte aligned float32 with n_total elements")
        arenas["params"] = params
    else:
        arenas["params"] = DeviceArray.zeros((max(layout.n_total, 4),), "float32")
    if grads is not None:
        if grads.dtype != "float32" or grads.size < layout.n_train or grads.ptr % 16:
            raise ValueError("gradient arena must be 16-byte aligned float32 with n_train elements")
        arenas["grads"] = grads
    else:
        arenas["grads"] = DeviceArray.zeros((max(layout.n_train, 4),), "float32")
    arenas["step"] = DeviceArray.zeros((1,), "int32")
    for name, value in parameters.items():
        host = np.asarray(value, np.float32)
        if host.shape != layout.specs[name].shape:
            raise ValueError(f"Full-weight parameter shape mismatch: {name}")
        if not np.isfinite(host).all():
            raise ValueError(f"Full-weight parameter is non-finite: {name}")
        dst = arenas["params"].view(layout.offsets[name], host.shape)
        _lib.call("mfb_memcpy_h2d", ctypes.c_void_p(dst.ptr), host.ctypes.data_as(ctypes.c_void_p), host.nbytes, None)
    return State(layout, arenas)


class _ResultStruct(ctypes.Structure):
    _fields_ = [("code", ctypes.c_int32), ("committed", ctypes.c_int32), ("loss", ctypes.c_float),
                ("gradient_norm", ctypes.c_float), ("clipped_gradient_norm", ctypes.c_float),
                ("update_norm", ctypes.c_float)]


class CommitResult:
    """State and diagnostics of one transaction (adamw.py:113-122); fields read on first access."""

    def __init__(self, state, device_result: DeviceArray, stream):
        self.state = state
        self._dev = device_result
        self._stream = stream
        self._host = None

    def _fetch(self):
        if self._host is None:
            r = _ResultStruct()
            _lib.call("mfb_memcpy_d2h", ctypes.c_void_p(ctypes.addressof(r)), ctypes.c_void_p(self._dev.ptr),
                      ctypes.sizeof(r), self._stream)
            _lib.call("mfb_stream_sync", self._stream)
            self._host = r
        return self._host

    committed = property(lambda self: bool(self._fetch().committed))
    code = property(lambda self: CommitCode(self._fetch().code))
    loss = property(lambda self: float(self._fetch().loss))
    gradient_norm = property(lambda self: float(self._fetch().gradient_norm))
    clipped_gradient_norm = property(lambda self: float(self._fetch().clipped_gradient_norm))
    update_norm = property(lambda self: float(self._fetch().update_norm))


def _device_scalar(value, dtype, cache, key):
    if isinstance(value, DeviceArray):
        return value
    arr = cache.get(key)
    if arr is None:
        arr = cache[key] = DeviceArray((1,), dtype)
    host = np.asarray([value], dtype=np.float32 if dtype == "float32" else np.uint8)
    _lib.call("mfb_memcpy_h2d", ctypes.c_void_p(arr.ptr), host.ctypes.data_as(ctypes.c_void_p), host.nbytes, None)
    return arr


def make_transaction(inventory: Inventory, config: AdamWConfig):
    """Build the commit (adamw.py:384-415): ``transition(state, gradients, active_loss, accumulation_valid, *, divisor=None, stream=None)``.

    ``gradients`` is ``state.gradient_tree()`` (already in the arena) or any
    name -> array mapping over exactly the trainable leaves, which is copied
    into the arena first. ``active_loss`` / ``accumulation_valid`` are Python
    scalars or device scalars; ``divisor`` (device float32) optionally divides
    the gradients first (the logical step's normalization).
    """
    workspace = DeviceArray((_lib.lib().mfb_adamw_workspace_size(),), "uint8")
    result_dev = DeviceArray((6,), "int32")
    scalars = {}

    names = set(inventory.names)

    def transition(state: State, gradients, active_loss, accumulation_valid, *, divisor=None, stream=None):
        if not isinstance(state, State) or set(state.layout.specs) != names:
            raise ValueError("Full-weight state does not match the inventory")
        layout = state.layout
        if set(gradients) != set(layout.trainable):
            missing = sorted(set(layout.trainable) - set(gradients))
            extra = sorted(set(gradients) - set(layout.trainable))
            raise ValueError(f"Full-weight gradient tree mismatch; missing={missing}, extra={extra}")
        grads = state.arenas["grads"]
        for name, g in gradients.items():
            dst = grads.view(layout.offsets[name], layout.specs[name].shape)
            if isinstance(g, DeviceArray):
                if g.ptr != dst.ptr:
                    if g.dtype != "float32" or g.shape != dst.shape:
                        raise ValueError(f"Full-weight gradient must be float32 of shape {dst.shape}: {name}")
                    dst.copy_(g, stream)
            else:
                host = np.asarray(g)
                if host.shape != dst.shape or host.dtype != np.float32:
                    raise ValueError(f"Full-weight gradient must be float32 of shape {dst.shape}: {name}")
                host = np.ascontiguousarray(host)
                _lib.call("mfb_memcpy_h2d", ctypes.c_void_p(dst.ptr), host.ctypes.data_as(ctypes.c_void_p),
                          host.nbytes, stream)
        loss = _device_scalar(active_loss, "float32", scalars, "loss")
        valid = _device_scalar(bool(accumulation_valid) if not isinstance(accumulation_valid, DeviceArray)
                               else accumulation_valid, "uint8", scalars, "valid")
        P = ctypes.c_void_p
        a = state.arenas
        _lib.call("mfb_adamw_commit", P(a["params"].ptr), P(a["m"].ptr), P(a["v"].ptr), P(grads.ptr), layout.n_train,
                  layout.n_decayed, layout.n_total, P(a["step"].ptr), P(loss.ptr), P(valid.ptr),
                  P(divisor.ptr) if divisor is not None else None, config.learning_rate, config.beta1, config.beta2,
                  config.epsilon, config.weight_decay, config.clip_norm, P(result_dev.ptr), P(workspace.ptr),
                  workspace.nbytes, stream)
        return CommitResult(state, result_dev, stream)

    return transition


# Passes of mfb_adamw_shard_pass (include/mfb200.h).
_CHECK, _CHECK_FINALIZE, _CANDIDATE, _CANDIDATE_FINALIZE, _COMMIT = range(5)


def shard_slices(n: int, world: int, rank: int):
    """(lo, hi, per) of ``rank``'s slice of [0, n): ``world`` slices of ``per``
    elements (a multiple of 4, per * world >= n), the last ones clipped at n."""
    per = -(-n // (4 * world)) * 4
    lo = min(rank * per, n)
    return lo, min(lo + per, n), per


def sharded_master_elements(layout, world: int) -> int:
    """Master arena size for a sharded transaction: the all-gather covers
    ``world`` equal trainable slices, which may run past n_total."""
    return max(layout.n_total, shard_slices(layout.n_train, world, 0)[2] * world, 4)


def make_sharded_transaction(inventory: Inventory, config: AdamWConfig, comm, slices=None):
    """The transaction of ``make_transaction`` with the elementwise passes split
    across the data-parallel ranks of ``comm`` (a comm.Communicator):
    ``transition(state, active_loss, accumulation_valid, *, divisor=None,
    stream=None)`` on the reduced gradients already in ``state.arenas["grads"]``.

    Each rank checks its slice of the state, runs the candidate and the commit
    on its slice of the trainable masters and moments, and the ranks
    all-gather the masters; the global decisions (gradient norm and flags,
    update norm and candidate flags) are SUM-allreduces of three doubles, so
    every rank reaches the same code. The moments outside a rank's slice are
    never read or written on that rank. ``state.arenas["params"]`` must hold
    ``sharded_master_elements`` floats (the all-gather writes every rank's
    whole slice).

    ``slices`` = (check_lo, check_hi, lo, hi) replaces the equal slices with
    the caller's partition (check ranges tiling [0, n_total), update ranges
    tiling [0, n_train) across the ranks, starts multiples of 4) and leaves
    the masters un-gathered: the caller brings every rank's updated range to
    the others (a data-parallel step overlaps that with its next forward).
    """
    world, rank = comm.world, comm.rank
    workspace = DeviceArray((_lib.lib().mfb_adamw_workspace_size(),), "uint8")
    result_dev = DeviceArray((6,), "int32")
    red = DeviceArray((3 * 8,), "uint8")  # three float64 partials, reduced across the ranks
    scalars = {}
    names = set(inventory.names)

    def transition(state: State, active_loss, accumulation_valid, *, divisor=None, stream=None):
        if not isinstance(state, State) or set(state.layout.specs) != names:
            raise ValueError("Full-weight state does not match the inventory")
        layout, a = state.layout, state.arenas
        if slices is None and a["params"].size < sharded_master_elements(layout, world):
            raise ValueError("sharded AdamW needs a master arena of sharded_master_elements floats")
        loss = _device_scalar(active_loss, "float32", scalars, "loss")
        valid = _device_scalar(bool(accumulation_valid) if not isinstance(accumulation_valid, DeviceArray)
                               else accumulation_valid, "uint8", scalars, "valid")
        P = ctypes.c_void_p
        if slices is None:
            c_lo, c_hi, _ = shard_slices(layout.n_total, world, rank)
            t_lo, t_hi, per = shard_slices(layout.n_train, world, rank)
        else:
            c_lo, c_hi, t_lo, t_hi = slices

        def run(pass_id, lo, hi):
            _lib.call("mfb_adamw_shard_pass", pass_id, P(a["params"].ptr), P(a["m"].ptr), P(a["v"].ptr),
                      P(a["grads"].ptr), lo, hi, layout.n_train, layout.n_decayed, layout.n_total,
                      P(a["step"].ptr), P(loss.ptr), P(valid.ptr), P(divisor.ptr) if divisor is not None else None,
                      config.learning_rate, config.beta1, config.beta2, config.epsilon, config.weight_decay,
                      config.clip_norm, P(red.ptr), P(result_dev.ptr), P(workspace.ptr), workspace.nbytes,
                      stream)

        # Every collective is enqueued on ``stream``, ordered between the passes.
        run(_CHECK, c_lo, c_hi)
        comm.allreduce_f64(red.ptr, 3, stream=stream)
        run(_CHECK_FINALIZE, 0, 0)
        run(_CANDIDATE, t_lo, t_hi)
        comm.allreduce_f64(red.ptr, 2, stream=stream)
        run(_CANDIDATE_FINALIZE, 0, 0)
        run(_COMMIT, t_lo, t_hi)
        if slices is None:
            masters = a["params"]
            comm.all_gather(masters.view(rank * per, (per,)), masters.view(0, (per * world,)), stream=stream)
        return CommitResult(state, result_dev, stream)

    return transition
