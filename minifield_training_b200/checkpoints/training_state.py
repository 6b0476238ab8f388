"""Atomic, hash-bound safetensors checkpoints of the full AdamW state.

The same on-disk contract as src/minifield_training/checkpoints/
training_state.py:23-260, so a native run can resume from a reference
checkpoint and the reference from a native one:

  <directory>/state.safetensors  tensors "params/<name>", "m/<name>",
                                 "v/<name>" (float32, the leaf's shape) and
                                 "step" (int32 scalar)
  <directory>/manifest.json      canonical JSON (sorted keys, no spaces) +
                                 newline: format "minifield.full-training-state/1",
                                 inventory_sha256, optimizer_id, cursor
                                 {run_id, data_sha256, source_id, next_batch},
                                 tensor_sha256 (SHA-256 of the tensor file)

A checkpoint is staged in a temporary sibling directory and published by one
rename. Loading checks the manifest's keys, format, inventory hash, optimizer
identity, cursor identity and the tensor file's SHA-256 before reading a
tensor, then the exact tensor set, dtypes and shapes, and finally that every
master and first moment is finite and every second moment finite and
non-negative (optimizers/adamw.py:232-260).

``save_arrays`` / ``load_arrays`` work on host NumPy arrays; ``save`` /
``load`` move an ``optimizers.adamw.State`` (device arenas) through them.
"""

import dataclasses
import hashlib
import json
import os
import tempfile
from pathlib import Path

import numpy as np

from ..optimizers import adamw

FORMAT = "minifield.full-training-state/1"
_GROUPS = ("params", "m", "v")
_INT32_MAX = 2**31 - 1


@dataclasses.dataclass(frozen=True)
class Cursor:
    """Identity and next unread batch of a deterministic input stream (training_state.py:26-44)."""

    run_id: str
    data_sha256: str
    source_id: str
    next_batch: int

    def __post_init__(self):
        if not self.run_id or not self.data_sha256 or not self.source_id or self.next_batch < 0:
            raise ValueError("Invalid checkpoint cursor")


def digest_file(path) -> str:
    """SHA-256 of a file, streamed (core/json_io.py:29-35)."""
    digest = hashlib.sha256()
    with open(path, "rb") as stream:
        for chunk in iter(lambda: stream.read(8 * 1024 * 1024), b""):
            digest.update(chunk)
    return digest.hexdigest()


def _check_state_values(groups, step, inventory):
    if step < 0 or step > _INT32_MAX:
        raise ValueError("Full-weight step is outside int32 range")
    for name in inventory.names:
        if not np.isfinite(groups["params"][name]).all():
            raise ValueError(f"Full-weight parameter is non-finite: {name}")
        if not np.isfinite(groups["m"][name]).all():
            raise ValueError(f"Full-weight first moment is non-finite: {name}")
        v = groups["v"][name]
        if not (np.isfinite(v) & (v >= 0)).all():
            raise ValueError(f"Full-weight second moment is invalid: {name}")


def _check_structure(groups, inventory):
    shapes = {sp.name: sp.shape for sp in inventory.specs}
    for g in _GROUPS:
        if set(groups[g]) != set(shapes):
            raise ValueError(f"Full-weight {g} tree mismatch")
        for name, value in groups[g].items():
            if value.dtype != np.float32 or tuple(value.shape) != shapes[name]:
                raise ValueError(f"Invalid checkpoint tensor: {g}/{name}")


def save_arrays(directory, groups, step, inventory, *, optimizer_id: str, cursor: Cursor) -> None:
    """Publish ``groups`` ({"params"|"m"|"v": {name: float32 array}}) and ``step``
    as a new checkpoint directory, atomically (training_state.py:58-95)."""
    from safetensors.numpy import save_file

    directory = Path(directory)
    if directory.exists():
        raise FileExistsError(directory)
    if not optimizer_id:
        raise ValueError("Optimizer identity is required")
    groups = {g: {n: np.asarray(v) for n, v in groups[g].items()} for g in _GROUPS}
    _check_structure(groups, inventory)
    _check_state_values(groups, int(step), inventory)
    arrays = {f"{g}/{n}": np.ascontiguousarray(v, dtype=np.float32) for g in _GROUPS for n, v in groups[g].items()}
    arrays["step"] = np.asarray(int(step), dtype=np.int32)
    directory.parent.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory(prefix=f".{directory.name}-", dir=directory.parent) as temporary:
        staging = Path(temporary)
        tensor_path = staging / "state.safetensors"
        save_file(arrays, str(tensor_path))
        manifest = {"format": FORMAT, "inventory_sha256": inventory.sha256, "optimizer_id": optimizer_id,
                    "cursor": dataclasses.asdict(cursor), "tensor_sha256": digest_file(tensor_path)}
        (staging / "manifest.json").write_text(adamw.canonical_json(manifest) + "\n", encoding="utf-8")
        if directory.exists():
            raise FileExistsError(directory)
        os.rename(staging, directory)


def load_arrays(directory, inventory, *, optimizer_id: str, run_id: str, data_sha256: str, source_id: str,
                tensor_filename: str = "state.safetensors"):
    """Verified host state of a checkpoint: ``(groups, step, cursor)`` (training_state.py:98-203)."""
    from safetensors.numpy import load_file

    directory = Path(directory)
    raw = json.loads((directory / "manifest.json").read_text(encoding="utf-8"))
    if not isinstance(raw, dict) or set(raw) != {"format", "inventory_sha256", "optimizer_id", "cursor",
                                                 "tensor_sha256"}:
        raise ValueError("Invalid checkpoint manifest")
    if (raw["format"] != FORMAT or raw["inventory_sha256"] != inventory.sha256
            or raw["optimizer_id"] != optimizer_id):
        raise ValueError("Incompatible checkpoint state identity")
    c = raw["cursor"]
    if not isinstance(c, dict) or set(c) != {"run_id", "data_sha256", "source_id", "next_batch"}:
        raise ValueError("Invalid checkpoint cursor")
    if (not isinstance(c["run_id"], str) or not isinstance(c["data_sha256"], str)
            or not isinstance(c["source_id"], str) or not isinstance(c["next_batch"], int)
            or isinstance(c["next_batch"], bool)):
        raise ValueError("Invalid checkpoint cursor types")
    cursor = Cursor(c["run_id"], c["data_sha256"], c["source_id"], c["next_batch"])
    if (cursor.run_id, cursor.data_sha256, cursor.source_id) != (run_id, data_sha256, source_id):
        raise ValueError("Checkpoint run/data/source identity mismatch")
    tensor_path = directory / tensor_filename
    if digest_file(tensor_path) != raw["tensor_sha256"]:
        raise ValueError("Checkpoint tensor SHA-256 mismatch")
    arrays = load_file(str(tensor_path))
    expected = {f"{g}/{n}" for g in _GROUPS for n in inventory.names} | {"step"}
    if set(arrays) != expected:
        raise ValueError("Checkpoint tensor inventory mismatch")
    groups = {g: {n: arrays[f"{g}/{n}"] for n in inventory.names} for g in _GROUPS}
    _check_structure(groups, inventory)
    step = arrays["step"]
    if step.dtype != np.int32 or step.shape:
        raise ValueError("Invalid checkpoint step")
    _check_state_values(groups, int(step), inventory)
    return groups, int(step), cursor


def host_state(state):
    """Host copies of a device State: ``(groups, step)``."""
    groups = {g: {n: state[g][n].numpy() for n in state.layout.specs} for g in _GROUPS}
    return groups, int(state["step"].numpy()[0])


def save(directory, state, inventory, *, optimizer_id: str, cursor: Cursor) -> None:
    """Checkpoint a device ``optimizers.adamw.State`` (call after a committed update)."""
    groups, step = host_state(state)
    save_arrays(directory, groups, step, inventory, optimizer_id=optimizer_id, cursor=cursor)


def load(directory, inventory, *, optimizer_id: str, run_id: str, data_sha256: str, source_id: str, order=None,
         grads=None, params=None):
    """Restore a device State from a checkpoint: ``(state, cursor)``.

    ``order``, ``grads`` and ``params`` are passed to
    ``optimizers.adamw.initialize_state`` (arena order and caller-owned arenas).
    """
    import ctypes

    from .. import _lib

    groups, step, cursor = load_arrays(directory, inventory, optimizer_id=optimizer_id, run_id=run_id,
                                       data_sha256=data_sha256, source_id=source_id)
    state = adamw.initialize_state(groups["params"], inventory, order=order, grads=grads, params=params)
    for g in ("m", "v"):
        for name, host in groups[g].items():
            host = np.ascontiguousarray(host, np.float32)
            _lib.call("mfb_memcpy_h2d", ctypes.c_void_p(state[g][name].ptr), host.ctypes.data_as(ctypes.c_void_p),
                      host.nbytes, None)
    s = np.array([step], np.int32)
    _lib.call("mfb_memcpy_h2d", ctypes.c_void_p(state["step"].ptr), s.ctypes.data_as(ctypes.c_void_p), 4, None)
    _lib.call("mfb_device_sync")
    return state, cursor


def load_warm_start_masters(directory, inventory, *, run_id: str, data_sha256: str, source_id: str,
                            tensor_filename: str = "state.safetensors"):
    """Verified FP32 masters of a prior checkpoint, for a new optimizer (training_state.py:206-238)."""
    raw = json.loads((Path(directory) / "manifest.json").read_text(encoding="utf-8"))
    if not isinstance(raw, dict) or not isinstance(raw.get("optimizer_id"), str):
        raise ValueError("Invalid warm-start checkpoint manifest")
    if tensor_filename not in {"state.safetensors", "model.safetensors"}:
        raise ValueError("Unsupported warm-start tensor filename")
    groups, _, _ = load_arrays(directory, inventory, optimizer_id=raw["optimizer_id"], run_id=run_id,
                               data_sha256=data_sha256, source_id=source_id, tensor_filename=tensor_filename)
    return groups["params"]


def verify_roundtrip(directory, state, cursor: Cursor, inventory, optimizer_id: str) -> None:
    """Check every saved master, moment and the step against the live device state."""
    groups, step, restored = load_arrays(directory, inventory, optimizer_id=optimizer_id, run_id=cursor.run_id,
                                         data_sha256=cursor.data_sha256, source_id=cursor.source_id)
    live, live_step = host_state(state)
    if restored != cursor or step != live_step:
        raise ValueError("Checkpoint round-trip mismatch")
    for g in _GROUPS:
        for name in inventory.names:
            if not np.array_equal(groups[g][name], live[g][name]):
                raise ValueError(f"Checkpoint round-trip mismatch: {g}/{name}")
