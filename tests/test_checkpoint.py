"""Checkpoint state I/O in the reference's format, on host arrays (CPU).

Mirrors tests/checkpoints/test_training_state.py of the reference (complete
round trip with the cursor, identity and SHA-256 tamper rejection, strided
host views), plus the inventory hash pinned against values the reference's own
build_inventory produced (tests/golden/checkpoint_inventory.json, written by
tests/golden/make_checkpoint_golden.py).
"""

import json
import os

import numpy as np
import pytest

from minifield_training_b200.checkpoints import training_state as ts
from minifield_training_b200.optimizers import adamw

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "checkpoint_inventory.json")


def _inv(shapes, **kw):
    return adamw.build_inventory({k: tuple(v) for k, v in shapes.items()}, **kw)


@pytest.mark.parametrize("case", json.load(open(GOLDEN)), ids=lambda c: c["format_id"])
def test_inventory_hash_matches_the_reference(case):
    inv = _inv(case["shapes"], format_id=case["format_id"], decayed_names=frozenset(case["decayed"]),
               frozen_names=frozenset(case.get("frozen", [])),
               quantization_profile=case.get("quantization_profile"),
               quantized_names=frozenset(case.get("quantized", [])),
               source_dtype=case.get("source_dtype", "bfloat16"))
    assert inv.sha256 == case["sha256"]
    assert inv.parameter_count == case["parameter_count"]


def _groups(values):
    return {g: {n: np.asarray(v, np.float32) for n, v in values[g].items()} for g in ("params", "m", "v")}


def test_complete_state_and_cursor_round_trip(tmp_path):
    inv = _inv({"weight": (2,)}, format_id="synthetic/1")
    groups = _groups({"params": {"weight": [1.0, -2.0]}, "m": {"weight": [0.25, 0.5]},
                      "v": {"weight": [0.125, 0.25]}})
    cursor = ts.Cursor("run", "data-hash", "source", 17)
    dest = tmp_path / "step-000003"
    ts.save_arrays(dest, groups, 3, inv, optimizer_id="adamw-config", cursor=cursor)
    got, step, restored_cursor = ts.load_arrays(dest, inv, optimizer_id="adamw-config", run_id="run",
                                                data_sha256="data-hash", source_id="source")
    assert restored_cursor == cursor and step == 3
    for g in ("params", "m", "v"):
        np.testing.assert_array_equal(got[g]["weight"], groups[g]["weight"])
    with pytest.raises(ValueError, match="identity"):
        ts.load_arrays(dest, inv, optimizer_id="adamw-config", run_id="other", data_sha256="data-hash",
                       source_id="source")
    with pytest.raises(ValueError, match="identity"):
        ts.load_arrays(dest, inv, optimizer_id="other-optimizer", run_id="run", data_sha256="data-hash",
                       source_id="source")
    manifest_path = dest / "manifest.json"
    text = manifest_path.read_text()
    assert text.endswith("\n") and ", " not in text and ": " not in text  # canonical JSON
    manifest = json.loads(text)
    assert manifest["format"] == "minifield.full-training-state/1"
    assert manifest["inventory_sha256"] == inv.sha256
    manifest["tensor_sha256"] = "0" * 64
    manifest_path.write_text(json.dumps(manifest))
    with pytest.raises(ValueError, match="SHA-256"):
        ts.load_arrays(dest, inv, optimizer_id="adamw-config", run_id="run", data_sha256="data-hash",
                       source_id="source")


def test_strided_parameter_and_moments_round_trip(tmp_path):
    inv = _inv({"conv.weight": (8, 1, 3)}, format_id="synthetic/strided")
    expected = np.arange(24, dtype=np.float32).reshape(8, 1, 3)[:, :, ::-1]
    assert not expected.flags.c_contiguous
    groups = {"params": {"conv.weight": expected}, "m": {"conv.weight": expected + 24},
              "v": {"conv.weight": expected + 48}}
    dest = tmp_path / "checkpoint"
    ts.save_arrays(dest, groups, 0, inv, optimizer_id="adamw", cursor=ts.Cursor("run", "data", "source", 0))
    got, _, _ = ts.load_arrays(dest, inv, optimizer_id="adamw", run_id="run", data_sha256="data",
                               source_id="source")
    np.testing.assert_array_equal(got["params"]["conv.weight"], expected)
    np.testing.assert_array_equal(got["m"]["conv.weight"], expected + 24)
    np.testing.assert_array_equal(got["v"]["conv.weight"], expected + 48)


def test_tensor_file_is_plain_safetensors(tmp_path):
    """The reference loads the tensor file with safetensors.numpy.load_file: keys, dtypes and shapes."""
    from safetensors.numpy import load_file
    inv = _inv({"a": (3, 2), "b": (4,)}, format_id="synthetic/2", decayed_names=frozenset({"a"}))
    rng = np.random.default_rng(0)
    groups = {g: {"a": rng.standard_normal((3, 2)).astype(np.float32),
                  "b": rng.standard_normal(4).astype(np.float32)} for g in ("params", "m", "v")}
    groups["v"] = {n: np.abs(x) for n, x in groups["v"].items()}  # second moments are non-negative
    dest = tmp_path / "c"
    ts.save_arrays(dest, groups, 5, inv, optimizer_id="x", cursor=ts.Cursor("r", "d", "s", 1))
    arrays = load_file(str(dest / "state.safetensors"))
    assert set(arrays) == {"params/a", "params/b", "m/a", "m/b", "v/a", "v/b", "step"}
    assert arrays["step"].dtype == np.int32 and arrays["step"].shape == () and int(arrays["step"]) == 5
    np.testing.assert_array_equal(arrays["m/a"], groups["m"]["a"])
    assert ts.digest_file(dest / "state.safetensors") == json.loads((dest / "manifest.json").read_text())[
        "tensor_sha256"]


def test_invalid_state_and_layout_are_rejected(tmp_path):
    inv = _inv({"w": (2,)}, format_id="synthetic/1")
    ok = _groups({"params": {"w": [1, 2]}, "m": {"w": [0, 0]}, "v": {"w": [0, 0]}})
    cur = ts.Cursor("r", "d", "s", 0)
    for g, bad, what in (("params", [np.nan, 1], "parameter"), ("m", [np.inf, 0], "first moment"),
                         ("v", [-1, 0], "second moment")):
        groups = {k: dict(v) for k, v in ok.items()}
        groups[g] = {"w": np.asarray(bad, np.float32)}
        with pytest.raises(ValueError, match=what):
            ts.save_arrays(tmp_path / f"bad-{g}", groups, 0, inv, optimizer_id="x", cursor=cur)
    with pytest.raises(ValueError, match="Invalid checkpoint tensor"):
        ts.save_arrays(tmp_path / "shape", {k: {"w": np.zeros(3, np.float32)} for k in ok}, 0, inv,
                       optimizer_id="x", cursor=cur)
    ts.save_arrays(tmp_path / "good", ok, 0, inv, optimizer_id="x", cursor=cur)
    with pytest.raises(FileExistsError):
        ts.save_arrays(tmp_path / "good", ok, 0, inv, optimizer_id="x", cursor=cur)
    other = _inv({"w": (2,), "u": (1,)}, format_id="synthetic/1")
    with pytest.raises(ValueError, match="identity"):
        ts.load_arrays(tmp_path / "good", other, optimizer_id="x", run_id="r", data_sha256="d", source_id="s")
    with pytest.raises(ValueError):
        ts.Cursor("", "d", "s", 0)
    with pytest.raises(ValueError):
        ts.Cursor("r", "d", "s", -1)
