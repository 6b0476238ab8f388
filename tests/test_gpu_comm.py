"""The library's NCCL communicator (mfb_comm_*) on the GPU.

One GPU: a one-rank communicator's collectives are identities; a wait whose
deadline passes while the stream is still busy (queued GEMMs that finish on
their own) aborts the communicator and raises CommError, and the aborted
communicator rejects later calls; a communicator whose second rank never
joins fails its initialisation at the deadline instead of waiting for ever.
Two GPUs (skipped on one): SUM all-reduce, reduce-scatter, all-gather,
reduce to a root and broadcast from a root across two processes give the exact
sums and blocks (the non-root's reduce buffer keeps its own values). NVLS stays
off.
"""

import ctypes
import os

import numpy as np
import pytest

from tests._util import run_ranks
from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu


def _child_one_rank(uid_path, out):
    from minifield_training_b200 import comm, device
    from minifield_training_b200.device import DeviceArray

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    device.set_device(0)
    c = comm.Communicator(1, 0, comm.unique_id_via_file(uid_path, 0), timeout_s=60.0)
    x = np.arange(1000, dtype=np.float32) - 3.5
    a = DeviceArray.from_numpy(x, "float32")
    c.allreduce(a)
    g = DeviceArray((1000,), "float32")
    c.all_gather(a, g)
    r = DeviceArray((1000,), "float32")
    c.reduce_scatter(g, r)
    c.reduce(r, 0)
    c.broadcast(r, 0)
    c.wait()
    out["values"] = (a.numpy(), g.numpy(), r.numpy())
    c.close()


def _child_deadline(uid_path, out):
    from minifield_training_b200 import _lib, comm, device
    from minifield_training_b200.device import DeviceArray

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    device.set_device(0)
    c = comm.Communicator(1, 0, comm.unique_id_via_file(uid_path, 0), timeout_s=60.0)
    s = ctypes.c_void_p()
    _lib.call("mfb_stream_create", ctypes.byref(s))
    n = 8192
    a = DeviceArray.zeros((n, n), "bfloat16")
    o = DeviceArray((n, n), "float32")
    for _ in range(40):  # about 30 ms of tensor-core work that ends by itself
        _lib.call("mfb_gemm_bf16", ctypes.c_void_p(a.ptr), _lib.MAJOR_K, n, ctypes.c_void_p(a.ptr), _lib.MAJOR_K, n,
                  ctypes.c_void_p(o.ptr), n, _lib.DTYPE_F32, n, n, n, ctypes.c_float(1.0), None, s.value)
    try:
        c.wait(s.value, timeout_s=1e-4)
        out["wait"] = "returned"
    except comm.CommError as exc:
        out["wait"] = str(exc)
    try:
        c.allreduce(o.view(0, (16,)), stream=s.value)
        out["after"] = "accepted"
    except comm.CommError as exc:
        out["after"] = str(exc)
    _lib.call("mfb_stream_sync", s.value)
    _lib.call("mfb_stream_destroy", s.value)
    c.close()


def _child_missing_rank(uid_path, out):
    from minifield_training_b200 import comm, device

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    device.set_device(0)
    uid = comm.unique_id_via_file(uid_path, 0)
    try:
        comm.Communicator(2, 0, uid, timeout_s=3.0)  # rank 1 never joins
        out["init"] = "joined"
    except comm.CommError as exc:
        out["init"] = str(exc)


def _run_one(target, tmp_path, timeout=180):
    import multiprocessing as mp

    require_gpu()
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    run_ranks(ctx, target, [(str(tmp_path / "nccl.id"), out)], timeout)
    return dict(out)


def test_one_rank_collectives_are_identities(tmp_path):
    a, g, r = _run_one(_child_one_rank, tmp_path)["values"]
    x = np.arange(1000, dtype=np.float32) - 3.5
    for got in (a, g, r):
        np.testing.assert_array_equal(got, x)


def test_a_missed_wait_deadline_aborts_the_communicator(tmp_path):
    out = _run_one(_child_deadline, tmp_path)
    assert "did not finish within" in out["wait"], out
    assert "aborted" in out["after"], out


def test_initialisation_fails_at_the_deadline_when_a_rank_never_joins(tmp_path):
    out = _run_one(_child_missing_rank, tmp_path)
    assert out["init"] != "joined" and "aborted" in out["init"], out


def _child_two_ranks(rank, uid_path, out):
    from minifield_training_b200 import comm, device
    from minifield_training_b200.device import DeviceArray

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    device.set_device(rank)
    c = comm.Communicator(2, rank, comm.unique_id_via_file(uid_path, rank), timeout_s=120.0)
    rng = np.random.default_rng(rank)
    x = rng.standard_normal(4096).astype(np.float32)
    a = DeviceArray.from_numpy(x, "float32")
    c.allreduce(a)
    r = DeviceArray((2048,), "float32")
    c.reduce_scatter(DeviceArray.from_numpy(x, "float32"), r)
    g = DeviceArray((8192,), "float32")
    c.all_gather(DeviceArray.from_numpy(x, "float32"), g)
    d = DeviceArray.from_numpy(np.array([rank + 0.5, -rank, 3.0], np.float64).view(np.uint8), "uint8")
    c.allreduce_f64(d.ptr, 3, op=comm.MAX)
    red = DeviceArray.from_numpy(x, "float32")
    c.reduce(red, 1)  # the sum lands on rank 1 only
    b = DeviceArray.from_numpy(x, "float32")
    c.broadcast(b, 0)  # rank 0's values everywhere
    c.wait()
    out[rank] = (x, a.numpy(), r.numpy(), g.numpy(), d.numpy().view(np.float64), red.numpy(), b.numpy())
    c.close()


def test_two_rank_collectives_are_exact(tmp_path):
    import multiprocessing as mp

    require_gpu()
    from minifield_training_b200 import device
    if device.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    uid = str(tmp_path / "nccl.id")
    run_ranks(ctx, _child_two_ranks, [(r, uid, out) for r in range(2)], 240)
    (x0, a0, r0, g0, d0, red0, b0), (x1, a1, r1, g1, d1, red1, b1) = out[0], out[1]
    total = x0 + x1  # a two-term float32 sum is the same in either order
    np.testing.assert_array_equal(a0, total)
    np.testing.assert_array_equal(a1, total)
    np.testing.assert_array_equal(r0, total[:2048])
    np.testing.assert_array_equal(r1, total[2048:])
    for g in (g0, g1):
        np.testing.assert_array_equal(g, np.concatenate((x0, x1)))
    for d in (d0, d1):
        np.testing.assert_array_equal(d, [1.5, 0.0, 3.0])
    np.testing.assert_array_equal(red1, total)
    np.testing.assert_array_equal(red0, x0)
    np.testing.assert_array_equal(b0, x0)
    np.testing.assert_array_equal(b1, x0)
