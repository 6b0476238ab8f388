"""Host side of the NCCL communicator (no GPU): loading NCCL, the unique id, its file exchange, and
argument errors raised before any collective is enqueued."""

import multiprocessing as mp

import pytest

from minifield_training_b200 import comm


def test_nccl_loads_and_draws_distinct_unique_ids():
    assert comm.load() >= 21900  # ncclCommInitRankConfig non-blocking mode and ncclCommFinalize
    a, b = comm.unique_id(), comm.unique_id()
    assert len(a) == len(b) == 128 and a != b


def _reader(path, out):
    out["id"] = comm.unique_id_via_file(path, 1, timeout_s=60.0)


def test_unique_id_reaches_the_other_rank_through_a_file(tmp_path):
    path = str(tmp_path / "nccl.id")
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    p = ctx.Process(target=_reader, args=(path, out))
    p.start()
    try:
        uid = comm.unique_id_via_file(path, 0)
        p.join(60)
    finally:
        if p.is_alive():
            p.kill()
            p.join(5)
    assert p.exitcode == 0 and out["id"] == uid


def test_unique_id_wait_is_bounded(tmp_path):
    with pytest.raises(comm.CommError, match="no NCCL unique id"):
        comm.unique_id_via_file(str(tmp_path / "never"), 1, timeout_s=0.2)


def test_collectives_reject_bad_arguments_before_enqueueing():
    import ctypes

    from minifield_training_b200 import _lib

    comm.load()
    with pytest.raises(ValueError, match="communicator is NULL"):
        _lib.call("mfb_comm_allreduce", None, None, None, 0, comm.F32, comm.SUM, None)
    with pytest.raises(ValueError, match="rank 2 out of range"):
        h = ctypes.c_void_p()
        uid = comm.unique_id()
        _lib.call("mfb_comm_init", uid, len(uid), 2, 2, ctypes.c_double(1.0), ctypes.byref(h))
    with pytest.raises(ValueError, match="unique id must be"):
        h = ctypes.c_void_p()
        _lib.call("mfb_comm_init", b"x" * 16, 16, 1, 0, ctypes.c_double(1.0), ctypes.byref(h))
