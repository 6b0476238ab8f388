"""Data-parallel encoder step on two GPUs against one GPU (needs >= 2 GPUs; skipped otherwise).

Two NCCL ranks (the library's communicator, mfb_comm_*; the unique id goes
through a file) each take one row of a two-row batch; after the bucketed
allreduce their gradient sums, loss sum and count must equal a single GPU's
over both rows (up to FP32 summation order: rel-L2 1e-4 per leaf), and after
the AdamW commit both ranks must hold bit-identical masters (replicated state,
engine/step.py:62 and the data-parallel known answers' replication checks),
with the replicated transaction and with the optimizer sharded across the
ranks (each rank owns a bucket-aligned range: its gradients are reduced to it,
it updates it, and it broadcasts the masters back, overlapped with the next
step's forward).
Ranks run as child processes; NCCL's NVLS is off, as for every multi-rank
test on this pool.
"""

import dataclasses
import os

import numpy as np
import pytest

from tests._util import run_ranks
from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu


def _cfg():
    from minifield_training_b200 import workloads
    return dataclasses.replace(workloads.CONFIG5, global_batch=2, length=128, ffn=256,
                               layer_types=("conv", "full_attention"), vocab=1000)


def _comm(rank, uid_path):
    from minifield_training_b200 import comm as mcomm
    from minifield_training_b200 import device

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    device.set_device(rank)
    return mcomm.Communicator(2, rank, mcomm.unique_id_via_file(uid_path, rank), timeout_s=120.0)


def _rank_graph(rank, uid_path, out, shard=False):
    """Two captured-graph steps per rank (forward/per-layer backward/commit graphs around the bucket reductions)."""
    import ctypes

    from minifield_training_b200 import _lib, workloads
    from minifield_training_b200.models import encoder as me
    comm = _comm(rank, uid_path)
    cfg = _cfg()
    s = ctypes.c_void_p()
    _lib.call("mfb_stream_create", ctypes.byref(s))
    step = me.EncoderStep(cfg, rows=1, seed=0, comm=comm, stream=s.value, shard_optimizer=shard)
    step.set_batch(*workloads.encoder_batch(cfg, 7, rows=1, row0=rank))
    step.capture()
    losses = []
    for _ in range(2):
        res = step.step()
        losses.append((res.committed, res.loss))
    step.settle()  # the sharded optimizer's last master broadcast
    comm.wait(s.value)
    params = {n: v.numpy() for n, v in step.params.items() if n != "lfm2.embed_tokens.weight"}
    out[rank] = (losses, params)
    step.close()
    comm.close()


def _rank(rank, uid_path, out, shard=False):
    from minifield_training_b200 import workloads
    from minifield_training_b200.models import encoder as me
    comm = _comm(rank, uid_path)
    cfg = _cfg()
    step = me.EncoderStep(cfg, rows=1, seed=0, comm=comm, shard_optimizer=shard)
    step.set_batch(*workloads.encoder_batch(cfg, 7, rows=1, row0=rank))
    step.quantize()
    step.forward()
    red = step.reducer()
    step.backward(red.layer_done)
    red.finish()
    comm.wait(None)
    grads = {n: v.numpy() for n, v in step.gviews.items()}
    lc = step.loss_count.numpy()
    step._commit()
    step.settle()
    comm.wait(None)
    committed = step.result.committed
    params = {n: v.numpy() for n, v in step.params.items() if n != "lfm2.embed_tokens.weight"}
    owners = {n: step.grad_owner(n) for n in grads}
    out[rank] = (grads, lc, committed, params, owners)
    step.close()
    comm.close()


@pytest.mark.parametrize("shard", [False, True], ids=["replicated", "sharded_optimizer"])
def test_two_rank_step_matches_one_gpu(shard, tmp_path):
    require_gpu()
    from minifield_training_b200 import device
    if device.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    uid = str(tmp_path / "nccl.id")
    run_ranks(ctx, _rank, [(r, uid, out, shard) for r in range(2)], 300)
    # One GPU over both rows.
    from minifield_training_b200 import workloads
    from minifield_training_b200.device import sync
    from minifield_training_b200.models import encoder as me
    cfg = _cfg()
    ref = me.EncoderStep(cfg, rows=2, seed=0)
    ref.set_batch(*workloads.encoder_batch(cfg, 7))
    ref.quantize()
    ref.forward()
    ref.backward()
    sync()
    g0, lc0, c0, p0, own = out[0]
    g1, lc1, c1, p1, _ = out[1]
    np.testing.assert_allclose(lc0, ref.loss_count.numpy(), rtol=1e-4)
    np.testing.assert_array_equal(lc0, lc1)
    for name, v in ref.gviews.items():
        r = v.numpy().astype(np.float64)
        # Replicated: both ranks hold the sum. Sharded: the leaf's owner does (the other keeps its own part).
        g = (g0, g1)[own[name]][name]
        if not shard:
            np.testing.assert_array_equal(g0[name], g1[name])
        err = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)
        assert err < 1e-4, (name, err)
    assert c0 and c1
    for name in p0:
        np.testing.assert_array_equal(p0[name], p1[name])


@pytest.mark.parametrize("shard", [False, True], ids=["replicated", "sharded_optimizer"])
def test_two_rank_graph_steps_stay_replicated_and_match_eager(shard, tmp_path):
    """Captured-graph steps on two NCCL ranks: both ranks commit, stay bit-identical, and match one eager GPU."""
    require_gpu()
    from minifield_training_b200 import device
    if device.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    uid = str(tmp_path / "nccl.id")
    run_ranks(ctx, _rank_graph, [(r, uid, out, shard) for r in range(2)], 300)
    (l0, p0), (l1, p1) = out[0], out[1]
    assert all(c for c, _ in l0) and l0 == l1
    for name in p0:
        np.testing.assert_array_equal(p0[name], p1[name])
    # One eager GPU over both rows, two steps.
    from minifield_training_b200 import workloads
    from minifield_training_b200.models import encoder as me
    cfg = _cfg()
    ref = me.EncoderStep(cfg, rows=2, seed=0)
    ref.set_batch(*workloads.encoder_batch(cfg, 7))
    for k in range(2):
        r = ref.step()
        # Step 0's loss is the same sum in another order; step 1's follows the
        # first update, where sign flips of near-zero gradients (below) move it.
        np.testing.assert_allclose(l0[k][1], r.loss, rtol=1e-4 if k == 0 else 2e-3)
    # Adam's first steps move each master by about lr * sign(g): a gradient
    # within summation noise of zero may flip sign between the two reduction
    # orders (a 2 * lr difference), so allow that bound on a tiny fraction.
    for name in p0:
        diff = np.abs(p0[name] - ref.params[name].numpy())
        assert diff.max() <= 4.5 * cfg.learning_rate, name
        assert np.mean(diff > cfg.learning_rate) < 2e-3, name  # only sign flips move a master by ~lr
