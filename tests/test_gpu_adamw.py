"""AdamW transaction on the GPU (mfb_adamw_commit via optimizers.adamw) against oracle/adamw.py.

Without clipping both sides run the same float32 operations in the same order,
so committed leaves must match bit for bit; with clipping the device's FP64
norm can move the clip scale by an ulp, so leaves are compared at rtol 2e-6.
Rejections must leave every arena byte unchanged.
"""

import ctypes
import os

import numpy as np
import pytest

from oracle import adamw as oa
from tests._util import run_ranks
from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu
F = np.float32


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


def _upload(view, host):
    from minifield_training_b200 import _lib
    host = np.ascontiguousarray(np.asarray(host, F))
    _lib.call("mfb_memcpy_h2d", ctypes.c_void_p(view.ptr), host.ctypes.data_as(ctypes.c_void_p), host.nbytes, None)


def _make(shapes, decayed, frozen, params, m, v, step=0):
    from minifield_training_b200.optimizers import adamw
    inv = adamw.build_inventory(shapes, decayed_names=frozenset(decayed), frozen_names=frozenset(frozen))
    st = adamw.initialize_state(params, inv)
    for name in shapes:
        _upload(st["m"][name], m[name])
        _upload(st["v"][name], v[name])
    np_step = np.array([step], np.int32)
    from minifield_training_b200 import _lib
    _lib.call("mfb_memcpy_h2d", ctypes.c_void_p(st["step"].ptr), np_step.ctypes.data_as(ctypes.c_void_p), 4, None)
    return inv, st


def _read(st):
    return ({g: {n: st[g][n].numpy() for n in st[g]} for g in ("params", "m", "v")}, int(st["step"].numpy()[0]))


def _fixture():
    from tests.test_adamw_oracle import _grads, _state
    s = _state()
    shapes = {k: v.shape for k, v in s["params"].items()}
    return shapes, s, _grads()


def _cfg(**kw):
    c = dict(learning_rate=0.1, beta1=0.9, beta2=0.95, epsilon=1e-8, weight_decay=0.01, clip_norm=1.0)
    c.update(kw)
    return c


def _run_gpu(shapes, decayed, frozen, s, grads, loss=1.0, valid=True, **kw):
    from minifield_training_b200.optimizers import adamw
    inv, st = _make(shapes, decayed, frozen, s["params"], s["m"], s["v"], s["step"])
    before = _read(st)
    tr = adamw.make_transaction(inv, adamw.AdamWConfig(**_cfg(**kw)))
    res = tr(st, grads, F(loss), valid)
    return res, before, _read(st)


def test_reference_fixture_commits_bit_exactly():
    shapes, s, grads = _fixture()
    res, _, (after, step) = _run_gpu(shapes, {"w.matrix"}, {"w.frozen_matrix", "w.frozen_vector"}, s, grads,
                                     clip_norm=10.0)
    ref = oa.transition(s, grads, 1.0, True, _cfg(clip_norm=10.0), {"w.matrix", "w.vector"}, {"w.matrix"})
    assert res.committed and res.code == 0 and step == 1
    for g in ("params", "m", "v"):
        for n in shapes:
            np.testing.assert_array_equal(after[g][n], ref[0][g][n], err_msg=f"{g}/{n}")
    np.testing.assert_allclose(res.gradient_norm, ref[4], rtol=1e-6)
    np.testing.assert_allclose(res.clipped_gradient_norm, ref[5], rtol=1e-6)
    np.testing.assert_allclose(res.update_norm, ref[6], rtol=1e-5)


@pytest.mark.parametrize("case,code", [("grad", 4), ("loss", 2), ("acc", 1), ("m_inf", 3), ("v_neg", 3),
                                       ("v_nan", 3), ("step", 5), ("candidate", 6)])
def test_rejections_write_nothing(case, code):
    shapes, s, grads = _fixture()
    loss, valid, kw = 1.0, True, {}
    if case == "grad":
        grads["w.vector"] = np.array([np.nan, 0, 0], F)
    elif case == "loss":
        loss = np.nan
    elif case == "acc":
        valid = False
    elif case == "m_inf":
        s["m"]["w.vector"] = np.array([np.inf, 0, 0], F)
    elif case == "v_neg":
        s["v"]["w.vector"] = np.array([-1.0, 0, 0], F)
    elif case == "v_nan":
        s["v"]["w.frozen_vector"] = np.array([0, np.nan, 0, 0], F)
    elif case == "step":
        s["step"] = 2**31 - 1
    elif case == "candidate":
        s["params"]["w.matrix"] = np.full((2, 3), 1e38, F)
        grads = {k: np.zeros_like(v) for k, v in grads.items()}
        kw = dict(learning_rate=1.0, weight_decay=4.0, clip_norm=1e30)
    from minifield_training_b200.optimizers import adamw
    inv, st = _make(shapes, {"w.matrix"}, {"w.frozen_matrix", "w.frozen_vector"}, s["params"], s["m"], s["v"],
                    s["step"])
    before = _read(st)
    res = adamw.make_transaction(inv, adamw.AdamWConfig(**_cfg(**kw)))(st, grads, F(loss), valid)
    assert not res.committed and int(res.code) == code
    after = _read(st)
    assert after[1] == before[1]
    for g in ("params", "m", "v"):
        for n in shapes:
            np.testing.assert_array_equal(after[0][g][n].view(np.uint32), before[0][g][n].view(np.uint32))
    if code != 6:
        assert np.isnan(res.gradient_norm) and np.isnan(res.update_norm)


@pytest.mark.parametrize("clip", [1e6, 0.5])
def test_large_ragged_arena_matches_oracle(clip):
    rng = np.random.default_rng(7)
    shapes = {"a.decayed": (1023, 517), "b.decayed": (3, 5), "c.plain": (1001,), "d.plain": (64, 3, 7),
              "e.frozen": (333, 129), "f.plain": (7,)}
    decayed, frozen = {"a.decayed", "b.decayed"}, {"e.frozen"}
    s = {"params": {k: rng.standard_normal(sh, dtype=F) for k, sh in shapes.items()},
         "m": {k: (rng.standard_normal(sh, dtype=F) * F(0.01)) for k, sh in shapes.items()},
         "v": {k: np.abs(rng.standard_normal(sh, dtype=F)) * F(1e-4) for k, sh in shapes.items()}, "step": 41}
    for k in frozen:
        s["m"][k][:] = 0
        s["v"][k][:] = 0
    grads = {k: rng.standard_normal(sh, dtype=F) * F(1e-3) for k, sh in shapes.items() if k not in frozen}
    grads["c.plain"][:10] = 0  # m_hat == 0 where the moment is also zero
    s["m"]["c.plain"][:10] = 0
    res, _, (after, step) = _run_gpu(shapes, decayed, frozen, s, grads, clip_norm=clip, weight_decay=0.1)
    ref = oa.transition(s, grads, 1.0, True, _cfg(clip_norm=clip, weight_decay=0.1), set(grads), decayed)
    assert res.committed and ref[1] and step == 42
    np.testing.assert_allclose(res.gradient_norm, ref[4], rtol=1e-5)
    np.testing.assert_allclose(res.update_norm, ref[6], rtol=1e-4)
    for g in ("params", "m", "v"):
        for n in shapes:
            if clip > 1e5:
                np.testing.assert_array_equal(after[g][n], ref[0][g][n], err_msg=f"{g}/{n}")
            else:
                np.testing.assert_allclose(after[g][n], ref[0][g][n], rtol=2e-6, atol=1e-12, err_msg=f"{g}/{n}")


def test_normalized_step_divides_gradients_and_loss():
    from minifield_training_b200 import _lib
    from minifield_training_b200.device import DeviceArray
    from minifield_training_b200.optimizers import adamw
    shapes, s, grads = _fixture()
    count = F(6.0)
    sums = {k: v * count for k, v in grads.items()}
    inv, st = _make(shapes, {"w.matrix"}, {"w.frozen_matrix", "w.frozen_vector"}, s["params"], s["m"], s["v"])
    dev = lambda x, dt: DeviceArray.from_numpy(np.array([x]), dt)
    ls, cs = dev(F(12.0), "float32"), dev(count, "float32")
    loss, div, ok = DeviceArray((1,), "float32"), DeviceArray((1,), "float32"), DeviceArray((1,), "uint8")
    P = ctypes.c_void_p
    _lib.call("mfb_step_normalize", P(ls.ptr), P(cs.ptr), None, P(loss.ptr), P(div.ptr), P(ok.ptr), None)
    res = adamw.make_transaction(inv, adamw.AdamWConfig(**_cfg(clip_norm=10.0)))(st, sums, loss, ok, divisor=div)
    ref_loss, ref_grads, ref_valid = oa.normalize(F(12.0), count, sums)
    ref = oa.transition(s, ref_grads, ref_loss, ref_valid, _cfg(clip_norm=10.0), {"w.matrix", "w.vector"},
                        {"w.matrix"})
    assert res.committed and res.loss == pytest.approx(2.0)
    after, _ = _read(st)
    for g in ("params", "m", "v"):
        for n in shapes:
            np.testing.assert_array_equal(after[g][n], ref[0][g][n], err_msg=f"{g}/{n}")


def _sharded_vs_full(out, uid_path):
    """Child process: one-rank communicator, full vs sharded transaction on the same state."""
    from minifield_training_b200 import comm as mcomm
    from minifield_training_b200 import device
    from minifield_training_b200.device import DeviceArray, sync
    from minifield_training_b200.optimizers import adamw

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    device.set_device(0)
    communicator = mcomm.Communicator(1, 0, mcomm.unique_id_via_file(uid_path, 0), timeout_s=60.0)
    rng = np.random.default_rng(3)
    shapes = {"a.matrix": (37, 53), "b.matrix": (64, 16), "c.vector": (61,), "d.frozen": (9, 7)}
    inv = adamw.build_inventory(shapes, decayed_names=frozenset({"a.matrix", "b.matrix"}),
                                frozen_names=frozenset({"d.frozen"}))
    params = {n: rng.standard_normal(s).astype(F) for n, s in shapes.items()}
    m = {n: (rng.standard_normal(s) * 0.1).astype(F) for n, s in shapes.items()}
    v = {n: (rng.random(s) * 0.01).astype(F) for n, s in shapes.items()}
    cfg = adamw.AdamWConfig(**_cfg(clip_norm=0.5))
    results = {}
    for bad in (False, True):
        grads = {n: rng.standard_normal(shapes[n]).astype(F) for n in shapes if n != "d.frozen"}
        if bad:
            grads["b.matrix"][3, 5] = np.inf
        layout = adamw.Layout(inv)
        masters = DeviceArray.zeros((adamw.sharded_master_elements(layout, 1),), "float32")
        states = {}
        for kind in ("full", "sharded"):
            st = adamw.initialize_state(params, inv, params=masters if kind == "sharded" else None)
            for name in shapes:
                _upload(st["m"][name], m[name])
                _upload(st["v"][name], v[name])
            for name, g in grads.items():
                _upload(st.arenas["grads"].view(st.layout.offsets[name], g.shape), g)
            states[kind] = st
        r_full = adamw.make_transaction(inv, cfg)(states["full"], states["full"].gradient_tree(), F(0.7), True)
        r_sh = adamw.make_sharded_transaction(inv, cfg, communicator)(states["sharded"], F(0.7), True)
        sync()
        results[bad] = ([(r.code, r.committed, r.loss, r.gradient_norm, r.update_norm) for r in (r_full, r_sh)],
                        [_read(states[k]) for k in ("full", "sharded")])
    out["results"] = results
    communicator.close()


def test_sharded_transaction_on_one_rank_matches_the_full_one(tmp_path):
    """The sharded passes over a one-rank communicator reproduce mfb_adamw_commit bit for bit (commit and
    rejection)."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    run_ranks(ctx, _sharded_vs_full, [(out, str(tmp_path / "nccl.id"))], 240)
    for bad, (res, arenas) in out["results"].items():
        full, sharded = res
        assert full[0] == sharded[0] and full[1] == sharded[1], (bad, full, sharded)
        assert full[1] == (not bad)
        np.testing.assert_array_equal(np.array(full[2:], np.float64), np.array(sharded[2:], np.float64))
        (fa, fs), (sa, ss) = arenas
        assert fs == ss
        for g in ("params", "m", "v"):
            for n in fa[g]:
                np.testing.assert_array_equal(fa[g][n], sa[g][n], err_msg=f"{bad} {g}/{n}")


def test_checkpoint_resumes_the_device_state_exactly(tmp_path):
    """save -> verify_roundtrip -> load into fresh arenas -> the next commit matches the uninterrupted state."""
    from minifield_training_b200.checkpoints import training_state as ts
    from minifield_training_b200.optimizers import adamw

    shapes, s, grads = _fixture()
    decayed, frozen = {"w.matrix"}, {"w.frozen_matrix", "w.frozen_vector"}
    inv, st = _make(shapes, decayed, frozen, s["params"], s["m"], s["v"], s["step"])
    tr = adamw.make_transaction(inv, adamw.AdamWConfig(**_cfg(clip_norm=10.0)))
    assert tr(st, grads, F(1.0), True).committed
    cursor = ts.Cursor("run", "data", "source", 1)
    ts.save(tmp_path / "ck", st, inv, optimizer_id="adamw", cursor=cursor)
    ts.verify_roundtrip(tmp_path / "ck", st, cursor, inv, "adamw")
    st2, cur2 = ts.load(tmp_path / "ck", inv, optimizer_id="adamw", run_id="run", data_sha256="data",
                        source_id="source")
    assert cur2 == cursor
    (a1, s1), (a2, s2) = _read(st), _read(st2)
    assert s1 == s2
    for g in ("params", "m", "v"):
        for n in shapes:
            np.testing.assert_array_equal(a1[g][n], a2[g][n], err_msg=f"{g}/{n}")
    assert tr(st, grads, F(1.0), True).committed and tr(st2, grads, F(1.0), True).committed
    (a1, s1), (a2, s2) = _read(st), _read(st2)
    assert s1 == s2
    for g in ("params", "m", "v"):
        for n in shapes:
            np.testing.assert_array_equal(a1[g][n], a2[g][n], err_msg=f"after resume {g}/{n}")
