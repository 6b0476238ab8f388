"""Attention forward/backward kernels vs the oracle (and the reference KATs).

The oracle evaluates the reference's FP32 path on the same bf16-rounded
inputs the GPU receives. Gate: max-abs 2e-2 and relative-L2 1e-2 (see
tests/_util.py for the scaled max-abs on gradients); id encodings bit-exact.
"""

import numpy as np
import pytest

from oracle import attention as oatt
from oracle.bf16 import round_bf16
from tests._util import assert_close, report_errors
from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu

CAUSAL, PREFIX, PACKED, BIDIR = 0, 1, 2, 3


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


def _pad64(x):
    d = x.shape[-1]
    if d == 64:
        return x
    out = np.zeros(x.shape[:-1] + (64,), np.float32)
    out[..., :d] = x
    return out


def gpu_attention(mode, q, k, v, dout=None, mask=None, seg=None, aux=None, p=0):
    """Run ids + fwd (+ bwd) on the GPU. Head dims < 64 are zero-padded (same math)."""
    from minifield_training_b200.device import DeviceArray
    from minifield_training_b200.kernels import attention as A

    d = q.shape[-1]
    b, t = q.shape[0], q.shape[1]
    s = k.shape[1]
    qd = DeviceArray.from_numpy(_pad64(q), "bfloat16")
    kd = DeviceArray.from_numpy(_pad64(k), "bfloat16")
    vd = DeviceArray.from_numpy(_pad64(v), "bfloat16")

    def i32(x):
        return None if x is None else DeviceArray.from_numpy(np.asarray(x, np.int32), "int32")

    ids = A.build_ids(mode, i32(mask), i32(seg), i32(aux), b, t, s, p)
    out, res = A.attention_fwd_ids(qd, kd, vd, *ids, scale=d ** -0.5)
    result = {"out": out.float32()[..., :d], "qid": ids[0].numpy(), "kid": ids[1].numpy(), "ids": ids}
    if dout is not None:
        dq, dk, dv = A.attention_bwd(res, _pad64(dout))
        result.update(dq=dq.float32()[..., :d], dk=dk.float32()[..., :d], dv=dv.float32()[..., :d])
    return result


def oracle_attention(q, k, v, ids, dout=None, dtype=np.float64):
    qid, kid, causal, offset, policy = ids
    valid = oatt.valid_from_ids(qid, kid, causal, offset)
    qb, kb, vb = (round_bf16(x).astype(dtype) for x in (q, k, v))
    out = oatt.attention_forward(qb, kb, vb, valid, policy, dtype)
    if dout is None:
        return out, None
    return out, oatt.attention_backward(qb, kb, vb, valid, policy, round_bf16(dout).astype(dtype), dtype)


def _check(res, ref_out, ref_grads, what):
    assert_close(res["out"], ref_out, what=f"{what} O")
    report_errors(f"{what} O", res["out"], ref_out)
    if ref_grads is not None:
        for name, r in zip(("dq", "dk", "dv"), ref_grads):
            assert_close(res[name], r, scaled=True, what=f"{what} {name}")
            report_errors(f"{what} {name}", res[name], r)


# --- reference known answers -------------------------------------------------


def test_reference_dense_causal_case(golden):
    g = golden
    r = gpu_attention(CAUSAL, g["causal_q"], g["causal_k"], g["causal_v"], mask=g["causal_mask"])
    assert_close(r["out"], g["causal_out"], what="causal KAT")


def test_reference_prefix_case(golden):
    from minifield_training_b200.kernels import attention as A

    g = golden
    out = A.b200_prefix_causal_attention(
        _pad64(g["prefix_q"]), _pad64(g["prefix_pk"]), _pad64(g["prefix_pv"]), _pad64(g["prefix_k"]),
        _pad64(g["prefix_v"]), g["prefix_pmask"], g["prefix_smask"],
    )
    # Zero padding changes the default D^-0.5; compare on a D=64 recomputation instead.
    ids = oatt.prefix_ids(g["prefix_pmask"], g["prefix_smask"])
    kk = np.concatenate((g["prefix_pk"], g["prefix_k"]), 1)
    vv = np.concatenate((g["prefix_pv"], g["prefix_v"]), 1)
    valid = oatt.valid_from_ids(*ids[:4])
    ref = oatt.attention_forward(
        round_bf16(_pad64(g["prefix_q"])).astype(np.float64), round_bf16(_pad64(kk)).astype(np.float64),
        round_bf16(_pad64(vv)).astype(np.float64), valid, ids[4])
    assert_close(out.float32(), ref, what="prefix (D=64 scale)")
    r = gpu_attention(PREFIX, g["prefix_q"], kk, vv, mask=g["prefix_smask"], aux=g["prefix_pmask"],
                      p=g["prefix_pk"].shape[1])
    assert_close(r["out"], g["prefix_out"], what="prefix KAT")


def test_reference_packed_case(golden):
    g = golden
    r = gpu_attention(PACKED, g["packed_q"], g["packed_k"], g["packed_v"], mask=g["packed_mask"], seg=g["packed_seg"])
    assert_close(r["out"], g["packed_out"], what="packed KAT")


def test_reference_cached_case(golden):
    from minifield_training_b200.kernels import attention as A

    g = golden
    # Scale: D=8 in the KAT; pre-scale q so the kernel's D=64 scale reproduces it.
    q = _pad64(g["cached_q"]) * np.float32((8 ** -0.5) / (64 ** -0.5))
    out = A.b200_cached_attention(q, _pad64(g["cached_k"]), _pad64(g["cached_v"]), g["cached_len"])
    assert_close(out.float32()[..., :8], g["cached_out"], what="cached KAT")


def test_reference_bidirectional_uniform_case(golden):
    g = golden
    r = gpu_attention(BIDIR, g["bidir_uniform_q"], g["bidir_uniform_k"], g["bidir_uniform_v"],
                      dout=np.ones((1, 3, 2, 2), np.float32), mask=g["bidir_uniform_mask"])
    assert_close(r["out"], g["bidir_uniform_out"], what="uniform O")
    assert_close(r["dv"], g["bidir_uniform_dv"], what="uniform dV")
    r = gpu_attention(BIDIR, g["bidir_uniform_q"], g["bidir_uniform_k"], g["bidir_uniform_v"],
                      mask=np.zeros((1, 3), np.int32))
    np.testing.assert_array_equal(r["out"], np.zeros((1, 3, 2, 2)))


def test_reference_bidirectional_packed_case(golden):
    g = golden
    seg = g["bidir_packed_seg"]
    r = gpu_attention(BIDIR, g["bidir_packed_q"], g["bidir_packed_k"], g["bidir_packed_v"],
                      dout=np.ones((1, 6, 2, 2), np.float32), mask=(seg != 0).astype(np.int32), seg=seg)
    assert_close(r["out"], g["bidir_packed_out"], what="packed bidir O")
    assert_close(r["dv"], g["bidir_packed_dv"], what="packed bidir dV")


# --- randomized parity, every mask shape, ragged lengths ---------------------


def _qkvd(seed, b, t, s, h=4, hk=2, d=64):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((b, t, h, d), dtype=np.float32), rng.standard_normal((b, s, hk, d), dtype=np.float32),
            rng.standard_normal((b, s, hk, d), dtype=np.float32), rng.standard_normal((b, t, h, d), dtype=np.float32))


@pytest.mark.parametrize("t", [64, 200])
def test_causal_with_key_mask_and_empty_rows(t):
    q, k, v, do = _qkvd(1, 2, t, t)
    mask = np.ones((2, t), np.int32)
    mask[0, :3] = 0  # rows 0..2 of batch 0 have no valid key -> uniform average over all keys
    mask[1, t // 2 :] = 0
    r = gpu_attention(CAUSAL, q, k, v, do, mask=mask)
    ids = oatt.causal_ids(mask)
    np.testing.assert_array_equal(r["qid"], ids[0])
    np.testing.assert_array_equal(r["kid"], ids[1])
    out, grads = oracle_attention(q, k, v, ids, do)
    _check(r, out, grads, f"causal T={t}")


def test_packed_causal_segments():
    from minifield_training_b200 import workloads

    t = 320
    q, k, v, do = _qkvd(2, 2, t, t)
    seg = workloads.packed_segments(5, 2, t, lo=16, hi=120)
    seg[1, -20:] = 0
    mask = np.ones((2, t), np.int32)
    mask[0, 10] = 0  # an inactive token inside a segment
    r = gpu_attention(PACKED, q, k, v, do, mask=mask, seg=seg)
    ids = oatt.packed_ids(mask, seg)
    np.testing.assert_array_equal(r["qid"], ids[0])
    np.testing.assert_array_equal(r["kid"], ids[1])
    out, grads = oracle_attention(q, k, v, ids, do)
    _check(r, out, grads, "packed")


@pytest.mark.parametrize("with_segments", [False, True])
def test_bidirectional(with_segments):
    from minifield_training_b200 import workloads

    t = 300
    q, k, v, do = _qkvd(3, 3, t, t)
    mask = np.ones((3, t), np.int32)
    mask[1, 250:] = 0
    mask[2] = 0  # empty row: zeros out, zero gradients
    seg = workloads.packed_segments(9, 3, t, lo=20, hi=150) if with_segments else None
    r = gpu_attention(BIDIR, q, k, v, do, mask=mask, seg=seg)
    ids = oatt.bidirectional_ids(mask, seg)
    np.testing.assert_array_equal(r["qid"], ids[0])
    np.testing.assert_array_equal(r["kid"], ids[1])
    out, grads = oracle_attention(q, k, v, ids, do)
    _check(r, out, grads, f"bidir seg={with_segments}")
    assert not np.any(r["out"][2]) and not np.any(r["dq"][2])


def test_prefix_forward_and_backward():
    q, k, v, do = _qkvd(4, 2, 100, 137)
    pmask = np.ones((2, 37), np.int32)
    pmask[1, 20:] = 0
    smask = np.ones((2, 100), np.int32)
    smask[0, 90:] = 0
    r = gpu_attention(PREFIX, q, k, v, do, mask=smask, aux=pmask, p=37)
    ids = oatt.prefix_ids(pmask, smask)
    out, grads = oracle_attention(q, k, v, ids, do)
    _check(r, out, grads, "prefix")


def test_gqa_group_of_four():
    q, k, v, do = _qkvd(6, 1, 128, 128, h=8, hk=2)
    mask = np.ones((1, 128), np.int32)
    r = gpu_attention(CAUSAL, q, k, v, do, mask=mask)
    out, grads = oracle_attention(q, k, v, oatt.causal_ids(mask), do)
    _check(r, out, grads, "gqa4")


# --- benchmark configurations -----------------------------------------------


def test_config1_dense_causal_full_size():
    from minifield_training_b200 import workloads

    q, k, v, do, mask, _ = workloads.attention_inputs(workloads.CONFIG1, seed=0)
    r = gpu_attention(CAUSAL, q, k, v, do, mask=mask)
    out, grads = oracle_attention(q, k, v, oatt.causal_ids(mask), do, dtype=np.float32)
    _check(r, out, grads, "config1")


def test_config2_segment_bidirectional_full_batch_all_rows():
    """The headline batch (8 rows, each with its own segment layout) against the oracle, every row;
    the oracle runs two rows at a time (a chunk's FP32 score grids take about 2.5 GB)."""
    from minifield_training_b200 import workloads

    q, k, v, do, mask, seg = workloads.attention_inputs(workloads.CONFIG2, seed=0)
    r = gpu_attention(BIDIR, q, k, v, do, mask=mask, seg=seg)
    ids = oatt.bidirectional_ids(mask, seg)
    np.testing.assert_array_equal(r["qid"], ids[0])
    np.testing.assert_array_equal(r["kid"], ids[1])
    for lo in range(0, q.shape[0], 2):
        rows = slice(lo, lo + 2)
        sub = tuple(x[rows] for x in ids[:2]) + ids[2:]
        out, grads = oracle_attention(q[rows], k[rows], v[rows], sub, do[rows], dtype=np.float32)
        got = {key: r[key][rows] for key in ("out", "dq", "dk", "dv")}
        _check(got, out, grads, f"config2 rows {lo}-{lo + 1}")


def test_rows_of_one_warp_that_rescale_differently():
    """The forward's lazy rescale must stay warp-collective when rows diverge.

    Keys of the first 128-key tile score 0 for every query; keys of the later
    tiles score about 50 (> 2^8 in the log2 domain after the 1/8 scale) for
    even query rows only, so in every warp half the rows move their reference
    max after the first tile and half do not.
    """
    rng = np.random.default_rng(11)
    t, d = 512, 64
    u = np.zeros(d, np.float32)
    u[0] = np.sqrt(50.0)
    q = np.zeros((1, t, 2, d), np.float32)
    q[0, 0::2, :, :] = u
    q[0, 1::2, :, 1] = np.sqrt(50.0)  # orthogonal to every key
    k = np.zeros((1, t, 1, d), np.float32)
    k[0, 128:, 0, :] = u
    k += rng.standard_normal(k.shape).astype(np.float32) * 0.01
    v = rng.standard_normal((1, t, 1, d)).astype(np.float32)
    do = rng.standard_normal((1, t, 2, d)).astype(np.float32)
    mask = np.ones((1, t), np.int32)
    r = gpu_attention(BIDIR, q, k, v, do, mask=mask)
    ids = oatt.bidirectional_ids(mask, None)
    out, grads = oracle_attention(q, k, v, ids, do)
    _check(r, out, grads, "divergent rescale")


@pytest.mark.parametrize("b, t, rows", [(24, 4096, 8), (520, 1024, 260)])
def test_wide_batch_matches_the_same_rows_in_smaller_calls(b, t, rows):
    """Rows are independent, so a batch split into smaller calls must give the same results.

    24 rows of 4096 tokens make 3072 per-64 id-range records: more than the
    work-order kernel stages in shared memory (1536), so it reads them from the
    workspace; calls of 8 rows (1024 records) take the staged path. 520 rows of
    1024 tokens make 4160 work items per call: more than the kernel keeps
    weights for (4096), so it computes each weight twice; calls of 260 rows
    (2080 items) keep them. Each O, dK and dV value comes from one CTA in a
    fixed order whatever the work order, so those agree bit for bit; dQ is
    summed by reduce-adds in arrival order and agrees to the gradient gate.
    """
    from minifield_training_b200 import workloads

    q, k, v, do = _qkvd(21, b, t, t, h=2, hk=1)
    seg = workloads.packed_segments(23, b, t, lo=32, hi=1024)
    mask = (seg != 0).astype(np.int32)
    whole = gpu_attention(BIDIR, q, k, v, do, mask=mask, seg=seg)
    for r0 in range(0, b, rows):
        sl = slice(r0, r0 + rows)
        part = gpu_attention(BIDIR, q[sl], k[sl], v[sl], do[sl], mask=mask[sl], seg=seg[sl])
        for name in ("out", "dk", "dv"):
            np.testing.assert_array_equal(whole[name][sl], part[name], err_msg=f"{name} rows {r0}-{r0 + rows - 1}")
        assert_close(whole["dq"][sl], part["dq"], scaled=True, what=f"dq rows {r0}-{r0 + rows - 1}")


def test_whole_query_tiles_without_live_keys():
    """Whole 128-row query tiles with no valid key still write their rows.

    Such a tile issues no products, and its rows take the empty-row policy:
    zeros for the bidirectional operator (the second tile is all padding,
    segment id 0) and
    the uniform average over all keys for the causal one (batch row 1 masks
    every key). Its O rows go through the same shared staging and TMA store as
    any whole tile, after the tile's Q load has landed in that buffer.
    """
    t = 256
    q, k, v, do = _qkvd(31, 2, t, t)
    seg = np.zeros((2, t), np.int32)
    seg[:, :100] = 1  # segment id 0 from token 100 on: padding queries with no valid key
    mask = (seg != 0).astype(np.int32)
    r = gpu_attention(BIDIR, q, k, v, do, mask=mask, seg=seg)
    out, grads = oracle_attention(q, k, v, oatt.bidirectional_ids(mask, seg), do)
    _check(r, out, grads, "bidirectional, padded second tile")
    assert np.all(r["out"][:, 128:] == 0)

    mask = np.ones((2, t), np.int32)
    mask[1, :] = 0
    r = gpu_attention(CAUSAL, q, k, v, do, mask=mask)
    out, grads = oracle_attention(q, k, v, oatt.causal_ids(mask), do)
    _check(r, out, grads, "causal, row without valid keys")
