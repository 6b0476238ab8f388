"""Pin the CPU oracle to the reference test-suite's known answers (no GPU).

The fixtures in tests/golden/reference_kats.npz are transcribed from the
reference's tests (see tests/golden/make_golden.py for file:line sources).
"""

import numpy as np
import pytest

from oracle import attention as oatt
from oracle import decode as odec
from oracle import linear as olin
from oracle import quant as oq
from oracle.bf16 import round_bf16
from minifield_training_b200 import workloads


# --- quantization (tests/kernels/test_quantization.py) -----------------------


@pytest.mark.parametrize(
    "name,kind",
    [
        ("ternary_halfaway", oq.KIND_TERNARY_G128),
        ("nf4_codebook", oq.KIND_NF4_G128),
        ("ternary_nextafter", oq.KIND_TERNARY_G128),
        ("nf4_midpoints", oq.KIND_NF4_G128),
        ("underflow", oq.KIND_TERNARY_G128),
        ("underflow", oq.KIND_NF4_G128),
    ],
)
def test_reference_quantizer_kats(golden, name, kind):
    codes, scales, ste, eff = oq.fake_quant(golden[name + "_in"], kind)
    np.testing.assert_array_equal(eff, golden[name + "_out"])
    # Identity STE of the reference kinds: gradient of sum(effective) is ones.
    np.testing.assert_array_equal(ste, np.ones_like(ste))


def test_nf4_transitions_are_first_values_above_midpoints():
    levels = oq.NF4_LEVELS.astype(np.float64)
    for i, t in enumerate(oq.NF4_TRANSITIONS):
        mid = (levels[i] + levels[i + 1]) / 2
        assert float(t) > mid
        assert float(np.nextafter(t, np.float32(-np.inf))) <= mid


def test_quantizer_shape_errors():
    with pytest.raises(ValueError):
        oq.fake_quant(np.zeros((2, 100), np.float32), oq.KIND_NF4_G128)
    with pytest.raises(ValueError):
        oq.fake_quant(np.zeros((2, 128), np.float64), oq.KIND_INT8_CHANNEL)
    with pytest.raises(ValueError):
        oq.fake_quant(np.zeros((0, 128), np.float32), oq.KIND_INT4_G128)
    oq.fake_quant(np.zeros((3, 100), np.float32), oq.KIND_INT8_CHANNEL)  # per-channel: any K


@pytest.mark.parametrize("kind", [oq.KIND_INT8_CHANNEL, oq.KIND_INT4_G128])
def test_symmetric_int_quantizers_definition(kind):
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((33, 256)) * 0.02).astype(np.float32)
    w[3] = 0.0  # zero-scale row / groups
    codes, scales, ste, eff = oq.fake_quant(w, kind)
    qmax = 127 if kind == oq.KIND_INT8_CHANNEL else 7
    assert codes.min() >= -qmax and codes.max() <= qmax
    g = 256 if kind == oq.KIND_INT8_CHANNEL else 128
    s = np.repeat(scales, g, axis=1)
    np.testing.assert_array_equal(eff, (codes.astype(np.float32) * s).astype(np.float32))
    assert np.all(codes[3] == 0) and np.all(eff[3] == 0) and np.all(ste[3] == 1)
    # Absmax scaling never clamps: the STE mask is all ones.
    assert ste.all()
    # Every group's absmax element maps to +-qmax.
    grouped = np.abs(w.reshape(33, -1, g))
    idx = grouped.argmax(-1)
    cg = codes.reshape(33, -1, g)
    for r in range(33):
        if r == 3:
            continue
        for j in range(idx.shape[1]):
            assert abs(int(cg[r, j, idx[r, j]])) == qmax


def test_ste_mask_zero_outside_clamp():
    # A hand-set scale smaller than absmax/qmax is not reachable through absmax
    # scaling; emulate the definition directly on a ratio to check the mask rule.
    ratio = np.array([126.4, 127.49, 127.5, -128.2, 300.0], np.float32)
    rounded = np.rint(ratio)
    codes = np.clip(rounded, -127, 127)
    np.testing.assert_array_equal(rounded == codes, [True, True, False, False, False])


# --- linear (tests/kernels/test_linear.py) -----------------------------------


def test_linear_matrix_calculus(golden):
    x, w, probe = golden["linear_x"], golden["linear_w"], golden["linear_probe"]
    # The KAT's weights are exact in bf16, so the cast-before-dot is invisible here.
    np.testing.assert_array_equal(olin.full_linear(x, w, np.float32), golden["linear_out"])
    np.testing.assert_array_equal(probe @ round_bf16(w), golden["linear_dx"])
    np.testing.assert_array_equal(probe.reshape(-1, 2).T @ x.reshape(-1, 2), golden["linear_dw"])


def test_linear_casts_master_before_dot(golden):
    x, w = golden["linear_cast_x"], golden["linear_cast_w"]
    out = olin.full_linear(round_bf16(x), w, np.float32)
    np.testing.assert_array_equal(out, golden["linear_cast_out"])
    dy = np.ones((1, 1), np.float32)
    np.testing.assert_array_equal(dy @ round_bf16(w), golden["linear_cast_dx"])
    np.testing.assert_array_equal(dy.T @ round_bf16(x), golden["linear_cast_dw"])


# --- attention (tests/kernels/test_attention.py, test_bidirectional.py) ------


def test_dense_causal_matches_reference_fp64_oracle(golden):
    out = oatt.dense_causal_attention(golden["causal_q"], golden["causal_k"], golden["causal_v"], golden["causal_mask"])
    np.testing.assert_allclose(out, golden["causal_out"], rtol=2e-6, atol=2e-6)


def test_dense_prefix_matches_reference_fp64_oracle(golden):
    g = golden
    out = oatt.dense_prefix_causal_attention(
        g["prefix_q"], g["prefix_pk"], g["prefix_pv"], g["prefix_k"], g["prefix_v"], g["prefix_pmask"], g["prefix_smask"]
    )
    np.testing.assert_allclose(out, g["prefix_out"], rtol=2e-6, atol=2e-6)


def test_dense_packed_matches_reference_fp64_oracle(golden):
    g = golden
    out = oatt.dense_packed_causal_attention(g["packed_q"], g["packed_k"], g["packed_v"], g["packed_mask"], g["packed_seg"])
    np.testing.assert_allclose(out, g["packed_out"], rtol=2e-6, atol=2e-6)


def test_dense_cached_matches_reference_fp64_oracle(golden):
    g = golden
    out = oatt.dense_cached_attention(g["cached_q"], g["cached_k"], g["cached_v"], g["cached_len"])
    np.testing.assert_allclose(out, g["cached_out"], rtol=2e-6, atol=2e-6)
    o, _, _ = odec.decode_attention(g["cached_q"][:, 0], g["cached_k"], g["cached_v"], np.array([4, 4]))
    np.testing.assert_allclose(o, g["cached_out"][:, 0], rtol=2e-6, atol=2e-6)


def test_bidirectional_uniform_average_and_gradient(golden):
    g = golden
    out, (dq, dk, dv) = oatt.bidirectional_attention(
        g["bidir_uniform_q"], g["bidir_uniform_k"], g["bidir_uniform_v"], g["bidir_uniform_mask"],
        d_out=np.ones((1, 3, 2, 2)),
    )
    np.testing.assert_allclose(out, g["bidir_uniform_out"])
    np.testing.assert_allclose(dv, g["bidir_uniform_dv"])
    empty = oatt.bidirectional_attention(
        g["bidir_uniform_q"], g["bidir_uniform_k"], g["bidir_uniform_v"], np.zeros_like(g["bidir_uniform_mask"])
    )
    np.testing.assert_array_equal(empty, np.zeros((1, 3, 2, 2)))


def test_bidirectional_packed_segment_average_and_gradient(golden):
    g = golden
    seg = g["bidir_packed_seg"]
    out, (_, _, dv) = oatt.bidirectional_attention(
        g["bidir_packed_q"], g["bidir_packed_k"], g["bidir_packed_v"], (seg != 0).astype(np.int32), seg,
        d_out=np.ones((1, 6, 2, 2)),
    )
    np.testing.assert_allclose(out, g["bidir_packed_out"])
    np.testing.assert_allclose(dv, g["bidir_packed_dv"], rtol=1e-6)


# --- id encoding == the reference's own mask formulas (bit-exact) ------------


def _random_masks(seed, b=3, t=37):
    rng = np.random.default_rng(seed)
    mask = (rng.random((b, t)) > 0.2).astype(np.int32)
    seg = np.sort(rng.integers(0, 5, size=(b, t)), axis=1).astype(np.int32)
    seg[0, -5:] = 0
    return mask, seg


@pytest.mark.parametrize("seed", range(4))
def test_id_encoding_matches_reference_masks(seed):
    mask, seg = _random_masks(seed)
    qid, kid, causal, off, _ = oatt.causal_ids(mask)
    np.testing.assert_array_equal(oatt.valid_from_ids(qid, kid, causal, off), oatt.reference_causal_valid(mask))
    pm = mask[:, :7]
    qid, kid, causal, off, _ = oatt.prefix_ids(pm, mask)
    np.testing.assert_array_equal(oatt.valid_from_ids(qid, kid, causal, off), oatt.reference_prefix_valid(pm, mask))
    ref_valid, active = oatt.reference_packed_valid(mask, seg)
    qid, kid, causal, off, _ = oatt.packed_ids(mask, seg)
    mine = oatt.valid_from_ids(qid, kid, causal, off)
    # Identical on active query rows; inactive rows self-attend in the reference
    # and are zeroed afterwards, so they are empty (zero output) here.
    np.testing.assert_array_equal(mine[active], ref_valid[active])
    assert not mine[~active].any()
    for segs in (None, seg):
        ref_valid, present = oatt.reference_bidirectional_valid(mask, segs)
        qid, kid, causal, off, _ = oatt.bidirectional_ids(mask, segs)
        mine = oatt.valid_from_ids(qid, kid, causal, off)
        np.testing.assert_array_equal(mine[present], ref_valid[present])
        assert not mine[~present].any()
    lengths = np.array([0, 5, 37])
    qid, kid, causal, off, _ = oatt.cached_ids(lengths, 3, 37)
    np.testing.assert_array_equal(oatt.valid_from_ids(qid, kid, causal, off), oatt.reference_cached_valid(lengths, 3, 37))


# --- analytic backward vs finite differences ---------------------------------


@pytest.mark.parametrize("mode", ["causal", "packed", "bidir", "bidir_seg", "causal_empty_row"])
def test_attention_backward_matches_finite_differences(mode):
    rng = np.random.default_rng(11)
    b, t, h, hk, d = 2, 5, 4, 2, 3
    q = rng.standard_normal((b, t, h, d))
    k = rng.standard_normal((b, t, hk, d))
    v = rng.standard_normal((b, t, hk, d))
    dout = rng.standard_normal((b, t, h, d))
    mask = np.array([[1, 1, 1, 0, 1], [1, 1, 0, 0, 0]], np.int32)
    seg = np.array([[1, 1, 2, 2, 0], [1, 2, 2, 0, 0]], np.int32)
    if mode == "causal":
        ids = oatt.causal_ids(mask)
    elif mode == "causal_empty_row":
        ids = oatt.causal_ids(np.array([[0, 1, 1, 0, 1], [0, 0, 1, 1, 1]], np.int32))
    elif mode == "packed":
        ids = oatt.packed_ids(mask, seg)
    elif mode == "bidir":
        ids = oatt.bidirectional_ids(mask)
    else:
        ids = oatt.bidirectional_ids(mask, seg)
    valid = oatt.valid_from_ids(*ids[:4])
    policy = ids[4]

    def loss(qq, kk, vv):
        return float((oatt.attention_forward(qq, kk, vv, valid, policy) * dout).sum())

    dq, dk, dv = oatt.attention_backward(q, k, v, valid, policy, dout)
    eps = 1e-6
    for arr, grad in ((q, dq), (k, dk), (v, dv)):
        num = np.zeros_like(arr)
        it = np.nditer(arr, flags=["multi_index"])
        for _ in it:
            i = it.multi_index
            old = arr[i]
            arr[i] = old + eps
            lp = loss(q, k, v)
            arr[i] = old - eps
            lm = loss(q, k, v)
            arr[i] = old
            num[i] = (lp - lm) / (2 * eps)
        np.testing.assert_allclose(grad, num, rtol=1e-5, atol=1e-6)


def test_empty_causal_row_is_uniform_over_all_keys():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((1, 4, 2, 3))
    k = rng.standard_normal((1, 4, 1, 3))
    v = rng.standard_normal((1, 4, 1, 3))
    out = oatt.dense_causal_attention(q, k, v, np.array([[0, 1, 1, 1]], np.int32))
    np.testing.assert_allclose(out[0, 0, 0], v[0, :, 0].mean(0))


# --- QAT FFN backward vs finite differences ----------------------------------


def test_swiglu_qat_backward_matches_finite_differences():
    rng = np.random.default_rng(5)
    m, c, f = 3, 4, 128  # int8 per-channel admits any K; the down GEMM has K=f
    x = rng.standard_normal((m, c)).astype(np.float32)
    w_gu = (rng.standard_normal((2 * f, c)) * 0.3).astype(np.float32)
    w_d = (rng.standard_normal((c, f)) * 0.3).astype(np.float32)
    dy = rng.standard_normal((m, c)).astype(np.float32)
    kind = oq.KIND_INT8_CHANNEL
    dx, dwgu, dwd = olin.swiglu_qat_backward(x, w_gu, w_d, kind, dy, bf16_casts=False)
    eff_gu, _, eff_d, _ = olin.qat_weights(w_gu, w_d, kind)
    xb = round_bf16(x).astype(np.float64)

    def loss_gu(weff_gu):
        gu = xb @ weff_gu.T
        h = olin.silu(gu[:, :f]) * gu[:, f:]
        return float(((h @ eff_d.astype(np.float64).T) * round_bf16(dy)).sum())

    base = eff_gu.astype(np.float64)
    eps = 1e-6
    for (i, j) in [(0, 0), (5, 2), (f + 3, 1), (2 * f - 1, 3)]:
        p = base.copy()
        p[i, j] += eps
        mneg = base.copy()
        mneg[i, j] -= eps
        # h is not re-rounded here, so compare loosely against the analytic value.
        num = (loss_gu(p) - loss_gu(mneg)) / (2 * eps)
        assert abs(num - dwgu[i, j]) < 5e-2 * max(1.0, abs(num))
    assert dx.shape == x.shape and dwd.shape == w_d.shape


def test_config2_segments_match_stated_square_sum():
    seg = workloads.packed_segments(0, 8, 2048)
    assert workloads.segment_square_sum(seg) == 11_171_716
    assert seg.dtype == np.int32 and seg.shape == (8, 2048)


@pytest.mark.parametrize("kind", ["int8-channel-absmax-v1", "int4-g128-absmax-v1"])
def test_swiglu_step_equals_forward_and_backward(kind):
    """The one-pass chain (CPU baseline, full-size parity) returns exactly the values of the
    separate forward and backward restatements."""
    from oracle import linear as ol

    rng = np.random.default_rng(0)
    x = rng.standard_normal((64, 256)).astype(np.float32)
    wgu = (rng.standard_normal((256, 256)) * 0.02).astype(np.float32)
    wd = (rng.standard_normal((256, 128)) * 0.02).astype(np.float32)
    dy = rng.standard_normal((64, 256)).astype(np.float32)
    fwd = ol.swiglu_qat_forward(x, wgu, wd, kind)
    bwd = ol.swiglu_qat_backward(x, wgu, wd, kind, dy)
    for a, b in zip(fwd + bwd, ol.swiglu_qat_step(x, wgu, wd, kind, dy)):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("kind", ["int8-channel-absmax-v1", "int4-g128-absmax-v1"])
def test_swiglu_weight_grad_columns_equal_the_full_backward(kind):
    from oracle import linear as ol

    rng = np.random.default_rng(1)
    x = rng.standard_normal((48, 256)).astype(np.float32)
    wgu = (rng.standard_normal((2 * 128, 256)) * 0.02).astype(np.float32)
    wd = (rng.standard_normal((256, 128)) * 0.02).astype(np.float32)
    dy = rng.standard_normal((48, 256)).astype(np.float32)
    _, dwgu, dwd = ol.swiglu_qat_backward(x, wgu, wd, kind, dy)
    cols = np.array([0, 7, 64, 127])
    cd, cg, cu = ol.swiglu_qat_weight_grad_columns(x, wgu, wd, kind, dy, cols)
    np.testing.assert_allclose(cd, dwd[:, cols], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(cg, dwgu[cols], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(cu, dwgu[128 + cols], rtol=1e-12, atol=1e-12)
