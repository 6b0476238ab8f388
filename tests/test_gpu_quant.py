"""Fake-quant kernel vs the oracle: codes, scales, STE masks and decoded values bit-exact."""

import numpy as np
import pytest

from oracle import quant as oq
from oracle.bf16 import to_bf16_bits
from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


def _run(w, kind):
    from minifield_training_b200.kernels import quantization as q

    r = q.fake_quant(w, kind)
    return r.codes.numpy(), r.scales.numpy(), r.ste.numpy(), r.effective.numpy(), r.effective_bf16.numpy()


def _check_exact(w, kind):
    codes, scales, ste, eff, eff16 = _run(w, kind)
    rc, rs, rste, reff = oq.fake_quant(w, kind)
    np.testing.assert_array_equal(codes, rc)
    np.testing.assert_array_equal(scales.view(np.uint32), rs.view(np.uint32))
    np.testing.assert_array_equal(ste, rste)
    np.testing.assert_array_equal(eff.view(np.uint32), reff.view(np.uint32))
    np.testing.assert_array_equal(eff16.view(np.uint16), to_bf16_bits(reff))


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
def test_reference_kats_on_gpu(golden, name, kind):
    _, _, ste, eff, _ = _run(golden[name + "_in"], kind)
    np.testing.assert_array_equal(eff, golden[name + "_out"])
    np.testing.assert_array_equal(ste, np.ones_like(ste))


@pytest.mark.parametrize("kind", oq.KINDS)
@pytest.mark.parametrize("shape", [(7, 128), (33, 512), (64, 1024)])
def test_random_matrices_bit_exact(kind, shape):
    rng = np.random.default_rng(hash((kind, shape)) % 2**32)
    w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    w[0] = 0.0  # zero group / row
    w[1, :5] = [1e-9, -3e-8, 7e-6, 65504.0 / 4, -1e-3]  # fp16 underflow / large values
    _check_exact(w, kind)


def test_int8_channel_any_width_bit_exact():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((5, 777)) * 0.5).astype(np.float32)
    _check_exact(w, oq.KIND_INT8_CHANNEL)


@pytest.mark.parametrize("kind", [oq.KIND_INT8_CHANNEL, oq.KIND_INT4_G128])
def test_config4_weights_bit_exact(kind):
    from minifield_training_b200 import workloads

    _, w_gu, w_d, _ = workloads.qat_inputs(workloads.CONFIG4, seed=0, tokens=1)
    _check_exact(w_gu, kind)
    _check_exact(w_d, kind)


def test_published_ffn_width_4608_bit_exact():
    rng = np.random.default_rng(4608)
    w = (rng.standard_normal((1024, 4608)) * 0.02).astype(np.float32)
    _check_exact(w, oq.KIND_INT4_G128)
    _check_exact(w, oq.KIND_INT8_CHANNEL)


def test_shape_errors_are_value_errors():
    from minifield_training_b200.kernels import quantization as q

    with pytest.raises(ValueError):
        q.fake_quant(np.zeros((2, 100), np.float32), oq.KIND_NF4_G128)
    with pytest.raises(ValueError):
        q.fake_quant(np.zeros((2, 128), np.float64), oq.KIND_INT8_CHANNEL)
    with pytest.raises(ValueError):
        q.Group128Quantizer("int8-channel-absmax-v1")
