"""KV-cached decode kernel (fused cache append + split-K attention) vs the oracle."""

import numpy as np
import pytest

from oracle import decode as odec
from oracle.bf16 import round_bf16, to_bf16_bits
from tests._util import assert_close
from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


def _run_step(q, kc, vc, nk, nv, positions, lengths):
    from minifield_training_b200.device import DeviceArray
    from minifield_training_b200.layers.attention import decode_attention_step

    b, cap, hk, d = kc.shape
    kd = DeviceArray.from_numpy(kc, "bfloat16")
    vd = DeviceArray.from_numpy(vc, "bfloat16")
    out, kd, vd = decode_attention_step(q[:, None], nk[:, None], nv[:, None], kd, vd, positions, lengths)
    return out.float32()[:, 0], kd.numpy(), vd.numpy()


def _check(q, kc, vc, nk, nv, positions, lengths, what):
    out, kd, vd = _run_step(q, kc, vc, nk, nv, positions, lengths)
    ref, rk, rv = odec.decode_attention(
        round_bf16(q).astype(np.float64), round_bf16(kc), round_bf16(vc), lengths, round_bf16(nk), round_bf16(nv),
        positions)
    assert_close(out, ref, what=what)
    np.testing.assert_array_equal(kd.view(np.uint16), to_bf16_bits(rk))
    np.testing.assert_array_equal(vd.view(np.uint16), to_bf16_bits(rv))


def test_config3_layer_full_size():
    from minifield_training_b200 import workloads

    cfg = workloads.CONFIG3
    lens = workloads.decode_lengths(cfg, 0)
    q, kc, vc, nk, nv = workloads.decode_layer_inputs(cfg, 0, 0)
    _check(q, kc, vc, nk, nv, lens - 1, lens, "config3 layer0")


@pytest.mark.parametrize("cap", [64, 300, 1024])
def test_ragged_lengths_and_edge_rows(cap):
    rng = np.random.default_rng(cap)
    b, h, hk, d = 6, 16, 8, 64
    q = rng.standard_normal((b, h, d), dtype=np.float32)
    kc = rng.standard_normal((b, cap, hk, d), dtype=np.float32)
    vc = rng.standard_normal((b, cap, hk, d), dtype=np.float32)
    nk = rng.standard_normal((b, hk, d), dtype=np.float32)
    nv = rng.standard_normal((b, hk, d), dtype=np.float32)
    lens = np.array([1, cap, cap // 2 + 1, 0, 257 % cap + 1, cap + 5], np.int32)  # 0: uniform; > cap: all slots
    pos = np.array([0, cap - 1, cap // 2, 3, 257 % cap, cap + 10], np.int32)  # last one clamps to cap-1
    _check(q, kc, vc, nk, nv, pos, lens, f"ragged cap={cap}")


def test_gqa_groups_one_and_four():
    rng = np.random.default_rng(11)
    for h, hk in ((8, 8), (16, 4)):
        b, cap, d = 3, 500, 64
        q = rng.standard_normal((b, h, d), dtype=np.float32)
        kc = rng.standard_normal((b, cap, hk, d), dtype=np.float32)
        vc = rng.standard_normal((b, cap, hk, d), dtype=np.float32)
        nk = rng.standard_normal((b, hk, d), dtype=np.float32)
        nv = rng.standard_normal((b, hk, d), dtype=np.float32)
        lens = np.array([500, 17, 260], np.int32)
        _check(q, kc, vc, nk, nv, lens - 1, lens, f"h={h} hk={hk}")


def test_repeated_steps_equal_single_shot_attention():
    """Decoding step by step appends exactly what a full-cache attention sees."""
    from minifield_training_b200.device import DeviceArray
    from minifield_training_b200.kernels.attention import b200_cached_attention
    from minifield_training_b200.layers.attention import decode_attention_step

    rng = np.random.default_rng(5)
    b, cap, h, hk, d, steps = 2, 128, 16, 8, 64, 5
    start = np.array([40, 90], np.int32)
    kc = rng.standard_normal((b, cap, hk, d), dtype=np.float32)
    vc = rng.standard_normal((b, cap, hk, d), dtype=np.float32)
    kd = DeviceArray.from_numpy(kc, "bfloat16")
    vd = DeviceArray.from_numpy(vc, "bfloat16")
    ref_k, ref_v = round_bf16(kc), round_bf16(vc)
    for i in range(steps):
        q = rng.standard_normal((b, 1, h, d), dtype=np.float32)
        nk = rng.standard_normal((b, 1, hk, d), dtype=np.float32)
        nv = rng.standard_normal((b, 1, hk, d), dtype=np.float32)
        pos = start + i
        out, kd, vd = decode_attention_step(q, nk, nv, kd, vd, pos, pos + 1)
        ref, ref_k, ref_v = odec.decode_attention(round_bf16(q[:, 0]).astype(np.float64), ref_k, ref_v, pos + 1,
                                                  round_bf16(nk[:, 0]), round_bf16(nv[:, 0]), pos)
        assert_close(out.float32()[:, 0], ref, what=f"step {i}")
        again = b200_cached_attention(q, kd, vd, pos + 1)
        np.testing.assert_array_equal(again.numpy().view(np.uint16), out.numpy().view(np.uint16))
