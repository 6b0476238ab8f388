"""The allocation-free decode entry point against the workspace one.

mfb_decode_attn_noalloc serves callers that cannot call cudaMalloc (a CUDA
graph being captured, an XLA FFI handler limited to the buffers it is given,
a serving loop that allocates nothing after start-up). Its scratch is a fixed
array inside the library, shared by every call on a device, so this test runs
it twice in a row -- with different lengths, so the second call starts from
the first call's leftovers -- and compares each call's output and cache
writes with mfb_decode_attn given a caller workspace. It also checks that a
shape needing more than the fixed maximum is rejected. The file is named to
be collected last and passes alone in a fresh process or after the rest.
"""

import ctypes

import numpy as np
import pytest

from tests._util import assert_close
from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


def _decode(entry, q, kc, vc, nk, nv, pos, lens):
    """Call one decode entry point through the C ABI; return (o, k_cache, v_cache) on the host."""
    from minifield_training_b200 import _lib
    from minifield_training_b200.device import DeviceArray, sync

    b, cap, hk, d = kc.shape
    h = q.shape[1]
    dev = DeviceArray.from_numpy
    qd, kd, vd, nkd, nvd = (dev(x, "bfloat16") for x in (q, kc, vc, nk, nv))
    pd, ld = dev(pos, "int32"), dev(lens, "int32")
    o = DeviceArray((b, h, d), "bfloat16")
    P = ctypes.c_void_p
    args = [P(qd.ptr), P(kd.ptr), P(vd.ptr), P(nkd.ptr), P(nvd.ptr), P(pd.ptr), P(ld.ptr), P(o.ptr), b, cap, h, hk, d,
            ctypes.c_float(d ** -0.5)]
    if entry == "mfb_decode_attn":
        ws = DeviceArray((_lib.lib().mfb_decode_workspace_size(b, cap, h, d),), "uint8")
        args += [P(ws.ptr), ws.nbytes]
    _lib.call(entry, *args, None)
    sync()
    return o.float32(), kd.numpy().view(np.uint16), vd.numpy().view(np.uint16)


def _inputs(seed, b, cap, h=16, hk=8, d=64):
    rng = np.random.default_rng(seed)
    s = np.float32(0.02)
    return (rng.standard_normal((b, h, d), dtype=np.float32) * s,
            rng.standard_normal((b, cap, hk, d), dtype=np.float32) * s,
            rng.standard_normal((b, cap, hk, d), dtype=np.float32) * s,
            rng.standard_normal((b, hk, d), dtype=np.float32) * s,
            rng.standard_normal((b, hk, d), dtype=np.float32) * s)


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row():
    b, cap = 64, 4096  # the benchmark's decode shape fits the fixed scratch
    rng = np.random.default_rng(0)
    for call, seed in enumerate((1, 2)):
        q, kc, vc, nk, nv = _inputs(seed, b, cap)
        lens = rng.integers(1, cap + 1, size=b).astype(np.int32)
        lens[call] = 0  # a uniform-average row on each call
        pos = np.maximum(lens - 1, 0).astype(np.int32)
        ref_o, ref_k, ref_v = _decode("mfb_decode_attn", q, kc, vc, nk, nv, pos, lens)
        got_o, got_k, got_v = _decode("mfb_decode_attn_noalloc", q, kc, vc, nk, nv, pos, lens)
        assert_close(got_o, ref_o, what=f"no-alloc call {call + 1}")
        np.testing.assert_array_equal(got_k, ref_k)
        np.testing.assert_array_equal(got_v, ref_v)


def test_noalloc_rejects_shapes_beyond_the_fixed_scratch():
    from minifield_training_b200 import _lib
    from minifield_training_b200.device import DeviceArray

    b, cap, h = 4096, 1024, 16
    need = _lib.lib().mfb_decode_workspace_size(b, cap, h, 64)
    assert need > 8 << 20
    # Placeholder buffers: the size check rejects the call before any launch.
    dummy = DeviceArray((16,), "uint8")
    ptrs = [ctypes.c_void_p(dummy.ptr)] * 8
    with pytest.raises(ValueError, match="scratch bytes"):
        _lib.call("mfb_decode_attn_noalloc", *ptrs, b, cap, h, 8, 64, ctypes.c_float(0.125), None)


_RESET_CHILD = r"""
import sys
import numpy as np
sys.path.insert(0, {root!r})
from minifield_training_b200 import _lib, device
from tests import test_zz_no_alloc as t
from tests._util import assert_close

device.set_device(0)
b, cap = 8, 512
rng = np.random.default_rng(5)
for round_ in range(2):
    q, kc, vc, nk, nv = t._inputs(10 + round_, b, cap)
    lens = rng.integers(1, cap + 1, size=b).astype(np.int32)
    pos = (lens - 1).astype(np.int32)
    ref = t._decode("mfb_decode_attn", q, kc, vc, nk, nv, pos, lens)
    got = t._decode("mfb_decode_attn_noalloc", q, kc, vc, nk, nv, pos, lens)
    assert_close(got[0], ref[0], what=f"no-alloc context {{round_}}")
    np.testing.assert_array_equal(got[1], ref[1])
    np.testing.assert_array_equal(got[2], ref[2])
    if round_ == 0:
        _lib.call("mfb_device_reset")  # every device buffer above is already freed
print("ok")
"""


def test_noalloc_after_a_device_reset_uses_the_new_context():
    """A reset destroys the context the scratch address was looked up in; the next call must
    look it up again in the new context. Runs in a child process, so the reset touches no
    buffer of the other tests."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _RESET_CHILD.format(root=root)], cwd=root, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-2000:]
