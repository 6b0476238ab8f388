"""GPU test prerequisites: the built library and an sm_100 device, else skip."""

import pytest


def require_gpu():
    from minifield_training_b200 import _lib, build, device

    try:
        _lib.lib()
    except ImportError:
        build.build()
        _lib._lib = None
        _lib.lib()
    try:
        n = device.device_count()
    except RuntimeError as exc:
        pytest.skip(f"no CUDA device: {exc}")
    if n < 1:
        pytest.skip("no CUDA device")
    device.set_device(0)
    device.require_b200(0)
