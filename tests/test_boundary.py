"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU)."""

import ctypes
import os

import pytest

from tests._util import header_functions
from minifield_training_b200 import _lib


@pytest.fixture(scope="module")
def built_lib():
    if not os.path.exists(_lib.LIB_PATH):
        from minifield_training_b200 import build

        try:
            build.build()
        except RuntimeError as exc:  # no nvcc on this host
            pytest.skip(f"library not built: {exc}")
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_declares_the_hot_path():
    names = header_functions()
    for required in ("mfb_attn_fwd", "mfb_attn_bwd", "mfb_decode_attn", "mfb_fakequant", "mfb_gemm_bf16"):
        assert required in names


def test_library_exports_every_header_symbol(built_lib):
    missing = [n for n in header_functions() if not hasattr(built_lib, n)]
    assert not missing, f"not exported: {missing}"


def test_ctypes_signatures_cover_the_header():
    assert sorted(_lib.SIGNATURES) == header_functions()


def test_python_layer_loads_library(built_lib):
    lib = _lib.lib()
    assert lib.mfb_version() == 1
    assert lib.mfb_attn_workspace_size(8, 2048, 2048, 16, 8, 64) > 0
    assert lib.mfb_decode_workspace_size(64, 4096, 16, 64) > 0


def test_invalid_arguments_raise_before_launch(built_lib):
    lib = _lib.lib()
    # K not divisible by 128 for a group-128 kind: ValueError, no device touched.
    with pytest.raises(ValueError, match="K divisible by 128"):
        _lib.check(lib.mfb_fakequant(None, 3, 2, 100, None, None, None, None, None, None), "fakequant")
    with pytest.raises(ValueError, match="head_dim"):
        _lib.check(
            lib.mfb_attn_fwd(None, None, None, None, None, None, None, 1, 4, 4, 2, 1, 128, 1, 0, 0,
                             ctypes.c_float(1.0), None, 0, None),
            "attn",
        )
    with pytest.raises(ValueError, match="divisible"):
        _lib.check(
            lib.mfb_decode_attn(None, None, None, None, None, None, None, None, 2, 16, 3, 2, 64,
                                ctypes.c_float(1.0), None, 0, None),
            "decode",
        )
    a = ctypes.c_void_p(16)  # never dereferenced: the checks fail first
    with pytest.raises(ValueError, match="created stream"):
        _lib.check(lib.mfb_gemm_bf16_ws(a, 0, 64, a, 0, 64, a, 64, 0, 64, 64, 64, ctypes.c_float(1.0), None,
                                        _lib.GEMM_PDL, None, 0, None), "gemm")
    with pytest.raises(ValueError, match="unknown GEMM flags"):
        _lib.check(lib.mfb_gemm_bf16_ws(a, 0, 64, a, 0, 64, a, 64, 0, 64, 64, 64, ctypes.c_float(1.0), None,
                                        6, None, 0, None), "gemm")
    with pytest.raises(ValueError, match="alias"):
        _lib.check(lib.mfb_conv_causal(a, a, a, a, a, 2, 4, 8, None), "conv")


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libmfb200.so")
    with pytest.raises(ImportError, match="no CPU fallback"):
        _lib.lib()


def test_unknown_backend_names_raise_like_the_reference():
    from minifield_training_b200.kernels import attention

    with pytest.raises(ValueError, match="Unsupported causal attention backend: dense"):
        attention.causal_attention(None, None, None, None, backend="dense")
    with pytest.raises(ValueError, match="Unsupported packed attention backend"):
        attention.packed_causal_attention(None, None, None, None, None, backend="splash")
    with pytest.raises(ValueError, match="Unsupported cached attention backend"):
        attention.cached_attention(None, None, None, None, backend="cudnn")


def test_attention_block_functions_reject_unknown_backends_before_any_launch():
    from minifield_training_b200.layers import attention as la

    with pytest.raises(ValueError, match="Unsupported causal attention backend: dense"):
        la.attention_block(None, None, None, None, head_dim=64, rope_theta=1e6, eps=1e-5, backend="dense")
    with pytest.raises(ValueError, match="Unsupported causal attention backend: cudnn"):
        la.attention_block_prefill(None, None, None, None, capacity=8, head_dim=64, rope_theta=1e6, eps=1e-5,
                                   backend="cudnn")
    with pytest.raises(ValueError, match="Unsupported cached attention backend: dense"):
        la.attention_block_step(None, None, None, None, None, 0, 1, head_dim=64, rope_theta=1e6, eps=1e-5,
                                backend="dense")
