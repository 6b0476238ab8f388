"""ctypes binding of libmfb200.so (the C ABI declared in include/mfb200.h).

The library is loaded from this package directory; if it is missing the import
fails loudly (there is no CPU fallback). Nonzero statuses become exceptions:
MFB_ERR_INVALID -> ValueError (the reference raises ValueError for shape and
argument errors, e.g. src/minifield_training/kernels/attention.py:276-279),
everything else -> RuntimeError.
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmfb200.so")

OK, ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_DEVICE, ERR_COMM = range(7)

QUANT_KINDS = {
    "int8-channel-absmax-v1": 0,
    "int4-g128-absmax-v1": 1,
    "ternary-g128-absmax-f16-v1": 2,
    "nf4-g128-absmax-f16-v1": 3,
}
MASK_CAUSAL, MASK_PREFIX, MASK_PACKED, MASK_BIDIR, MASK_CACHED = range(5)
EMPTY_UNIFORM, EMPTY_ZERO = 0, 1
MAJOR_K, MAJOR_MN = 0, 1
DTYPE_BF16, DTYPE_F32 = 0, 1
GEMM_PDL = 1

P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float
SZ = ctypes.c_size_t
LL = ctypes.c_longlong
IP = ctypes.POINTER(ctypes.c_int)

# name -> (restype, argtypes); mirrors include/mfb200.h one to one.
SIGNATURES = {
    "mfb_last_error": (ctypes.c_char_p, []),
    "mfb_version": (I, []),
    "mfb_device_count": (I, [IP]),
    "mfb_set_device": (I, [I]),
    "mfb_device_sm_version": (I, [I, IP, IP]),
    "mfb_malloc": (I, [ctypes.POINTER(P), SZ]),
    "mfb_free": (I, [P]),
    "mfb_host_alloc": (I, [ctypes.POINTER(P), SZ]),
    "mfb_host_free": (I, [P]),
    "mfb_memcpy_h2d": (I, [P, P, SZ, P]),
    "mfb_memcpy_d2h": (I, [P, P, SZ, P]),
    "mfb_memcpy_d2d": (I, [P, P, SZ, P]),
    "mfb_memcpy2d_d2d": (I, [P, SZ, P, SZ, SZ, SZ, P]),
    "mfb_memset": (I, [P, I, SZ, P]),
    "mfb_stream_create": (I, [ctypes.POINTER(P)]),
    "mfb_stream_destroy": (I, [P]),
    "mfb_stream_sync": (I, [P]),
    "mfb_device_sync": (I, []),
    "mfb_device_reset": (I, []),
    "mfb_event_create": (I, [ctypes.POINTER(P)]),
    "mfb_event_destroy": (I, [P]),
    "mfb_event_record": (I, [P, P]),
    "mfb_stream_wait_event": (I, [P, P]),
    "mfb_event_elapsed_ms": (I, [P, P, ctypes.POINTER(F)]),
    "mfb_fakequant": (I, [P, I, I, I, P, P, P, P, P, P]),
    "mfb_attn_ids": (I, [I, P, P, P, P, P, I, I, I, I, IP, IP, IP, P]),
    "mfb_attn_workspace_size": (SZ, [I, I, I, I, I, I]),
    "mfb_attn_fwd": (I, [P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, I, F, P, SZ, P]),
    "mfb_attn_bwd": (I, [P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, I, F, P, SZ, P]),
    "mfb_attn_status": (I, [IP]),
    "mfb_decode_workspace_size": (SZ, [I, I, I, I]),
    "mfb_decode_attn": (I, [P, P, P, P, P, P, P, P, I, I, I, I, I, F, P, SZ, P]),
    "mfb_decode_attn_noalloc": (I, [P, P, P, P, P, P, P, P, I, I, I, I, I, F, P]),
    "mfb_gemm_bf16": (I, [P, I, I, P, I, I, P, I, I, I, I, I, F, P, P]),
    "mfb_gemm_workspace_size": (SZ, [I, I, I]),
    "mfb_gemm_bf16_ws": (I, [P, I, I, P, I, I, P, I, I, I, I, I, F, P, I, P, SZ, P]),
    "mfb_gemm_status": (I, [IP]),
    "mfb_gemm_swiglu_fwd": (I, [P, I, I, P, I, P, P, I, I, I, P]),
    "mfb_gemm_swiglu_bwd": (I, [P, I, I, P, I, I, P, P, I, I, I, P]),
    "mfb_graph_begin": (I, [P]),
    "mfb_graph_end": (I, [P, ctypes.POINTER(ctypes.c_void_p)]),
    "mfb_graph_launch": (I, [P, P]),
    "mfb_graph_destroy": (I, [P]),
    "mfb_adamw_workspace_size": (SZ, []),
    "mfb_adamw_commit": (I, [P, P, P, P, LL, LL, LL, P, P, P, P, F, F, F, F, F, F, P, P, SZ, P]),
    "mfb_adamw_shard_pass": (I, [I, P, P, P, P, LL, LL, LL, LL, LL, P, P, P, P, F, F, F, F, F, F, P, P, P, SZ, P]),
    "mfb_step_normalize": (I, [P, P, P, P, P, P, P]),
    "mfb_norm_workspace_size": (SZ, [I, I]),
    "mfb_rmsnorm_fwd": (I, [P, P, P, P, P, P, P, I, I, F, P]),
    "mfb_rmsnorm_bwd": (I, [P, P, P, P, P, P, P, P, I, I, I, P, SZ, P]),
    "mfb_qknorm_rope_fwd": (I, [P, I, P, P, P, P, P, P, P, P, P, I, I, I, F, P]),
    "mfb_qknorm_rope_bwd": (I, [P, I, P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, P, SZ, P]),
    "mfb_embed_gather": (I, [P, P, P, LL, I, I, P]),
    "mfb_conv_fwd": (I, [P, P, P, P, LL, I, I, P]),
    "mfb_encoder_workspace_size": (SZ, [I, I]),
    "mfb_conv_bwd": (I, [P, P, P, P, P, P, I, LL, I, I, P, SZ, P]),
    "mfb_head_loss": (I, [P, P, P, P, P, P, P, I, I, I, P, SZ, P]),
    "mfb_swiglu_fwd": (I, [P, P, I, I, P]),
    "mfb_swiglu_bwd": (I, [P, P, P, I, I, P]),
    "mfb_cast_f32_bf16": (I, [P, P, ctypes.c_longlong, P]),
    "mfb_cast_bf16_f32": (I, [P, P, LL, P]),
    "mfb_add_bf16": (I, [P, P, P, LL, P]),
    "mfb_comm_load": (I, [ctypes.c_char_p, IP]),
    "mfb_comm_unique_id_bytes": (SZ, []),
    "mfb_comm_unique_id": (I, [P, SZ]),
    "mfb_comm_init": (I, [P, SZ, I, I, ctypes.c_double, ctypes.POINTER(P)]),
    "mfb_comm_rank": (I, [P, IP, IP]),
    "mfb_comm_allreduce": (I, [P, P, P, SZ, I, I, P]),
    "mfb_comm_reduce_scatter": (I, [P, P, P, SZ, I, I, P]),
    "mfb_comm_allgather": (I, [P, P, P, SZ, I, P]),
    "mfb_comm_reduce": (I, [P, P, P, SZ, I, I, I, P]),
    "mfb_comm_broadcast": (I, [P, P, P, SZ, I, I, P]),
    "mfb_comm_wait": (I, [P, P, ctypes.c_double]),
    "mfb_comm_abort": (I, [P]),
    "mfb_comm_destroy": (I, [P]),
    "mfb_conv_step": (I, [P, P, P, P, I, I, P]),
    "mfb_conv_causal": (I, [P, P, P, P, P, I, I, I, P]),
}

_lib = None


def lib():
    """Load (once) and return the configured ctypes library."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is not built; run `python -m minifield_training_b200.build` "
                "(the B200 path has no CPU fallback)"
            )
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().mfb_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str = "") -> None:
    if status == OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if status == ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(f"[mfb status {status}] {msg}")


def call(name: str, *args):
    """Call ``name`` and raise on a nonzero status."""
    check(getattr(lib(), name)(*args), name)
