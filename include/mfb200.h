/*
 * libmfb200 -- C ABI of the B200 (sm_100a) hot path of minifield-training.
 *
 * Every entry point takes plain device pointers and sizes owned by the
 * caller, a CUDA stream (as void*; NULL = legacy default stream) and returns
 * an int status (MFB_OK = 0). On failure mfb_last_error() returns a message
 * for the calling thread. Shape and argument checks run on the host before
 * any launch and mirror the reference's ValueError checks. Device-side work is
 * asynchronous on the given stream. No entry point allocates device memory
 * except mfb_malloc / mfb_host_alloc; scratch comes from the caller through
 * (workspace, workspace_bytes) sized by the matching *_workspace_size().
 *
 * Element types: bf16 tensors are passed as uint16_t payloads (IEEE bfloat16);
 * masks / segment ids / lengths are int32.
 *
 * Layouts follow the reference's array contracts: attention operands are
 * "bthd" -- q [B,T,H,D], k/v [B,S,Hk,D] -- and query head h reads KV head
 * h / (H/Hk) (src/minifield_training/kernels/attention.py:19-22).
 */
#ifndef MFB200_H_
#define MFB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum mfb_status_code {
  MFB_OK = 0,
  MFB_ERR_INVALID = 1,     /* bad shape / argument (reference: ValueError) */
  MFB_ERR_CUDA = 2,        /* CUDA runtime error */
  MFB_ERR_UNSUPPORTED = 3, /* valid but not implemented on this build / device */
  MFB_ERR_WORKSPACE = 4,   /* workspace pointer NULL or too small */
  MFB_ERR_DEVICE = 5       /* a device-side status word reported an error */
};

/* ---- runtime helpers (for hosts that have no device allocator of their own) */
const char* mfb_last_error(void);
int mfb_version(void);
int mfb_device_count(int* count);
int mfb_set_device(int device);
int mfb_device_sm_version(int device, int* major, int* minor);
int mfb_malloc(void** ptr, size_t bytes);
int mfb_free(void* ptr);
int mfb_host_alloc(void** ptr, size_t bytes); /* pinned host memory */
int mfb_host_free(void* ptr);
int mfb_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
int mfb_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
int mfb_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
int mfb_memset(void* dst, int value, size_t bytes, void* stream);
int mfb_stream_create(void** stream);
int mfb_stream_destroy(void* stream);
int mfb_stream_sync(void* stream);
int mfb_device_sync(void);
int mfb_event_create(void** event);
int mfb_event_destroy(void* event);
int mfb_event_record(void* event, void* stream);
int mfb_event_elapsed_ms(void* start, void* end, float* ms);

/* ---- fake quantization ----------------------------------------------------
 * Replaces Quantizer.effective (src/minifield_training/kernels/quantization.py:11-22,
 * Group128Quantizer :107-134) and adds the benchmark's symmetric int8 per-channel
 * and int4 group-128 kinds. w is the FP32 master [rows, cols] (row = output
 * channel). Outputs (each may be NULL): codes int8 [rows, cols] (ternary -1/0/1,
 * NF4 level index 0..15, int8/int4 signed codes), scales f32 [rows, groups]
 * (groups = 1 for int8 per-channel, cols/128 otherwise; the FP16-stored scale
 * widened to FP32 for the reference kinds), ste uint8 [rows, cols] (1 where the
 * straight-through gradient passes), eff_f32 / eff_bf16 [rows, cols] (the decoded
 * weight; bf16 is the cast full_linear applies, kernels/linear.py:11).
 */
enum mfb_quant_kind {
  MFB_QUANT_INT8_CHANNEL = 0, /* "int8-channel-absmax-v1" */
  MFB_QUANT_INT4_G128 = 1,    /* "int4-g128-absmax-v1" */
  MFB_QUANT_TERNARY_G128 = 2, /* "ternary-g128-absmax-f16-v1" */
  MFB_QUANT_NF4_G128 = 3      /* "nf4-g128-absmax-f16-v1" */
};
int mfb_fakequant(const float* w, int kind, int rows, int cols, int8_t* codes, float* scales, uint8_t* ste,
                  float* eff_f32, uint16_t* eff_bf16, void* stream);

/* ---- attention --------------------------------------------------------------
 * Mask encoding: query row t of batch b carries qid[b,t], key s carries
 * kid[b,s] (int32). Pair (t,s) is valid iff qid != 0, qid == kid and, when
 * causal, s <= t + causal_offset. empty_policy says what a row without any
 * valid key returns: MFB_EMPTY_UNIFORM = the uniform average of all S values
 * (the dense finfo.min fill, kernels/attention.py:26-28), MFB_EMPTY_ZERO = zeros
 * (kernels/bidirectional.py:35, kernels/attention.py:261).
 *
 * mfb_attn_ids builds (qid, kid) on the device from the reference's mask
 * arguments for each mask shape:
 *   MFB_MASK_CAUSAL   mask [B,T]                  dense_causal_attention        attention.py:206-222
 *   MFB_MASK_PREFIX   aux=prefix_mask [B,P], mask [B,T] (kid is [B,P+T])  attention.py:225-242
 *   MFB_MASK_PACKED   mask, segment_ids [B,T]      dense_packed_causal_attention attention.py:245-261
 *   MFB_MASK_BIDIR    mask [B,T] (segment_ids NULL or [B,T])  bidirectional.attention bidirectional.py:7-35
 *   MFB_MASK_CACHED   aux=valid_length [B], T=1, S=capacity  dense_cached_attention attention.py:264-282
 * and reports the matching (causal, offset, policy) through the out-params.
 */
enum mfb_mask_mode { MFB_MASK_CAUSAL = 0, MFB_MASK_PREFIX = 1, MFB_MASK_PACKED = 2, MFB_MASK_BIDIR = 3, MFB_MASK_CACHED = 4 };
enum mfb_empty_policy { MFB_EMPTY_UNIFORM = 0, MFB_EMPTY_ZERO = 1 };

int mfb_attn_ids(int mode, const int32_t* mask, const int32_t* segment_ids, const int32_t* aux, int32_t* qid,
                 int32_t* kid, int B, int T, int S, int P, int* causal, int* causal_offset, int* empty_policy,
                 void* stream);

size_t mfb_attn_workspace_size(int B, int T, int S, int H, int Hk, int D);

/* Forward: o [B,T,H,D] bf16 and lse [B,H,T] f32 (log2-domain row logsumexp of
 * the scaled logits; -inf marks a row with no valid key). Replaces
 * _dense_attention (kernels/attention.py:12-34) and the cudnn/splash backends
 * for every mask shape above. D must be 64. */
int mfb_attn_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, float* lse,
                 const int32_t* qid, const int32_t* kid, int B, int T, int S, int H, int Hk, int D, int causal,
                 int causal_offset, int empty_policy, float scale, void* workspace, size_t workspace_bytes,
                 void* stream);

/* Backward of the forward above for upstream gradient d_o: dq [B,T,H,D],
 * dk/dv [B,S,Hk,D] bf16 (GQA heads summed in-kernel). Replaces the JAX
 * autodiff of _dense_attention / bidirectional.attention. */
int mfb_attn_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o, const float* lse,
                 const uint16_t* d_o, uint16_t* dq, uint16_t* dk, uint16_t* dv, const int32_t* qid,
                 const int32_t* kid, int B, int T, int S, int H, int Hk, int D, int causal, int causal_offset,
                 int empty_policy, float scale, void* workspace, size_t workspace_bytes, void* stream);

/* Reads (and clears) the attention tensor-core kernels' device status word of
 * the current device: 0 = ok, otherwise the id of a bounded pipeline wait that
 * gave up (the kernel then unwound instead of hanging). Synchronous. */
int mfb_attn_status(int* code);

/* ---- KV-cached decode -------------------------------------------------------
 * One query per sequence: q [B,H,D], caches [B,cap,Hk,D] bf16. If new_k/new_v
 * are non-NULL, row b's new key/value [B,Hk,D] are written at slot positions[b]
 * (clamped into [0, cap-1] as dynamic_update_slice clamps its start index)
 * before attending -- the cache write of attention_block_step
 * (src/minifield_training/layers/attention.py:309-314).
 * The query attends to slots < valid_length[b] (dense_cached_attention,
 * kernels/attention.py:264-282; valid_length 0 = uniform over all slots).
 * Output o [B,H,D] bf16. The launch is stream-K over all valid positions of
 * all rows: every CTA takes an equal contiguous share, partials of the rows a
 * share cuts go to the workspace, and the last CTA of each such row combines
 * them. The workspace depends on B and H only, not on the capacity.
 * D must be 64; H/Hk in {1,2,4}; Hk in {1,2,4,8}; B <= 8192; B x capacity
 * < 2^31; q, o, the caches and new_k/new_v 16-byte aligned. */
size_t mfb_decode_workspace_size(int B, int capacity, int H, int D);
int mfb_decode_attn(const uint16_t* q, uint16_t* k_cache, uint16_t* v_cache, const uint16_t* new_k,
                    const uint16_t* new_v, const int32_t* positions, const int32_t* valid_length, uint16_t* o,
                    int B, int capacity, int H, int Hk, int D, float scale, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Allocation-free decode step. No counterpart in the reference: it exists for
 * callers that cannot call cudaMalloc -- work recorded inside a CUDA-graph
 * capture, an XLA FFI custom-call handler that may only touch the buffers it
 * is given, a serving loop that forbids allocation after start-up. Same
 * inputs, outputs and semantics as mfb_decode_attn, but the partial scratch is
 * a fixed array of MFB_DECODE_NOALLOC_SCRATCH_BYTES compiled into the library
 * (every GPU that loads the library holds it until the process exits);
 * shapes needing more (mfb_decode_workspace_size > the maximum; B=64 rows
 * of 16 query heads need about 4.6 MB at any capacity) are rejected with
 * MFB_ERR_INVALID. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture. Every call on a device shares the one array
 * and leaves its contents behind (each call clears the parts that must start
 * at zero), so calls that overlap on the GPU -- concurrent streams, or host
 * threads on one device -- race and must be serialised by the caller. No
 * cudaMalloc, cudaFree or allocating library routine is called. */
#define MFB_DECODE_NOALLOC_SCRATCH_BYTES (8 << 20)
int mfb_decode_attn_noalloc(const uint16_t* q, uint16_t* k_cache, uint16_t* v_cache, const uint16_t* new_k,
                            const uint16_t* new_v, const int32_t* positions, const int32_t* valid_length,
                            uint16_t* o, int B, int capacity, int H, int Hk, int D, float scale, void* stream);

/* ---- GEMM (tcgen05) ----------------------------------------------------------
 * C[M,N] = alpha * op(A) . op(B)^T, bf16 operands, fp32 accumulation in TMEM.
 * a_major / b_major: MFB_MAJOR_K when the operand is stored [rows, K] (K
 * contiguous, row stride lda/ldb), MFB_MAJOR_MN when stored [K, rows] (rows
 * contiguous). out_dtype: MFB_DTYPE_BF16 or MFB_DTYPE_F32. If mask is
 * non-NULL (uint8 [M,N], row stride N) the result is multiplied by it (the
 * STE mask of the QAT weight gradient). This is the GEMM of full_linear
 * (src/minifield_training/kernels/linear.py:7-13) and its two transposes. */
enum mfb_major { MFB_MAJOR_K = 0, MFB_MAJOR_MN = 1 };
enum mfb_dtype { MFB_DTYPE_BF16 = 0, MFB_DTYPE_F32 = 1 };
int mfb_gemm_bf16(const uint16_t* A, int a_major, int lda, const uint16_t* B, int b_major, int ldb, void* C,
                  int ldc, int out_dtype, int M, int N, int K, float alpha, const uint8_t* mask, void* stream);
/* Reads (and clears) the tensor-core kernels' device status word of the
 * current device: 0 = ok, otherwise the id of a bounded pipeline wait that gave
 * up (the kernel then unwound instead of hanging). Synchronous. */
int mfb_gemm_status(int* code);

/* ---- SwiGLU glue between the QAT GEMMs (layers/feed_forward.py:24-35) ------
 * gu [M, 2F] bf16 (gate columns first) -> h [M,F] = silu(gate) * up, bf16.
 * Backward: dh [M,F] -> dgu [M,2F] bf16. */
int mfb_swiglu_fwd(const uint16_t* gu, uint16_t* h, int M, int F, void* stream);
int mfb_swiglu_bwd(const uint16_t* gu, const uint16_t* dh, uint16_t* dgu, int M, int F, void* stream);

/* FP32 -> bf16 round-to-nearest-even cast of n elements: the master cast of
 * full_linear (src/minifield_training/kernels/linear.py:11). */
int mfb_cast_f32_bf16(const float* x, uint16_t* y, long long n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MFB200_H_ */
