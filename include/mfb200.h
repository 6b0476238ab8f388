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
  MFB_ERR_DEVICE = 5,      /* a device-side status word reported an error */
  MFB_ERR_COMM = 6         /* a collective failed or passed its deadline; the communicator is aborted */
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
/* Strided device copy of `height` rows of `width` bytes (pitches in bytes):
 * writes prompt keys/values into the fixed-capacity cache rows, the
 * jnp.pad(key * keep) of layers/attention.py:269-278. */
int mfb_memcpy2d_d2d(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width, size_t height,
                     void* stream);
int mfb_memset(void* dst, int value, size_t bytes, void* stream);
int mfb_stream_create(void** stream);
int mfb_stream_destroy(void* stream);
int mfb_stream_sync(void* stream);
int mfb_device_sync(void);
/* Ends this process's context on the current device (cudaDeviceReset): every
 * device pointer, stream, event and graph of it becomes invalid. Other
 * processes on the GPU are not affected. */
int mfb_device_reset(void);
int mfb_event_create(void** event);
int mfb_event_destroy(void* event);
int mfb_event_record(void* event, void* stream);
int mfb_stream_wait_event(void* stream, void* event);
int mfb_event_elapsed_ms(void* start, void* end, float* ms);
/* CUDA graphs: everything enqueued on `stream` (a created stream) between
 * mfb_graph_begin and mfb_graph_end is recorded into one executable graph;
 * mfb_graph_launch replays it. Arguments are fixed at capture. */
int mfb_graph_begin(void* stream);
int mfb_graph_end(void* stream, void** graph_exec);
int mfb_graph_launch(void* graph_exec, void* stream);
int mfb_graph_destroy(void* graph_exec);

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
 * MFB_ERR_INVALID. The first call in each CUDA context of a device looks up
 * the array's device address (cudaGetSymbolAddress) with that device
 * current, and caches it under the context's unique ID; a context destroyed
 * and re-created (cudaDeviceReset, mfb_device_reset) gets a new ID, so the
 * first call after it looks the address up again. Make the first call of each
 * context before any stream capture. Every call on a device shares the one array
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
/* The gate|up projection of the SwiGLU block with the SwiGLU product in its
 * epilogue (src/minifield_training/layers/feed_forward.py:24-35):
 * gu[M, 2F] = A[M,K] . W13^T (bf16, gate columns [0,F), up [F,2F); W13 is the
 * row-concatenation [gate; up] of the two [F, K] weights, K-major, row stride
 * ldw) and h[M, F] = silu(gate) * up (bf16), each value rounded where the
 * reference's bf16 graph rounds it. F a multiple of 128; gu, h, W13 16-byte
 * aligned. Replaces mfb_gemm_bf16 + mfb_swiglu_fwd (gu is not re-read). */
int mfb_gemm_swiglu_fwd(const uint16_t* A, int a_major, int lda, const uint16_t* W13, int ldw, uint16_t* gu,
                        uint16_t* h, int M, int F, int K, void* stream);
/* The down projection's input gradient with the SwiGLU backward in its
 * epilogue: dH = dY[M,K] . Wd (Wd stored [K, F] with b_major MFB_MAJOR_MN, or
 * [F, K] with MFB_MAJOR_K), rounded to bf16, then dgu[M, 2F] =
 * [dH * up * silu'(gate), dH * silu(gate)] from gu[M, 2F]. dH is not stored.
 * F a multiple of 32; gu and dgu distinct, 16-byte aligned. Replaces
 * mfb_gemm_bf16 + mfb_swiglu_bwd. */
int mfb_gemm_swiglu_bwd(const uint16_t* dY, int a_major, int lda, const uint16_t* Wd, int b_major, int ldb,
                        const uint16_t* gu, uint16_t* dgu, int M, int F, int K, void* stream);
/* The same product with a caller-owned workspace that enables split-K where
 * the output tiles fill the GPU poorly: small M (the decode step's [batch, C]
 * x W^T projections and logits, models/lfm2_5/decode.py:356-361,
 * layers/attention.py:281-322) and the weight gradients of full_linear's VJP
 * (kernels/linear.py:7-13: dW = dY^T X over all tokens, a few output tiles
 * with a very deep K). K is cut into slices whose FP32 partials are summed in
 * slice order (deterministic), then scaled and masked. The workspace (16-byte
 * aligned) needs mfb_gemm_workspace_size(M, N, K) bytes for the full split of
 * the unmasked product; a smaller one gets fewer slices, NULL or 0 none.
 * Unmasked products of at most 64 rows run as C^T = B A^T internally (the
 * weight rows fill the tensor core's 128-row side, C is stored transposed),
 * so a wide projection of a decode batch needs no split at all.
 * flags: MFB_GEMM_PDL launches the GEMM as a programmatic dependent of the
 * previous kernel on the stream (a created stream, not the legacy default
 * one): its first B tiles load while that kernel finishes, A and the output
 * wait for its completion. The caller asserts that no kernel still running on
 * the stream writes B (true of weights). */
enum mfb_gemm_flags { MFB_GEMM_PDL = 1 };
size_t mfb_gemm_workspace_size(int M, int N, int K);
int mfb_gemm_bf16_ws(const uint16_t* A, int a_major, int lda, const uint16_t* B, int b_major, int ldb, void* C,
                     int ldc, int out_dtype, int M, int N, int K, float alpha, const uint8_t* mask, int flags,
                     void* workspace, size_t workspace_bytes, void* stream);
/* Reads (and clears) the tensor-core kernels' device status word of the
 * current device: 0 = ok, otherwise the id of a bounded pipeline wait that gave
 * up (the kernel then unwound instead of hanging). Synchronous. */
int mfb_gemm_status(int* code);

/* ---- Transactional AdamW (src/minifield_training/optimizers/adamw.py:384-571)
 * One all-or-nothing clipped AdamW update over flat FP32 arenas ordered
 * [decayed trainable | undecayed trainable | frozen]: params, m and v hold
 * n_total elements, grads the first n_train (n_decayed <= n_train). Device
 * scalars: step (int32, incremented on commit), loss, accumulation_valid
 * (uint8) and, when non-NULL, grad_divisor (the logical step's denominator;
 * gradients are divided by it before anything else, as
 * src/minifield_training/engine/step.py:389 does). Codes and their precedence
 * follow CommitCode (adamw.py:30-39, :437-461); the gradient norm, clip scale
 * and update norm follow adamw.py:476-541; a candidate with a non-finite norm
 * or leaf is rejected (adamw.py:543-569). A rejected update writes nothing.
 * `result` is a device mfb_adamw_result written by the call. Arenas must be
 * 16-byte aligned. Calls on one workspace must not overlap. */
typedef struct {
  int32_t code; /* 0 committed, 1 accumulation invalid, 2 non-finite loss, 3 invalid state,
                   4 non-finite gradient, 5 step overflow, 6 candidate invalid */
  int32_t committed;
  float loss, gradient_norm, clipped_gradient_norm, update_norm; /* NaN norms when rejected before the attempt */
} mfb_adamw_result;
size_t mfb_adamw_workspace_size(void);
int mfb_adamw_commit(float* params, float* m, float* v, const float* grads, long long n_train, long long n_decayed,
                     long long n_total, int32_t* step, const float* loss, const uint8_t* accumulation_valid,
                     const float* grad_divisor, float learning_rate, float beta1, float beta2, float epsilon,
                     float weight_decay, float clip_norm, void* result, void* workspace, size_t workspace_bytes,
                     void* stream);
/* One pass of the same transaction over this rank's slice, for an AdamW state
 * sharded across data-parallel ranks (the reference keeps the state
 * replicated: adamw.py:384-571 applied to every rank's copy after the psum of
 * engine/step.py:62; slicing the elementwise update leaves the arithmetic per
 * element unchanged). Order per step: CHECK on [lo, hi) of [0, n_total) ->
 * SUM-allreduce red[0..2] -> CHECK_FINALIZE -> CANDIDATE on [lo, hi) of the
 * trainable range -> SUM-allreduce red[0..1] -> CANDIDATE_FINALIZE -> COMMIT
 * on that slice -> all-gather of the masters. `red` is a caller-owned device
 * buffer of 3 doubles. Nonempty slices start at multiples of 4 elements. */
enum {
  MFB_ADAMW_CHECK = 0,
  MFB_ADAMW_CHECK_FINALIZE = 1,
  MFB_ADAMW_CANDIDATE = 2,
  MFB_ADAMW_CANDIDATE_FINALIZE = 3,
  MFB_ADAMW_COMMIT = 4
};
int mfb_adamw_shard_pass(int pass, float* params, float* m, float* v, const float* grads, long long lo, long long hi,
                         long long n_train, long long n_decayed, long long n_total, int32_t* step, const float* loss,
                         const uint8_t* accumulation_valid, const float* grad_divisor, float learning_rate,
                         float beta1, float beta2, float epsilon, float weight_decay, float clip_norm, double* red,
                         void* result, void* workspace, size_t workspace_bytes, void* stream);
/* Logical-step normalization (src/minifield_training/engine/step.py:384-389):
 * accumulation_valid = counts_valid && isfinite(count_sum) && count_sum > 0;
 * divisor = count_sum if valid else 1; loss = loss_sum / divisor. All device
 * scalars; counts_valid may be NULL (true). */
int mfb_step_normalize(const float* loss_sum, const float* count_sum, const uint8_t* counts_valid, float* loss,
                       float* divisor, uint8_t* accumulation_valid, void* stream);

/* ---- Encoder training-step kernels -------------------------------------------
 * bf16 activations [M, C] (M = B*T packed tokens), FP32 masters and FP32
 * weight gradients. Weight-gradient outputs are written, or added to when
 * `accumulate` is nonzero. Workspaces hold per-block partial sums.
 *
 * rms_norm (src/minifield_training/kernels/normalization.py:7-22) with the
 * encoder block's bf16 residual add fused in front (encoder.py:64-110): when
 * `residual` is non-NULL, sum_out = bf16(x + residual) is written and
 * normalized; y = bf16(bf16(s * rstd) * bf16(weight)), times row_mask[m] when
 * row_mask is non-NULL (conv_input_projection, layers/convolution.py:29-37);
 * rstd [M] FP32 is saved for the backward. C a multiple of 256, <= 2048. */
size_t mfb_norm_workspace_size(int M, int C);
int mfb_rmsnorm_fwd(const uint16_t* x, const uint16_t* residual, const float* weight, const int32_t* row_mask,
                    uint16_t* sum_out, uint16_t* y, float* rstd, int M, int C, float eps, void* stream);
/* dx = dres + d(rms_norm)/dx . dy (dres may be NULL); dweight [C]. C <= 1024. */
int mfb_rmsnorm_bwd(const uint16_t* x, const float* weight, const float* rstd, const int32_t* row_mask,
                    const uint16_t* dy, const uint16_t* dres, uint16_t* dx, float* dweight, int accumulate, int M,
                    int C, void* workspace, size_t workspace_bytes, void* stream);
/* Per-head q/k RMSNorm (project_qkv, layers/attention.py:61-77) and rotary
 * embedding (apply_rotary, kernels/rotary.py:7-39) on the fused projection
 * output qkv [M, ld_qkv] = [q heads | k heads | v heads] x 64: writes q
 * [M,H,64], k and v [M,Hk,64]. freqs [32] = theta^(-2i/64) in FP32;
 * positions [M]. The backward writes d_qkv [M, ld_qkv] and the 64-wide gain
 * gradients. */
int mfb_qknorm_rope_fwd(const uint16_t* qkv, int ld_qkv, const float* wq, const float* wk, const int32_t* positions,
                        const float* freqs, uint16_t* q, uint16_t* k, uint16_t* v, float* rstd_q, float* rstd_k,
                        int M, int H, int Hk, float eps, void* stream);
int mfb_qknorm_rope_bwd(const uint16_t* qkv, int ld_qkv, const float* wq, const float* wk, const int32_t* positions,
                        const float* freqs, const float* rstd_q, const float* rstd_k, const uint16_t* dq,
                        const uint16_t* dk, const uint16_t* dv, uint16_t* dqkv, float* dwq, float* dwk, int accumulate,
                        int M, int H, int Hk, void* workspace, size_t workspace_bytes, void* stream);
/* Frozen token embedding rows cast to bf16 (encoder.py:231); ids clamped to [0, V). */
int mfb_embed_gather(const float* table, const int32_t* ids, uint16_t* out, long long M, int C, int V, void* stream);
/* Gated centered short convolution (encoder.py:76-86,
 * kernels/bidirectional.py:38-58): bcx [M, 3C] = [b | c | values] from the
 * in-projection, taps [C, 3] FP32, segment_ids [M] (rows of T tokens; 0 =
 * padding) -> mixed [M, C] = c * conv(b * values). */
int mfb_conv_fwd(const uint16_t* bcx, const float* taps, const int32_t* segment_ids, uint16_t* mixed, long long M,
                 int T, int C, void* stream);
size_t mfb_encoder_workspace_size(int C, int classes);
/* One decode step of the causal gated short convolution
 * (src/minifield_training/layers/convolution.py:153-178,
 * kernels/convolution.py:82-111): bcx [B, 3C] = [b | c | values] of one token
 * per row, taps [C, 3] FP32, history [B, 2, C] bf16 (the two preceding gated
 * inputs, oldest first; shifted in place) -> mixed [B, C]. */
int mfb_conv_step(const uint16_t* bcx, const float* taps, uint16_t* history, uint16_t* mixed, int B, int C,
                  void* stream);
/* The causal gated short convolution over T tokens per row
 * (kernels/convolution.py:7-22, and :82-111 when history_in is given): bcx
 * [B*T, 3C], taps [C, 3] FP32, history_in [B, 2, C] bf16 or NULL (zeros, the
 * prompt prefix of layers/convolution.py:77-101) -> mixed [B*T, C] and, when
 * history_out is non-NULL, the continuation history [B, 2, C] (state_tail,
 * kernels/convolution.py:56-79, at length T). history_out must not alias
 * history_in. */
int mfb_conv_causal(const uint16_t* bcx, const float* taps, const uint16_t* history_in, uint16_t* history_out,
                    uint16_t* mixed, int B, int T, int C, void* stream);
int mfb_conv_bwd(const uint16_t* bcx, const float* taps, const int32_t* segment_ids, const uint16_t* dmixed,
                 uint16_t* dbcx, float* dtaps, int accumulate, long long M, int T, int C, void* workspace,
                 size_t workspace_bytes, void* stream);
/* Token classification head and summed cross-entropy, forward and backward in
 * one pass: logits = bf16(encoded . bf16(weight)^T) [M, classes];
 * loss_count[0] = sum over rows with valid != 0 of logsumexp(logits) -
 * logits[label], loss_count[1] = number of such rows; d_encoded and d_weight
 * [classes, C] are the gradients of loss_count[0]. C = 1024, classes <= 4. */
int mfb_head_loss(const uint16_t* encoded, const float* weight, const int32_t* labels, const int32_t* valid,
                  uint16_t* d_encoded, float* d_weight, float* loss_count, int M, int C, int classes, void* workspace,
                  size_t workspace_bytes, void* stream);

/* ---- SwiGLU glue between the QAT GEMMs (layers/feed_forward.py:24-35) ------
 * gu [M, 2F] bf16 (gate columns first) -> h [M,F] = silu(gate) * up, bf16.
 * Backward: dh [M,F] -> dgu [M,2F] bf16. */
int mfb_swiglu_fwd(const uint16_t* gu, uint16_t* h, int M, int F, void* stream);
int mfb_swiglu_bwd(const uint16_t* gu, const uint16_t* dh, uint16_t* dgu, int M, int F, void* stream);

/* FP32 -> bf16 round-to-nearest-even cast of n elements: the master cast of
 * full_linear (src/minifield_training/kernels/linear.py:11). */
int mfb_cast_f32_bf16(const float* x, uint16_t* y, long long n, void* stream);
/* bf16 -> FP32 widening of n elements (the logits' .astype(float32),
 * src/minifield_training/models/lfm2_5/model.py:829). */
int mfb_cast_bf16_f32(const uint16_t* x, float* y, long long n, void* stream);
/* out = a + b over n bf16 elements, each sum rounded to nearest even: the
 * residual adds of the attention block and the SwiGLU block
 * (src/minifield_training/layers/attention.py:100-108,
 * layers/feed_forward.py:35). n a multiple of 8; 16-byte aligned buffers. */
int mfb_add_bf16(const uint16_t* a, const uint16_t* b, uint16_t* out, long long n, void* stream);

/* ---- NCCL communicator (data-parallel exchange) -------------------------------
 * The psum of (loss, count, gradient tree) over the data axis of the
 * reference's training step (src/minifield_training/engine/step.py:36-78,
 * psum at :62; shard_map over the 1-D "data" mesh :72-77), and the scalar
 * reductions and master all-gather of the sharded AdamW transaction. One
 * communicator per process (rank), one GPU each.
 *
 * mfb_comm_load dlopens NCCL from path (NULL: "libnccl.so.2") once per
 * process and reports its version (e.g. 22803 for 2.28.3). Rank 0 draws the
 * unique id (mfb_comm_unique_id_bytes() bytes) and the host hands it to the
 * other ranks by any means. The communicator is non-blocking: every call
 * below returns once its work is enqueued on the stream, and each is bounded
 * by timeout_s -- an NCCL error or a missed deadline aborts the communicator
 * (ncclCommAbort; NCCL's kernels on this GPU then return) and gives
 * MFB_ERR_COMM, and an aborted communicator rejects later calls.
 * mfb_comm_wait(comm, stream, timeout_s) waits for a stream while watching
 * the communicator: the bounded wait a host uses instead of a stream sync
 * when a peer may have failed. Element types and reductions: */
enum mfb_comm_dtype { MFB_COMM_F32 = 0, MFB_COMM_F64 = 1, MFB_COMM_BF16 = 2, MFB_COMM_U8 = 3, MFB_COMM_I32 = 4 };
enum mfb_comm_op { MFB_COMM_SUM = 0, MFB_COMM_MAX = 1, MFB_COMM_MIN = 2 };
int mfb_comm_load(const char* path, int* version);
size_t mfb_comm_unique_id_bytes(void);
int mfb_comm_unique_id(void* id, size_t bytes);
int mfb_comm_init(const void* id, size_t id_bytes, int world, int rank, double timeout_s, void** comm);
int mfb_comm_rank(void* comm, int* rank, int* world);
/* recv may equal send (in place). */
int mfb_comm_allreduce(void* comm, const void* send, void* recv, size_t count, int dtype, int op, void* stream);
/* send holds world * recv_count elements; rank r receives the reduction of block r. */
int mfb_comm_reduce_scatter(void* comm, const void* send, void* recv, size_t recv_count, int dtype, int op,
                            void* stream);
/* recv holds world * send_count elements, block r from rank r; send may be recv's own block. */
int mfb_comm_allgather(void* comm, const void* send, void* recv, size_t send_count, int dtype, void* stream);
/* Reduction of `count` elements of every rank's `send` into `recv` on rank
 * `root` only (in place when send == recv), and broadcast of root's `send`
 * into every rank's `recv` (in place likewise). A data-parallel step whose
 * optimizer state is partitioned across the ranks reduces each gradient range
 * to the rank that updates it and broadcasts the updated masters back, in
 * place of the allreduce of src/minifield_training/engine/step.py:62 (the
 * reference replicates the state on every rank). */
int mfb_comm_reduce(void* comm, const void* send, void* recv, size_t count, int dtype, int op, int root,
                    void* stream);
int mfb_comm_broadcast(void* comm, const void* send, void* recv, size_t count, int dtype, int root, void* stream);
int mfb_comm_wait(void* comm, void* stream, double timeout_s);
int mfb_comm_abort(void* comm);
/* Finalizes (bounded by the communicator's timeout) and frees; NULL is a no-op. */
int mfb_comm_destroy(void* comm);

#ifdef __cplusplus
}
#endif

#endif /* MFB200_H_ */
