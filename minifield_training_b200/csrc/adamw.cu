// Transactional clipped AdamW over flat FP32 state arenas, plus the logical
// step's loss/count normalization.
//
// Replaces src/minifield_training/optimizers/adamw.py:384-571
// (make_transaction) and the normalization of src/minifield_training/engine/
// step.py:384-395. Semantics kept: one commit of every trainable master and
// both moments, or the incoming state left untouched with a CommitCode; the
// code precedence INVALID_STATE > ACCUMULATION_INVALID > NONFINITE_LOSS >
// NONFINITE_GRADIENT > STEP_OVERFLOW; the clip scale
// min(1, clip / ||g||) (1 for a zero norm); bias-corrected moments; direction
// 0 where m_hat == 0; decoupled decay only on decayed leaves; frozen leaves
// bit-identical; CANDIDATE_INVALID when the norms or any candidate leaf is
// non-finite (or a candidate second moment negative).
//
// Layout: the caller orders each arena [decayed trainable | undecayed
// trainable | frozen]; params, m and v cover n_total elements, grads the
// first n_train. Three HBM-bound passes, each a grid-stride loop over 16-byte
// vectors with one ticketed last block that finalizes the scalars:
//   check     reads params, m, v (all) and grads; state/gradient flags and
//             sum (g/divisor)^2 in FP64 (no overflow, so no max pre-pass)
//   candidate recomputes the update without writing; candidate flags and
//             sum delta^2 in FP64
//   commit    if still COMMITTED, recomputes and writes params, m, v; step++
// The update is recomputed rather than staged so the arenas are written once,
// only after the whole candidate is known to be valid. Elementwise math uses
// explicitly rounded FP32 operations (no contraction into FMA) in the
// reference's operation order.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace mfb {
namespace adamw {

enum Code { COMMITTED = 0, ACCUMULATION_INVALID, NONFINITE_LOSS, INVALID_STATE, NONFINITE_GRADIENT, STEP_OVERFLOW,
            CANDIDATE_INVALID };

constexpr int THREADS = 256;
constexpr int MAX_BLOCKS = 1024;

// Device scalars shared by the three passes (at the workspace start).
struct Scalars {
  unsigned int ticket;  // last-block election of the current pass (zeroed per call)
  int code;
  float loss, divisor, clip_scale, bc1, bc2;
  double sum;
  int bad;
};

struct Partial {
  double sum;
  int bad;
  int pad;
};

struct Hyper {
  float lr, beta1, beta2, eps, wd, clip;
};

// Reported result, laid out as the header's mfb_adamw_result.
struct Result {
  int code, committed;
  float loss, gradient_norm, clipped_gradient_norm, update_norm;
};

__device__ __forceinline__ bool finite(float x) { return isfinite(x); }

// The candidate of one trainable element, rounded op by op.
__device__ __forceinline__ void update(float p, float g, float m, float v, bool decayed, const Scalars& s,
                                       const Hyper& h, float& p1, float& m1, float& v1) {
  const float gradient = __fmul_rn(__fdiv_rn(g, s.divisor), s.clip_scale);
  m1 = __fadd_rn(__fmul_rn(h.beta1, m), __fmul_rn(__fsub_rn(1.f, h.beta1), gradient));
  v1 = __fadd_rn(__fmul_rn(h.beta2, v), __fmul_rn(__fmul_rn(__fsub_rn(1.f, h.beta2), gradient), gradient));
  const float mh = __fdiv_rn(m1, s.bc1), vh = __fdiv_rn(v1, s.bc2);
  const float dir = mh == 0.f ? 0.f : __fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), h.eps));
  const float decay = decayed ? __fmul_rn(h.wd, p) : 0.f;
  p1 = __fsub_rn(p, __fmul_rn(h.lr, __fadd_rn(dir, decay)));
}

// Block reduction of (sum, bad) into partial[blockIdx.x]; returns true in the
// last block to finish (after its partial is visible), which then reads all.
__device__ bool block_finish(double sum, int bad, Partial* partial, Scalars* s) {
  __shared__ double ssum[THREADS / 32];
  __shared__ int sbad[THREADS / 32];
  __shared__ bool last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if (lane == 0) ssum[warp] = sum, sbad[warp] = bad;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0;
    int b = 0;
    for (int w = 0; w < THREADS / 32; ++w) t += ssum[w], b |= sbad[w];
    partial[blockIdx.x].sum = t;
    partial[blockIdx.x].bad = b;
    __threadfence();
    last = atomicAdd(&s->ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return false;
  __threadfence();
  if (threadIdx.x == 0) {
    double t = 0;
    int b = 0;
    for (unsigned i = 0; i < gridDim.x; ++i) t += __ldcg(&partial[i].sum), b |= __ldcg(&partial[i].bad);
    s->sum = t;
    s->bad = b;
    s->ticket = 0;  // the next pass elects its own last block
  }
  __syncthreads();
  return true;
}

// Code, clip scale and bias corrections from the (global) state/gradient
// flags and gradient sum of squares; one thread.
__device__ void check_finalize(double gsum, int bad, const int* step, const float* loss, const uint8_t* acc_valid,
                               float div, Hyper h, Scalars* s, Result* result) {
  const int st = *step;
  const float l = *loss;
  int code = COMMITTED;
  if ((bad & 1) || st < 0) code = INVALID_STATE;
  else if (!*acc_valid) code = ACCUMULATION_INVALID;
  else if (!finite(l)) code = NONFINITE_LOSS;
  else if (bad & 2) code = NONFINITE_GRADIENT;
  else if (st >= 0x7fffffff) code = STEP_OVERFLOW;
  const float gnorm = (float)sqrt(gsum);
  const float scale = gnorm == 0.f ? 1.f : fminf(1.f, __fdiv_rn(h.clip, gnorm));
  const float t = (float)((long long)st + 1);
  s->sum = gsum;
  s->bad = bad;
  s->code = code;
  s->loss = l;
  s->divisor = div;
  s->clip_scale = scale;
  s->bc1 = __fsub_rn(1.f, (float)pow((double)h.beta1, (double)t));
  s->bc2 = __fsub_rn(1.f, (float)pow((double)h.beta2, (double)t));
  result->code = code;
  result->committed = 0;
  result->loss = l;
  const float nan = __int_as_float(0x7fc00000);
  result->gradient_norm = code == COMMITTED ? gnorm : nan;
  result->clipped_gradient_norm = code == COMMITTED ? __fmul_rn(gnorm, scale) : nan;
  result->update_norm = nan;
}

// Pass 1: state and gradient checks and the gradient sum of squares over
// elements [lo, hi) (lo a multiple of 4; hi a multiple of 4 or n_total).
// Without `red` the last block finalizes the code and scalars; with `red` it
// stores this range's (sum, state flag, gradient flag) there as doubles for a
// cross-rank sum, and check_finalize_kernel finishes.
__global__ void __launch_bounds__(THREADS) check_kernel(const float* __restrict__ params, const float* __restrict__ m,
                                                        const float* __restrict__ v, const float* __restrict__ grads,
                                                        long long lo, long long hi, long long n_train,
                                                        long long n_total, const int* step, const float* loss,
                                                        const uint8_t* acc_valid, const float* divisor, Hyper h,
                                                        Scalars* s, Partial* partial, Result* result, double* red) {
  const float div = divisor ? *divisor : 1.f;
  double sum = 0;
  int bad = 0;  // bit 0: state invalid, bit 1: gradient non-finite
  const long long stride = (long long)gridDim.x * THREADS;
  const long long nv = min(hi, n_total) / 4, nt4 = n_train / 4;
  for (long long i = lo / 4 + blockIdx.x * (long long)THREADS + threadIdx.x; i < nv; i += stride) {
    const float4 p4 = __ldcs(reinterpret_cast<const float4*>(params) + i);
    const float4 m4 = __ldcs(reinterpret_cast<const float4*>(m) + i);
    const float4 v4 = __ldcs(reinterpret_cast<const float4*>(v) + i);
    const float pp[4] = {p4.x, p4.y, p4.z, p4.w}, mm[4] = {m4.x, m4.y, m4.z, m4.w}, vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (!finite(pp[k]) || !finite(mm[k]) || !finite(vv[k]) || vv[k] < 0.f) bad |= 1;
    if (i < nt4) {
      const float4 g4 = __ldcs(reinterpret_cast<const float4*>(grads) + i);
      const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float g = __fdiv_rn(gg[k], div);
        if (!finite(g)) bad |= 2;
        sum += (double)g * (double)g;
      }
    }
  }
  // Scalar tails (fewer than four elements each) inside the range.
  if (blockIdx.x == 0) {
    const long long e = nv * 4 + threadIdx.x;
    if (e >= lo && e < min(hi, n_total) && (!finite(params[e]) || !finite(m[e]) || !finite(v[e]) || v[e] < 0.f))
      bad |= 1;
    const long long f = nt4 * 4 + threadIdx.x;
    if (f >= lo && f < min(hi, n_train)) {
      const float g = __fdiv_rn(grads[f], div);
      if (!finite(g)) bad |= 2;
      sum += (double)g * (double)g;
    }
  }
  if (!block_finish(sum, bad, partial, s)) return;
  if (threadIdx.x != 0) return;
  if (red) {
    red[0] = s->sum;
    red[1] = (s->bad & 1) ? 1.0 : 0.0;
    red[2] = (s->bad & 2) ? 1.0 : 0.0;
    return;
  }
  check_finalize(s->sum, s->bad, step, loss, acc_valid, div, h, s, result);
}

__global__ void check_finalize_kernel(const double* red, const int* step, const float* loss, const uint8_t* acc_valid,
                                      const float* divisor, Hyper h, Scalars* s, Result* result) {
  const int bad = (red[1] > 0.0 ? 1 : 0) | (red[2] > 0.0 ? 2 : 0);
  check_finalize(red[0], bad, step, loss, acc_valid, divisor ? *divisor : 1.f, h, s, result);
}

// Update norm and candidate verdict from the (global) sum of squared deltas
// and candidate flag; one thread.
__device__ void candidate_finalize(double usum, int bad, Scalars* s, Result* result) {
  const float unorm = (float)sqrt(usum);
  const bool ok = finite(result->gradient_norm) && finite(unorm) && !bad;
  result->update_norm = unorm;
  if (!ok) {
    s->code = CANDIDATE_INVALID;
    result->code = CANDIDATE_INVALID;
  }
}

// Pass 2 (commit = false): candidate checks and update norm, no writes.
// Pass 3 (commit = true): the same arithmetic, written back when committed.
// Both over trainable elements [lo, hi) (lo a multiple of 4; hi a multiple of
// 4 or n_train). With `red`, the candidate pass stores this range's (sum,
// flag) there for a cross-rank sum and candidate_finalize_kernel finishes.
template <bool COMMIT>
__global__ void __launch_bounds__(THREADS) update_kernel(float* __restrict__ params, float* __restrict__ m,
                                                         float* __restrict__ v, const float* __restrict__ grads,
                                                         long long lo, long long hi, long long n_decayed, int* step,
                                                         Hyper h, Scalars* s, Partial* partial, Result* result,
                                                         double* red) {
  const Scalars sc = *s;
  if (sc.code != COMMITTED) return;  // uniform across the grid: no pass election needed
  double sum = 0;
  int bad = 0;
  const long long stride = (long long)gridDim.x * THREADS;
  const long long nt4 = hi / 4;
  for (long long i = lo / 4 + blockIdx.x * (long long)THREADS + threadIdx.x; i < nt4; i += stride) {
    const float4 p4 = reinterpret_cast<const float4*>(params)[i];
    const float4 m4 = __ldcs(reinterpret_cast<const float4*>(m) + i);
    const float4 v4 = __ldcs(reinterpret_cast<const float4*>(v) + i);
    const float4 g4 = __ldcs(reinterpret_cast<const float4*>(grads) + i);
    const float pp[4] = {p4.x, p4.y, p4.z, p4.w}, mm[4] = {m4.x, m4.y, m4.z, m4.w};
    const float vv[4] = {v4.x, v4.y, v4.z, v4.w}, gg[4] = {g4.x, g4.y, g4.z, g4.w};
    float p1[4], m1[4], v1[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      update(pp[k], gg[k], mm[k], vv[k], i * 4 + k < n_decayed, sc, h, p1[k], m1[k], v1[k]);
      if (!COMMIT) {
        if (!finite(p1[k]) || !finite(m1[k]) || !finite(v1[k]) || v1[k] < 0.f) bad = 1;
        const double d = (double)__fsub_rn(p1[k], pp[k]);
        sum += d * d;
      }
    }
    if (COMMIT) {
      reinterpret_cast<float4*>(params)[i] = make_float4(p1[0], p1[1], p1[2], p1[3]);
      __stcs(reinterpret_cast<float4*>(m) + i, make_float4(m1[0], m1[1], m1[2], m1[3]));
      __stcs(reinterpret_cast<float4*>(v) + i, make_float4(v1[0], v1[1], v1[2], v1[3]));
    }
  }
  if (blockIdx.x == 0) {
    const long long e = nt4 * 4 + threadIdx.x;
    if (e >= lo && e < hi) {
      float p1, m1, v1;
      update(params[e], grads[e], m[e], v[e], e < n_decayed, sc, h, p1, m1, v1);
      if (COMMIT) {
        params[e] = p1, m[e] = m1, v[e] = v1;
      } else {
        if (!finite(p1) || !finite(m1) || !finite(v1) || v1 < 0.f) bad = 1;
        const double d = (double)__fsub_rn(p1, params[e]);
        sum += d * d;
      }
    }
  }
  if (COMMIT) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      *step = *step + 1;
      result->committed = 1;
    }
    return;
  }
  if (!block_finish(sum, bad, partial, s)) return;
  if (threadIdx.x != 0) return;
  if (red) {
    red[0] = s->sum;
    red[1] = s->bad ? 1.0 : 0.0;
    return;
  }
  candidate_finalize(s->sum, s->bad, s, result);
}

__global__ void candidate_finalize_kernel(const double* red, Scalars* s, Result* result) {
  if (s->code != COMMITTED) return;
  candidate_finalize(red[0], red[1] > 0.0 ? 1 : 0, s, result);
}

// engine/step.py:384-389: valid count, denominator, normalized loss.
__global__ void normalize_kernel(const float* loss_sum, const float* count_sum, const uint8_t* counts_valid,
                                 float* loss, float* divisor, uint8_t* valid) {
  const float c = *count_sum;
  const bool ok = (counts_valid ? *counts_valid != 0 : true) && isfinite(c) && c > 0.f;
  const float d = ok ? c : 1.f;
  *divisor = d;
  *loss = __fdiv_rn(*loss_sum, d);
  *valid = ok;
}

size_t workspace_bytes() { return 256 + sizeof(Partial) * MAX_BLOCKS; }

}  // namespace adamw
}  // namespace mfb

using namespace mfb;

extern "C" size_t mfb_adamw_workspace_size(void) { return adamw::workspace_bytes(); }

extern "C" int mfb_adamw_commit(float* params, float* m, float* v, const float* grads, long long n_train,
                                long long n_decayed, long long n_total, int32_t* step, const float* loss,
                                const uint8_t* accumulation_valid, const float* grad_divisor, float learning_rate,
                                float beta1, float beta2, float epsilon, float weight_decay, float clip_norm,
                                void* result, void* workspace, size_t workspace_bytes, void* stream) {
  MFB_CHECK_ARG(n_train > 0 && n_decayed >= 0 && n_decayed <= n_train && n_total >= n_train,
                "AdamW needs 0 <= n_decayed <= n_train <= n_total and a trainable leaf (%lld, %lld, %lld)", n_decayed,
                n_train, n_total);
  MFB_CHECK_ARG(params && m && v && grads && step && loss && accumulation_valid && result, "NULL AdamW argument");
  MFB_CHECK_ARG((((uintptr_t)params | (uintptr_t)m | (uintptr_t)v | (uintptr_t)grads) & 15) == 0,
                "AdamW arenas must be 16-byte aligned");
  MFB_CHECK_ARG(learning_rate > 0.f && beta1 >= 0.f && beta1 < 1.f && beta2 >= 0.f && beta2 < 1.f && epsilon > 0.f &&
                    weight_decay >= 0.f && clip_norm > 0.f,
                "invalid AdamW hyperparameters");
  MFB_CHECK_ARG(workspace && workspace_bytes >= adamw::workspace_bytes(), "AdamW workspace needs %zu bytes",
                adamw::workspace_bytes());
  cudaStream_t s = (cudaStream_t)stream;
  auto* sc = reinterpret_cast<adamw::Scalars*>(workspace);
  auto* partial = reinterpret_cast<adamw::Partial*>(static_cast<char*>(workspace) + 256);
  auto* res = reinterpret_cast<adamw::Result*>(result);
  int dev = 0, sms = 148;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  MFB_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const long long vec = (n_total + 3) / 4;
  const int blocks = (int)std::min<long long>(std::max<long long>(1, (vec + adamw::THREADS - 1) / adamw::THREADS),
                                              std::min(4 * sms, adamw::MAX_BLOCKS));
  const adamw::Hyper h{learning_rate, beta1, beta2, epsilon, weight_decay, clip_norm};
  MFB_CUDA_TRY(cudaMemsetAsync(sc, 0, sizeof(adamw::Scalars), s));
  adamw::check_kernel<<<blocks, adamw::THREADS, 0, s>>>(params, m, v, grads, 0, n_total, n_train, n_total, step,
                                                        loss, accumulation_valid, grad_divisor, h, sc, partial, res,
                                                        nullptr);
  MFB_LAUNCH_CHECK("adamw check");
  adamw::update_kernel<false><<<blocks, adamw::THREADS, 0, s>>>(params, m, v, grads, 0, n_train, n_decayed, step, h,
                                                                sc, partial, res, nullptr);
  MFB_LAUNCH_CHECK("adamw candidate");
  adamw::update_kernel<true><<<blocks, adamw::THREADS, 0, s>>>(params, m, v, grads, 0, n_train, n_decayed, step, h,
                                                               sc, partial, res, nullptr);
  MFB_LAUNCH_CHECK("adamw commit");
  return MFB_OK;
}

// One pass of the transaction over this rank's slice, for an optimizer
// sharded across data-parallel ranks. Every rank holds the full reduced
// gradients and calls, in order: CHECK over its slice of [0, n_total) ->
// SUM-allreduce red[0..2] -> CHECK_FINALIZE -> CANDIDATE over its slice of the
// trainable range -> SUM-allreduce red[0..1] -> CANDIDATE_FINALIZE -> COMMIT
// over the same trainable slice; then the ranks all-gather the updated
// masters. The finalize passes see the same reduced values on every rank, so
// every rank reaches the same code. Nonempty slices start at multiples of 4
// elements.
extern "C" int mfb_adamw_shard_pass(int pass, float* params, float* m, float* v, const float* grads, long long lo,
                                    long long hi, long long n_train, long long n_decayed, long long n_total,
                                    int32_t* step, const float* loss, const uint8_t* accumulation_valid,
                                    const float* grad_divisor, float learning_rate, float beta1, float beta2,
                                    float epsilon, float weight_decay, float clip_norm, double* red, void* result,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  MFB_CHECK_ARG(pass >= MFB_ADAMW_CHECK && pass <= MFB_ADAMW_COMMIT, "unknown AdamW pass %d", pass);
  MFB_CHECK_ARG(n_train > 0 && n_decayed >= 0 && n_decayed <= n_train && n_total >= n_train,
                "AdamW needs 0 <= n_decayed <= n_train <= n_total and a trainable leaf (%lld, %lld, %lld)", n_decayed,
                n_train, n_total);
  const long long lim = (pass == MFB_ADAMW_CHECK) ? n_total : n_train;
  MFB_CHECK_ARG(lo >= 0 && lo <= hi && hi <= lim && (lo % 4 == 0 || lo == hi) && (hi % 4 == 0 || hi == lim),
                "AdamW slice [%lld, %lld) must start at a multiple of 4 inside [0, %lld)", lo, hi, lim);
  MFB_CHECK_ARG(params && m && v && grads && step && loss && accumulation_valid && result && red,
                "NULL AdamW argument");
  MFB_CHECK_ARG((((uintptr_t)params | (uintptr_t)m | (uintptr_t)v | (uintptr_t)grads) & 15) == 0,
                "AdamW arenas must be 16-byte aligned");
  MFB_CHECK_ARG(learning_rate > 0.f && beta1 >= 0.f && beta1 < 1.f && beta2 >= 0.f && beta2 < 1.f && epsilon > 0.f &&
                    weight_decay >= 0.f && clip_norm > 0.f,
                "invalid AdamW hyperparameters");
  MFB_CHECK_ARG(workspace && workspace_bytes >= adamw::workspace_bytes(), "AdamW workspace needs %zu bytes",
                adamw::workspace_bytes());
  cudaStream_t s = (cudaStream_t)stream;
  auto* sc = reinterpret_cast<adamw::Scalars*>(workspace);
  auto* partial = reinterpret_cast<adamw::Partial*>(static_cast<char*>(workspace) + 256);
  auto* res = reinterpret_cast<adamw::Result*>(result);
  int dev = 0, sms = 148;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  MFB_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const long long vec = (hi - lo + 3) / 4;
  const int blocks = (int)std::min<long long>(std::max<long long>(1, (vec + adamw::THREADS - 1) / adamw::THREADS),
                                              std::min(4 * sms, adamw::MAX_BLOCKS));
  const adamw::Hyper h{learning_rate, beta1, beta2, epsilon, weight_decay, clip_norm};
  switch (pass) {
    case MFB_ADAMW_CHECK:
      MFB_CUDA_TRY(cudaMemsetAsync(sc, 0, sizeof(adamw::Scalars), s));
      adamw::check_kernel<<<blocks, adamw::THREADS, 0, s>>>(params, m, v, grads, lo, hi, n_train, n_total, step, loss,
                                                            accumulation_valid, grad_divisor, h, sc, partial, res, red);
      break;
    case MFB_ADAMW_CHECK_FINALIZE:
      adamw::check_finalize_kernel<<<1, 1, 0, s>>>(red, step, loss, accumulation_valid, grad_divisor, h, sc, res);
      break;
    case MFB_ADAMW_CANDIDATE:
      adamw::update_kernel<false><<<blocks, adamw::THREADS, 0, s>>>(params, m, v, grads, lo, hi, n_decayed, step, h,
                                                                    sc, partial, res, red);
      break;
    case MFB_ADAMW_CANDIDATE_FINALIZE:
      adamw::candidate_finalize_kernel<<<1, 1, 0, s>>>(red, sc, res);
      break;
    default:
      adamw::update_kernel<true><<<blocks, adamw::THREADS, 0, s>>>(params, m, v, grads, lo, hi, n_decayed, step, h,
                                                                   sc, partial, res, nullptr);
      break;
  }
  MFB_LAUNCH_CHECK("adamw shard pass");
  return MFB_OK;
}

extern "C" int mfb_step_normalize(const float* loss_sum, const float* count_sum, const uint8_t* counts_valid,
                                  float* loss, float* divisor, uint8_t* accumulation_valid, void* stream) {
  MFB_CHECK_ARG(loss_sum && count_sum && loss && divisor && accumulation_valid, "NULL normalization argument");
  adamw::normalize_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(loss_sum, count_sum, counts_valid, loss, divisor,
                                                             accumulation_valid);
  MFB_LAUNCH_CHECK("step normalize");
  return MFB_OK;
}
