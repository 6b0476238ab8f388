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

// Pass 1: state and gradient checks, gradient norm, code and scalars.
__global__ void __launch_bounds__(THREADS) check_kernel(const float* __restrict__ params, const float* __restrict__ m,
                                                        const float* __restrict__ v, const float* __restrict__ grads,
                                                        long long n_train, long long n_total, const int* step,
                                                        const float* loss, const uint8_t* acc_valid,
                                                        const float* divisor, Hyper h, Scalars* s, Partial* partial,
                                                        Result* result) {
  const float div = divisor ? *divisor : 1.f;
  double sum = 0;
  int bad = 0;  // bit 0: state invalid, bit 1: gradient non-finite
  const long long stride = (long long)gridDim.x * THREADS;
  const long long nv = n_total / 4, nt4 = n_train / 4;
  for (long long i = blockIdx.x * (long long)THREADS + threadIdx.x; i < nv; i += stride) {
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
  // Scalar tails (fewer than four elements each).
  if (blockIdx.x == 0) {
    const long long e = nv * 4 + threadIdx.x;
    if (e < n_total && (!finite(params[e]) || !finite(m[e]) || !finite(v[e]) || v[e] < 0.f)) bad |= 1;
    const long long f = nt4 * 4 + threadIdx.x;
    if (f < n_train) {
      const float g = __fdiv_rn(grads[f], div);
      if (!finite(g)) bad |= 2;
      sum += (double)g * (double)g;
    }
  }
  if (!block_finish(sum, bad, partial, s)) return;
  if (threadIdx.x != 0) return;
  const int st = *step;
  const float l = *loss;
  int code = COMMITTED;
  if ((s->bad & 1) || st < 0) code = INVALID_STATE;
  else if (!*acc_valid) code = ACCUMULATION_INVALID;
  else if (!finite(l)) code = NONFINITE_LOSS;
  else if (s->bad & 2) code = NONFINITE_GRADIENT;
  else if (st >= 0x7fffffff) code = STEP_OVERFLOW;
  const float gnorm = (float)sqrt(s->sum);
  const float scale = gnorm == 0.f ? 1.f : fminf(1.f, __fdiv_rn(h.clip, gnorm));
  const float t = (float)((long long)st + 1);
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

// Pass 2 (commit = false): candidate checks and update norm, no writes.
// Pass 3 (commit = true): the same arithmetic, written back when committed.
template <bool COMMIT>
__global__ void __launch_bounds__(THREADS) update_kernel(float* __restrict__ params, float* __restrict__ m,
                                                         float* __restrict__ v, const float* __restrict__ grads,
                                                         long long n_train, long long n_decayed, int* step, Hyper h,
                                                         Scalars* s, Partial* partial, Result* result) {
  const Scalars sc = *s;
  if (sc.code != COMMITTED) return;  // uniform across the grid: no pass election needed
  double sum = 0;
  int bad = 0;
  const long long stride = (long long)gridDim.x * THREADS;
  const long long nt4 = n_train / 4;
  for (long long i = blockIdx.x * (long long)THREADS + threadIdx.x; i < nt4; i += stride) {
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
    if (e < n_train) {
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
  const float unorm = (float)sqrt(s->sum);
  const bool ok = finite(result->gradient_norm) && finite(unorm) && !s->bad;
  result->update_norm = unorm;
  if (!ok) {
    s->code = CANDIDATE_INVALID;
    result->code = CANDIDATE_INVALID;
  }
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
  adamw::check_kernel<<<blocks, adamw::THREADS, 0, s>>>(params, m, v, grads, n_train, n_total, step, loss,
                                                        accumulation_valid, grad_divisor, h, sc, partial, res);
  MFB_LAUNCH_CHECK("adamw check");
  adamw::update_kernel<false><<<blocks, adamw::THREADS, 0, s>>>(params, m, v, grads, n_train, n_decayed, step, h, sc,
                                                                partial, res);
  MFB_LAUNCH_CHECK("adamw candidate");
  adamw::update_kernel<true><<<blocks, adamw::THREADS, 0, s>>>(params, m, v, grads, n_train, n_decayed, step, h, sc,
                                                               partial, res);
  MFB_LAUNCH_CHECK("adamw commit");
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
