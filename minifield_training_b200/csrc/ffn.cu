// SwiGLU glue between the QAT GEMMs of the feed-forward block
// (src/minifield_training/layers/feed_forward.py:24-35):
//   forward   h = silu(gate) * up
//   backward  d_gate = dh * up * silu'(gate), d_up = dh * silu(gate)
// gu is the gate/up GEMM output [M, 2F] (gate columns first). Elementwise in
// FP32 on bf16 storage, 8 elements per thread with 16-byte accesses.
#include "common.cuh"

namespace mfb {
namespace {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* f) {
  uint4 u;
  u.x = pack_bf16(f[0], f[1]);
  u.y = pack_bf16(f[2], f[3]);
  u.z = pack_bf16(f[4], f[5]);
  u.w = pack_bf16(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float sigmoid(float x) { return 1.f / (1.f + expf(-x)); }

__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h, int M, int F) {
  allow_dependents();
  const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= (long long)M * F) return;
  const long long m = i / F, f = i % F;
  float g[8], u[8], o[8];
  load8(gu + m * 2 * F + f, g);
  load8(gu + m * 2 * F + F + f, u);
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = g[e] * sigmoid(g[e]) * u[e];
  store8(h + i, o);
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu, const __nv_bfloat16* __restrict__ dh,
                                  __nv_bfloat16* __restrict__ dgu, int M, int F) {
  const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= (long long)M * F) return;
  const long long m = i / F, f = i % F;
  float g[8], u[8], d[8], dg[8], du[8];
  load8(gu + m * 2 * F + f, g);
  load8(gu + m * 2 * F + F + f, u);
  load8(dh + i, d);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float s = sigmoid(g[e]);
    du[e] = d[e] * g[e] * s;
    dg[e] = d[e] * u[e] * s * (1.f + g[e] * (1.f - s));
  }
  store8(dgu + m * 2 * F + f, dg);
  store8(dgu + m * 2 * F + F + f, du);
}

}  // namespace
}  // namespace mfb

using namespace mfb;

extern "C" int mfb_swiglu_fwd(const uint16_t* gu, uint16_t* h, int M, int F, void* stream) {
  MFB_CHECK_ARG(M > 0 && F > 0 && F % 8 == 0, "SwiGLU needs M > 0 and F a multiple of 8 (M=%d F=%d)", M, F);
  MFB_CHECK_ARG(gu && h, "NULL tensor argument");
  const long long n = (long long)M * F / 8;
  swiglu_fwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu), reinterpret_cast<__nv_bfloat16*>(h), M, F);
  MFB_LAUNCH_CHECK("mfb_swiglu_fwd");
  return MFB_OK;
}

extern "C" int mfb_swiglu_bwd(const uint16_t* gu, const uint16_t* dh, uint16_t* dgu, int M, int F, void* stream) {
  MFB_CHECK_ARG(M > 0 && F > 0 && F % 8 == 0, "SwiGLU needs M > 0 and F a multiple of 8 (M=%d F=%d)", M, F);
  MFB_CHECK_ARG(gu && dh && dgu, "NULL tensor argument");
  const long long n = (long long)M * F / 8;
  swiglu_bwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu), reinterpret_cast<const __nv_bfloat16*>(dh),
      reinterpret_cast<__nv_bfloat16*>(dgu), M, F);
  MFB_LAUNCH_CHECK("mfb_swiglu_bwd");
  return MFB_OK;
}

namespace mfb {
namespace {
__global__ void cast_f32_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2bfloat16_rn(x[i]);
}
__global__ void add_bf16_kernel(const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b,
                                __nv_bfloat16* __restrict__ out, long long n8) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float x[8], y[8];
  load8(a + 8 * i, x);
  load8(b + 8 * i, y);
#pragma unroll
  for (int e = 0; e < 8; ++e) x[e] += y[e];
  store8(out + 8 * i, x);
}
__global__ void cast_bf16_f32_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ y, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __bfloat162float(x[i]);
}
}  // namespace
}  // namespace mfb

// The master-to-activation-dtype cast of full_linear (kernels/linear.py:11),
// round to nearest even.
extern "C" int mfb_cast_f32_bf16(const float* x, uint16_t* y, long long n, void* stream) {
  MFB_CHECK_ARG(n >= 0 && (n == 0 || (x && y)), "bad cast arguments");
  if (n == 0) return MFB_OK;
  cast_f32_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      x, reinterpret_cast<__nv_bfloat16*>(y), n);
  MFB_LAUNCH_CHECK("mfb_cast_f32_bf16");
  return MFB_OK;
}

// bf16 -> FP32 widening (exact): the `.astype(float32)` of the logits
// (src/minifield_training/models/lfm2_5/model.py:829).
extern "C" int mfb_cast_bf16_f32(const uint16_t* x, float* y, long long n, void* stream) {
  MFB_CHECK_ARG(n >= 0 && (n == 0 || (x && y)), "bad cast arguments");
  if (n == 0) return MFB_OK;
  cast_bf16_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), y, n);
  MFB_LAUNCH_CHECK("mfb_cast_bf16_f32");
  return MFB_OK;
}

// bf16 residual add, each sum rounded to nearest even: the `x + hidden` and
// `x + down(...)` of layers/attention.py:100-108 and layers/feed_forward.py:35.
extern "C" int mfb_add_bf16(const uint16_t* a, const uint16_t* b, uint16_t* out, long long n, void* stream) {
  MFB_CHECK_ARG(n >= 0 && n % 8 == 0, "bf16 add needs n a multiple of 8 (n=%lld)", n);
  MFB_CHECK_ARG(n == 0 || (a && b && out), "NULL add argument");
  MFB_CHECK_ARG(((uintptr_t)a | (uintptr_t)b | (uintptr_t)out) % 16 == 0, "bf16 add needs 16-byte aligned buffers");
  if (n == 0) return MFB_OK;
  const long long n8 = n / 8;
  add_bf16_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(a), reinterpret_cast<const __nv_bfloat16*>(b),
      reinterpret_cast<__nv_bfloat16*>(out), n8);
  MFB_LAUNCH_CHECK("mfb_add_bf16");
  return MFB_OK;
}
