// Fake quantizers (Quantizer.effective) for FP32 masters, bit-exact with the
// reference semantics.
//
// Reference kinds follow src/minifield_training/kernels/quantization.py:
//   _groups :68-79 (absmax per 128-column group, stored as FP16 then widened),
//   _decoded :82-104 (ternary half-away thresholds; NF4 code = number of
//   transitions <= w/scale), _nf4_transitions :46-61.
// The symmetric int8 per-channel / int4 group-128 kinds: scale = absmax/qmax,
// code = clamp(rint_half_even(w/scale), -qmax, qmax), STE mask = clamp inactive,
// zero scale -> code 0 / mask 1 / value 0.
//
// Every division is IEEE correctly rounded (__fdiv_rn) and every product
// __fmul_rn so the results equal the NumPy FP32 restatement bit for bit.
// The weight pass is HBM-bound: one warp per 128-column group with 16-byte
// loads, or one CTA per row for the per-channel kind.
#include <math.h>

#include "common.cuh"

namespace mfb {
namespace {

struct Nf4Table {
  float level[16];
  float transition[15];
};

// The reference's NF4 codebook (quantization.py:25-43), as FP32.
const double kNf4Levels[16] = {-1.0,
                               -0.6961928009986877,
                               -0.5250730514526367,
                               -0.39491748809814453,
                               -0.28444138169288635,
                               -0.18477343022823334,
                               -0.09105003625154495,
                               0.0,
                               0.07958029955625534,
                               0.16093020141124725,
                               0.24611230194568634,
                               0.33791524171829224,
                               0.44070982933044434,
                               0.5626170039176941,
                               0.7229568362236023,
                               1.0};

// First FP32 value at or above each exact midpoint of adjacent levels: the
// midpoint is formed in double from the FP32 levels, rounded to FP32, and
// moved one ulp up when the rounding did not land above it.
Nf4Table make_nf4_table() {
  Nf4Table t;
  for (int i = 0; i < 16; ++i) t.level[i] = (float)kNf4Levels[i];
  for (int i = 0; i < 15; ++i) {
    const double mid = ((double)t.level[i] + (double)t.level[i + 1]) * 0.5;
    float r = (float)mid;
    if ((double)r <= mid) r = nextafterf(r, INFINITY);
    t.transition[i] = r;
  }
  return t;
}

struct QuantOut {
  int8_t* codes;
  float* scales;
  uint8_t* ste;
  float* eff_f32;
  __nv_bfloat16* eff_bf16;
};

// Quantizes one element given its group's absmax. Returns the decoded value.
__device__ __forceinline__ float quantize_one(int kind, float w, float scale, const Nf4Table& nf4, int8_t& code,
                                              uint8_t& ste) {
  if (kind == MFB_QUANT_INT8_CHANNEL || kind == MFB_QUANT_INT4_G128) {
    const float qmax = kind == MFB_QUANT_INT8_CHANNEL ? 127.f : 7.f;
    const float ratio = scale == 0.f ? 0.f : __fdiv_rn(w, scale);
    const float r = rintf(ratio);
    const float c = fminf(fmaxf(r, -qmax), qmax);
    code = (int8_t)c;
    ste = (r == c) ? 1 : 0;
    return __fmul_rn(c, scale);
  }
  ste = 1;  // reference kinds: identity STE (quantization.py:127-129)
  if (kind == MFB_QUANT_TERNARY_G128) {
    const float thr = __fmul_rn(0.5f, scale);
    float v = 0.f;
    if (scale != 0.f) v = (w >= thr) ? 1.f : ((w <= -thr) ? -1.f : 0.f);
    code = (int8_t)v;
    return __fmul_rn(v, scale);
  }
  const float normalized = scale == 0.f ? 0.f : __fdiv_rn(w, scale);
  int c = 0;
#pragma unroll
  for (int i = 0; i < 15; ++i) c += (normalized >= nf4.transition[i]) ? 1 : 0;
  code = (int8_t)c;
  return __fmul_rn(nf4.level[c], scale);
}

__device__ __forceinline__ float group_scale(int kind, float absmax) {
  if (kind == MFB_QUANT_INT8_CHANNEL) return __fdiv_rn(absmax, 127.f);
  if (kind == MFB_QUANT_INT4_G128) return __fdiv_rn(absmax, 7.f);
  return __half2float(__float2half_rn(absmax));  // FP16-stored scale (quantization.py:77-79)
}

// One warp per (row, 128-column group); lane handles 4 consecutive columns.
__global__ void __launch_bounds__(256) fakequant_g128_kernel(const float* __restrict__ w, int kind, int rows,
                                                             int cols, QuantOut out, Nf4Table nf4) {
  const int lane = threadIdx.x & 31;
  const int groups = cols / 128;
  const long long gid = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (gid >= (long long)rows * groups) return;
  const int row = (int)(gid / groups);
  const int grp = (int)(gid % groups);
  const size_t base = (size_t)row * cols + (size_t)grp * 128 + lane * 4;
  const float4 x = *reinterpret_cast<const float4*>(w + base);
  float m = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
  m = warp_max(m);
  const float scale = group_scale(kind, m);
  if (lane == 0 && out.scales) out.scales[(size_t)row * groups + grp] = scale;
  int8_t c[4];
  uint8_t s[4];
  float e[4];
  e[0] = quantize_one(kind, x.x, scale, nf4, c[0], s[0]);
  e[1] = quantize_one(kind, x.y, scale, nf4, c[1], s[1]);
  e[2] = quantize_one(kind, x.z, scale, nf4, c[2], s[2]);
  e[3] = quantize_one(kind, x.w, scale, nf4, c[3], s[3]);
  if (out.codes) *reinterpret_cast<char4*>(out.codes + base) = make_char4(c[0], c[1], c[2], c[3]);
  if (out.ste) *reinterpret_cast<uchar4*>(out.ste + base) = make_uchar4(s[0], s[1], s[2], s[3]);
  if (out.eff_f32) *reinterpret_cast<float4*>(out.eff_f32 + base) = make_float4(e[0], e[1], e[2], e[3]);
  if (out.eff_bf16) {
    uint2 p;
    p.x = pack_bf16(e[0], e[1]);
    p.y = pack_bf16(e[2], e[3]);
    *reinterpret_cast<uint2*>(out.eff_bf16 + base) = p;
  }
}

// One CTA per row (per-output-channel scale over any number of columns).
// VEC4: cols % 4 == 0 and every buffer aligned for 4-column vectors.
template <bool VEC4>
__global__ void __launch_bounds__(256) fakequant_channel_kernel(const float* __restrict__ w, int kind, int rows,
                                                                int cols, QuantOut out, Nf4Table nf4) {
  __shared__ float red[8];
  const int row = blockIdx.x;
  const float* wr = w + (size_t)row * cols;
  float m = 0.f;
  if constexpr (VEC4) {
    for (int c = 4 * threadIdx.x; c < cols; c += 4 * blockDim.x) {
      const float4 x = *reinterpret_cast<const float4*>(wr + c);
      m = fmaxf(fmaxf(m, fmaxf(fabsf(x.x), fabsf(x.y))), fmaxf(fabsf(x.z), fabsf(x.w)));
    }
  } else {
    for (int c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, fabsf(wr[c]));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float scale = group_scale(kind, red[0]);
  if (threadIdx.x == 0 && out.scales) out.scales[row] = scale;
  if constexpr (VEC4) {
    // Four consecutive columns per thread: one 16-byte load and one store per
    // output (4 codes, 4 mask bytes, 8 bytes of bf16, 16 of FP32).
    const size_t i0 = (size_t)row * cols;
    for (int c = 4 * threadIdx.x; c < cols; c += 4 * blockDim.x) {
      const float4 x = *reinterpret_cast<const float4*>(wr + c);
      const float xs[4] = {x.x, x.y, x.z, x.w};
      float e[4];
      uint32_t codes = 0, stes = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        int8_t code;
        uint8_t ste;
        e[k] = quantize_one(kind, xs[k], scale, nf4, code, ste);
        codes |= (uint32_t)(uint8_t)code << (8 * k);
        stes |= (uint32_t)ste << (8 * k);
      }
      if (out.codes) *reinterpret_cast<uint32_t*>(out.codes + i0 + c) = codes;
      if (out.ste) *reinterpret_cast<uint32_t*>(out.ste + i0 + c) = stes;
      if (out.eff_f32) *reinterpret_cast<float4*>(out.eff_f32 + i0 + c) = make_float4(e[0], e[1], e[2], e[3]);
      if (out.eff_bf16) {
        uint2 p;
        p.x = pack_bf16(e[0], e[1]);
        p.y = pack_bf16(e[2], e[3]);
        *reinterpret_cast<uint2*>(out.eff_bf16 + i0 + c) = p;
      }
    }
  } else {
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      int8_t code;
      uint8_t ste;
      const float e = quantize_one(kind, wr[c], scale, nf4, code, ste);
      const size_t i = (size_t)row * cols + c;
      if (out.codes) out.codes[i] = code;
      if (out.ste) out.ste[i] = ste;
      if (out.eff_f32) out.eff_f32[i] = e;
      if (out.eff_bf16) out.eff_bf16[i] = __float2bfloat16_rn(e);
    }
  }
}

const Nf4Table& nf4_table() {
  static const Nf4Table t = make_nf4_table();
  return t;
}

}  // namespace
}  // namespace mfb

extern "C" int mfb_fakequant(const float* w, int kind, int rows, int cols, int8_t* codes, float* scales,
                             uint8_t* ste, float* eff_f32, uint16_t* eff_bf16, void* stream) {
  using namespace mfb;
  MFB_CHECK_ARG(kind >= MFB_QUANT_INT8_CHANNEL && kind <= MFB_QUANT_NF4_G128, "Unknown quantizer kind %d", kind);
  MFB_CHECK_ARG(rows > 0 && cols > 0, "Quantized matrix requires rank 2 and a nonempty shape (%d, %d)", rows, cols);
  MFB_CHECK_ARG(kind == MFB_QUANT_INT8_CHANNEL || cols % 128 == 0,
                "Quantized matrix requires rank 2 and K divisible by 128 (K=%d)", cols);
  MFB_CHECK_ARG(w != nullptr, "weight is NULL");
  QuantOut out{codes, scales, ste, eff_f32, reinterpret_cast<__nv_bfloat16*>(eff_bf16)};
  cudaStream_t s = (cudaStream_t)stream;
  if (kind == MFB_QUANT_INT8_CHANNEL) {
    const bool vec4 = cols % 4 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(codes) & 3) == 0 && (reinterpret_cast<uintptr_t>(ste) & 3) == 0 &&
                      (reinterpret_cast<uintptr_t>(eff_f32) & 15) == 0 && (reinterpret_cast<uintptr_t>(eff_bf16) & 7) == 0;
    if (vec4)
      fakequant_channel_kernel<true><<<rows, 256, 0, s>>>(w, kind, rows, cols, out, nf4_table());
    else
      fakequant_channel_kernel<false><<<rows, 256, 0, s>>>(w, kind, rows, cols, out, nf4_table());
  } else {
    MFB_CHECK_ARG((reinterpret_cast<uintptr_t>(w) & 15) == 0, "weight must be 16-byte aligned");
    const long long groups = (long long)rows * (cols / 128);
    const long long blocks = (groups + 7) / 8;
    MFB_CHECK_ARG(blocks < (1LL << 31), "matrix too large");
    fakequant_g128_kernel<<<(unsigned)blocks, 256, 0, s>>>(w, kind, rows, cols, out, nf4_table());
  }
  MFB_LAUNCH_CHECK("mfb_fakequant");
  return MFB_OK;
}
