// RMSNorm (with a fused residual add and row mask) and per-head q/k RMSNorm +
// rotary embedding, forward and backward, bf16 activations, FP32 statistics.
//
// rms_norm (src/minifield_training/kernels/normalization.py:7-22): the input
// is taken to FP32, scaled by rsqrt(mean(x^2) + eps), cast to bf16 and
// multiplied by the weight cast to bf16 (a bf16 product). The encoder block
// (src/minifield_training/models/lfm2_5/encoder.py:64-110) adds the residual
// in bf16 first (`hidden + residual`), and the conv branch zeroes padded rows
// after the norm (src/minifield_training/layers/convolution.py:29-37); both
// are fused here. project_qkv (layers/attention.py:61-77) RMS-normalizes each
// 64-wide q and k head with its own gain, and apply_rotary (kernels/
// rotary.py:7-39) rotates split halves: out = x*cos + [-x2, x1]*sin with FP32
// angles pos * theta^(-2i/D) and cos/sin cast to bf16, every product and the
// sum rounded to bf16.
//
// Layout: rows of C bf16 values (C a multiple of 256), one warp per row, each
// lane holding C/256 16-byte vectors; per-head kernels use 8 lanes per 64-wide
// head (one 16-byte vector per lane), so a warp covers four heads and the
// rotate-half partner of lane l is lane l ^ 4. Weight gradients are reduced
// per block into FP32 partials, then summed over blocks by a column kernel
// (deterministic, no atomics).
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace mfb {
namespace norm {

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  u.x = pack_bf16(f[0], f[1]);
  u.y = pack_bf16(f[2], f[3]);
  u.z = pack_bf16(f[4], f[5]);
  u.w = pack_bf16(f[6], f[7]);
  return u;
}

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float warp_sum_all(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int WARPS = 8;

// ---- RMSNorm forward -------------------------------------------------------
template <int V>  // 16-byte vectors per lane: C = 256 * V
__global__ void __launch_bounds__(32 * WARPS) rms_fwd_kernel(const uint16_t* __restrict__ x,
                                                             const uint16_t* __restrict__ res,
                                                             const float* __restrict__ w,
                                                             const int32_t* __restrict__ row_mask,
                                                             uint16_t* __restrict__ sum_out, uint16_t* __restrict__ y,
                                                             float* __restrict__ rstd, int M, float eps) {
  allow_dependents();
  constexpr int C = 256 * V;
  const int lane = threadIdx.x & 31;
  const int warp = blockIdx.x * WARPS + (threadIdx.x >> 5), nwarps = gridDim.x * WARPS;
  float wb[V][8];
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) wb[j][e] = bf(w[(j * 32 + lane) * 8 + e]);
  for (int row = warp; row < M; row += nwarps) {
    const long long base = (long long)row * C;
    float v[V][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const long long at = base + (j * 32 + lane) * 8;
      unpack8(*reinterpret_cast<const uint4*>(x + at), v[j]);
      if (res) {
        float r[8];
        unpack8(*reinterpret_cast<const uint4*>(res + at), r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[j][e] = bf(v[j][e] + r[e]);
        *reinterpret_cast<uint4*>(sum_out + at) = pack8(v[j]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[j][e], v[j][e], ss);
    }
    ss = warp_sum_all(ss);
    const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)C), eps));
    const float keep = row_mask ? (row_mask[row] != 0 ? 1.f : 0.f) : 1.f;
    if (rstd && lane == 0) rstd[row] = r;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = bf(bf(v[j][e] * r) * wb[j][e]) * keep;
      *reinterpret_cast<uint4*>(y + base + (j * 32 + lane) * 8) = pack8(o);
    }
  }
}

// ---- RMSNorm backward ------------------------------------------------------
// dx = dres + r * (dn - n * mean(dn * n)), n = x * r, dn = dy' * bf16(w), with
// dy' = dy * mask; per-block partial dw[c] = sum_rows dy' * bf16(n).
template <int V>
__global__ void __launch_bounds__(32 * WARPS) rms_bwd_kernel(const uint16_t* __restrict__ x,
                                                             const float* __restrict__ w,
                                                             const float* __restrict__ rstd,
                                                             const int32_t* __restrict__ row_mask,
                                                             const uint16_t* __restrict__ dy,
                                                             const uint16_t* __restrict__ dres,
                                                             uint16_t* __restrict__ dx, float* __restrict__ partial,
                                                             int M) {
  constexpr int C = 256 * V;
  __shared__ float sdw[WARPS][C];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int warp = blockIdx.x * WARPS + wid, nwarps = gridDim.x * WARPS;
  float wb[V][8], acc[V][8];
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) wb[j][e] = bf(w[(j * 32 + lane) * 8 + e]), acc[j][e] = 0.f;
  for (int row = warp; row < M; row += nwarps) {
    const long long base = (long long)row * C;
    const float r = rstd[row];
    const float keep = row_mask ? (row_mask[row] != 0 ? 1.f : 0.f) : 1.f;
    float n[V][8], dn[V][8];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const long long at = base + (j * 32 + lane) * 8;
      float xv[8], g[8];
      unpack8(*reinterpret_cast<const uint4*>(x + at), xv);
      unpack8(*reinterpret_cast<const uint4*>(dy + at), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        n[j][e] = xv[e] * r;
        const float gm = g[e] * keep;
        dn[j][e] = gm * wb[j][e];
        acc[j][e] = fmaf(gm, bf(n[j][e]), acc[j][e]);
        dot = fmaf(dn[j][e], n[j][e], dot);
      }
    }
    const float mean = warp_sum_all(dot) * (1.f / (float)C);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const long long at = base + (j * 32 + lane) * 8;
      float o[8], d0[8];
      if (dres) unpack8(*reinterpret_cast<const uint4*>(dres + at), d0);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = r * (dn[j][e] - n[j][e] * mean) + (dres ? d0[e] : 0.f);
      *reinterpret_cast<uint4*>(dx + at) = pack8(o);
    }
  }
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) sdw[wid][(j * 32 + lane) * 8 + e] = acc[j][e];
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += 32 * WARPS) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < WARPS; ++k) t += sdw[k][c];
    partial[(long long)blockIdx.x * C + c] = t;
  }
}

// out[c] = sum_b partial[b * ld + c] (+ out[c] when accumulate), c < C.
__global__ void colsum_kernel(const float* __restrict__ partial, int nblocks, int C, int ld, float* __restrict__ out,
                              int accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float t = 0.f;
  for (int b = 0; b < nblocks; ++b) t += partial[(long long)b * ld + c];
  out[c] = accumulate ? out[c] + t : t;
}

// ---- per-head q/k norm + rotary --------------------------------------------
// Lane l of an 8-lane group holds dims [8l, 8l + 8) of one head; l ^ 4 holds
// the rotate-half partner dims.
struct Rope {
  float c[8], s[8];
};

__device__ __forceinline__ Rope rope_at(int pos, const float* freqs, int sub) {
  Rope r;
  const float p = (float)pos;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a = __fmul_rn(p, freqs[(sub * 8 + e) & 31]);
    float sn, cs;
    sincosf(a, &sn, &cs);
    r.c[e] = bf(cs);
    r.s[e] = bf(sn);
  }
  return r;
}

// Forward of one head: x (8 values per lane) -> rotated bf16 output; returns rstd.
__device__ __forceinline__ float head_fwd(float* x, const float* wb, const Rope& rp, int sub, float eps, float* out) {
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  ss += __shfl_xor_sync(0xffffffffu, ss, 2);
  ss += __shfl_xor_sync(0xffffffffu, ss, 4);
  const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, 64.f), eps));
  float n[8], partner[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) n[e] = bf(bf(x[e] * r) * wb[e]);
#pragma unroll
  for (int e = 0; e < 8; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, n[e], 4);
  const bool low = sub < 4;  // dims < 32: rotated = -x2; dims >= 32: rotated = x1
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float rot = low ? -partner[e] : partner[e];
    out[e] = bf(bf(n[e] * rp.c[e]) + bf(rot * rp.s[e]));
  }
  return r;
}

template <int HPW>  // heads per warp = 4
__global__ void __launch_bounds__(256) qk_fwd_kernel(const uint16_t* __restrict__ qkv, int ld, const float* __restrict__ wq,
                                                     const float* __restrict__ wk, const int32_t* __restrict__ positions,
                                                     const float* __restrict__ freqs, uint16_t* __restrict__ q,
                                                     uint16_t* __restrict__ k, uint16_t* __restrict__ v,
                                                     float* __restrict__ rstd_q, float* __restrict__ rstd_k, int M,
                                                     int H, int Hk, float eps) {
  const int lane = threadIdx.x & 31, sub = lane & 7, grp = lane >> 3;
  const int heads = H + 2 * Hk;  // q heads, k heads, v heads
  const long long items = (long long)M * heads;
  const long long gw = (long long)blockIdx.x * 8 + (threadIdx.x >> 5), nw = (long long)gridDim.x * 8;
  for (long long it = gw * HPW + grp; it - grp < items; it += nw * HPW) {
    const bool live = it < items;
    const int row = live ? (int)(it / heads) : 0, hh = live ? (int)(it % heads) : 0;
    float x[8];
    unpack8(*reinterpret_cast<const uint4*>(qkv + (long long)row * ld + hh * 64 + sub * 8), x);
    const bool is_q = hh < H, is_k = !is_q && hh < H + Hk;
    // All lanes take part in the shuffles; v heads are copied through.
    float wb[8];
    const float* w = is_q ? wq : wk;
#pragma unroll
    for (int e = 0; e < 8; ++e) wb[e] = bf(w[sub * 8 + e]);
    const Rope rp = rope_at(positions[row], freqs, sub);
    float out[8];
    const float r = head_fwd(x, wb, rp, sub, eps, out);
    if (!live) continue;
    if (is_q) {
      *reinterpret_cast<uint4*>(q + ((long long)row * H + hh) * 64 + sub * 8) = pack8(out);
      if (sub == 0 && rstd_q) rstd_q[(long long)row * H + hh] = r;
    } else if (is_k) {
      *reinterpret_cast<uint4*>(k + ((long long)row * Hk + hh - H) * 64 + sub * 8) = pack8(out);
      if (sub == 0 && rstd_k) rstd_k[(long long)row * Hk + hh - H] = r;
    } else {
      *reinterpret_cast<uint4*>(v + ((long long)row * Hk + hh - H - Hk) * 64 + sub * 8) =
          *reinterpret_cast<const uint4*>(qkv + (long long)row * ld + hh * 64 + sub * 8);
    }
  }
}

// Backward: d_qkv row = [d(q heads) | d(k heads) | dv]; partial[blk][0..63] wq, [64..127] wk.
__global__ void __launch_bounds__(256) qk_bwd_kernel(const uint16_t* __restrict__ qkv, int ld, const float* __restrict__ wq,
                                                     const float* __restrict__ wk, const int32_t* __restrict__ positions,
                                                     const float* __restrict__ freqs, const float* __restrict__ rstd_q,
                                                     const float* __restrict__ rstd_k, const uint16_t* __restrict__ dq,
                                                     const uint16_t* __restrict__ dk, const uint16_t* __restrict__ dv,
                                                     uint16_t* __restrict__ dqkv, float* __restrict__ partial, int M,
                                                     int H, int Hk) {
  __shared__ float sdw[8][4][128];
  const int lane = threadIdx.x & 31, sub = lane & 7, grp = lane >> 3, wid = threadIdx.x >> 5;
  const int heads = H + 2 * Hk;
  const long long items = (long long)M * heads;
  const long long gw = (long long)blockIdx.x * 8 + wid, nw = (long long)gridDim.x * 8;
  float accq[8], acck[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) accq[e] = acck[e] = 0.f;
  for (long long it = gw * 4 + grp; it - grp < items; it += nw * 4) {
    const bool live = it < items;
    const int row = live ? (int)(it / heads) : 0, hh = live ? (int)(it % heads) : 0;
    const bool is_q = hh < H, is_k = !is_q && hh < H + Hk;
    const long long src = (long long)row * ld + hh * 64 + sub * 8;
    float x[8], g[8];
    unpack8(*reinterpret_cast<const uint4*>(qkv + src), x);
    const uint16_t* gsrc = is_q ? dq + ((long long)row * H + hh) * 64
                                : (is_k ? dk + ((long long)row * Hk + hh - H) * 64 : dv + ((long long)row * Hk + hh - H - Hk) * 64);
    unpack8(*reinterpret_cast<const uint4*>(gsrc + sub * 8), g);
    const Rope rp = rope_at(positions[row], freqs, sub);
    // Through the rotation: dn[j] = g[j] c[j] + (j < 32 ? g[j+32] s[j+32] : -g[j-32] s[j-32]).
    float gs[8], pg[8], dn[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) gs[e] = g[e] * rp.s[e];
#pragma unroll
    for (int e = 0; e < 8; ++e) pg[e] = __shfl_xor_sync(0xffffffffu, gs[e], 4);
    const bool low = sub < 4;
#pragma unroll
    for (int e = 0; e < 8; ++e) dn[e] = g[e] * rp.c[e] + (low ? pg[e] : -pg[e]);
    // Through the head RMSNorm.
    const float r = is_q ? rstd_q[(long long)row * H + hh] : (is_k ? rstd_k[(long long)row * Hk + hh - H] : 0.f);
    const float* w = is_q ? wq : wk;
    float n[8], dnw[8], dot = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      n[e] = x[e] * r;
      dnw[e] = dn[e] * bf(w[sub * 8 + e]);
      dot = fmaf(dnw[e], n[e], dot);
    }
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    dot += __shfl_xor_sync(0xffffffffu, dot, 4);
    const float mean = dot * (1.f / 64.f);
    if (!live) continue;
    if (is_q || is_k) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o[e] = r * (dnw[e] - n[e] * mean);
        if (is_q) accq[e] = fmaf(dn[e], bf(n[e]), accq[e]);
        else acck[e] = fmaf(dn[e], bf(n[e]), acck[e]);
      }
      *reinterpret_cast<uint4*>(dqkv + (long long)row * ld + hh * 64 + sub * 8) = pack8(o);
    } else {
      *reinterpret_cast<uint4*>(dqkv + (long long)row * ld + hh * 64 + sub * 8) =
          *reinterpret_cast<const uint4*>(gsrc + sub * 8);
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    sdw[wid][grp][sub * 8 + e] = accq[e];
    sdw[wid][grp][64 + sub * 8 + e] = acck[e];
  }
  __syncthreads();
  if (threadIdx.x < 128) {
    float t = 0.f;
    for (int a = 0; a < 8; ++a)
      for (int b = 0; b < 4; ++b) t += sdw[a][b][threadIdx.x];
    partial[(long long)blockIdx.x * 128 + threadIdx.x] = t;
  }
}

int grid_for(long long work_items, int per_block, int cap) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long need = (work_items + per_block - 1) / per_block;
  return (int)std::max<long long>(1, std::min<long long>(need, (long long)cap * sms));
}

constexpr int BWD_BLOCKS_PER_SM = 2;  // bounds the partial buffers

}  // namespace norm
}  // namespace mfb

using namespace mfb;

extern "C" size_t mfb_norm_workspace_size(int M, int C) {
  (void)M;
  // Partials for up to BWD_BLOCKS_PER_SM blocks on 160 SMs, C or 128 columns.
  return sizeof(float) * (size_t)norm::BWD_BLOCKS_PER_SM * 160 * (size_t)std::max(C, 128);
}

extern "C" int mfb_rmsnorm_fwd(const uint16_t* x, const uint16_t* residual, const float* weight,
                               const int32_t* row_mask, uint16_t* sum_out, uint16_t* y, float* rstd, int M, int C,
                               float eps, void* stream) {
  MFB_CHECK_ARG(M > 0 && C > 0 && C % 256 == 0 && C <= 2048, "rms_norm supports C a multiple of 256 up to 2048 (C=%d)", C);
  MFB_CHECK_ARG(x && weight && y, "NULL rms_norm argument");
  MFB_CHECK_ARG(!residual || sum_out, "rms_norm with a residual needs sum_out");
  const int grid = norm::grid_for(M, norm::WARPS, 8);
  cudaStream_t s = (cudaStream_t)stream;
  switch (C / 256) {
    case 1: norm::rms_fwd_kernel<1><<<grid, 32 * norm::WARPS, 0, s>>>(x, residual, weight, row_mask, sum_out, y, rstd, M, eps); break;
    case 2: norm::rms_fwd_kernel<2><<<grid, 32 * norm::WARPS, 0, s>>>(x, residual, weight, row_mask, sum_out, y, rstd, M, eps); break;
    case 4: norm::rms_fwd_kernel<4><<<grid, 32 * norm::WARPS, 0, s>>>(x, residual, weight, row_mask, sum_out, y, rstd, M, eps); break;
    case 8: norm::rms_fwd_kernel<8><<<grid, 32 * norm::WARPS, 0, s>>>(x, residual, weight, row_mask, sum_out, y, rstd, M, eps); break;
    default: return set_error(MFB_ERR_UNSUPPORTED, "rms_norm C=%d: supported 256, 512, 1024, 2048", C);
  }
  MFB_LAUNCH_CHECK("rms_norm fwd");
  return MFB_OK;
}

extern "C" int mfb_rmsnorm_bwd(const uint16_t* x, const float* weight, const float* rstd, const int32_t* row_mask,
                               const uint16_t* dy, const uint16_t* dres, uint16_t* dx, float* dweight,
                               int accumulate, int M, int C, void* workspace, size_t workspace_bytes, void* stream) {
  MFB_CHECK_ARG(M > 0 && C > 0 && C % 256 == 0 && C <= 1024, "rms_norm bwd supports C a multiple of 256 up to 1024 (C=%d)",
                C);
  MFB_CHECK_ARG(x && weight && rstd && dy && dx && dweight, "NULL rms_norm bwd argument");
  const int grid = norm::grid_for(M, norm::WARPS * 8, norm::BWD_BLOCKS_PER_SM);
  MFB_CHECK_ARG(workspace && workspace_bytes >= sizeof(float) * (size_t)grid * C, "rms_norm bwd workspace needs %zu bytes",
                sizeof(float) * (size_t)grid * C);
  float* partial = static_cast<float*>(workspace);
  cudaStream_t s = (cudaStream_t)stream;
  switch (C / 256) {
    case 1: norm::rms_bwd_kernel<1><<<grid, 32 * norm::WARPS, 0, s>>>(x, weight, rstd, row_mask, dy, dres, dx, partial, M); break;
    case 2: norm::rms_bwd_kernel<2><<<grid, 32 * norm::WARPS, 0, s>>>(x, weight, rstd, row_mask, dy, dres, dx, partial, M); break;
    case 4: norm::rms_bwd_kernel<4><<<grid, 32 * norm::WARPS, 0, s>>>(x, weight, rstd, row_mask, dy, dres, dx, partial, M); break;
    default: return set_error(MFB_ERR_UNSUPPORTED, "rms_norm bwd C=%d: supported 256, 512, 1024", C);
  }
  MFB_LAUNCH_CHECK("rms_norm bwd");
  norm::colsum_kernel<<<(C + 255) / 256, 256, 0, s>>>(partial, grid, C, C, dweight, accumulate);
  MFB_LAUNCH_CHECK("rms_norm dweight");
  return MFB_OK;
}

extern "C" int mfb_qknorm_rope_fwd(const uint16_t* qkv, int ld_qkv, const float* wq, const float* wk,
                                   const int32_t* positions, const float* freqs, uint16_t* q, uint16_t* k,
                                   uint16_t* v, float* rstd_q, float* rstd_k, int M, int H, int Hk, float eps,
                                   void* stream) {
  MFB_CHECK_ARG(M > 0 && H > 0 && Hk > 0 && ld_qkv >= (H + 2 * Hk) * 64 && ld_qkv % 8 == 0,
                "q/k norm + rope: bad shape (M=%d H=%d Hk=%d ld=%d)", M, H, Hk, ld_qkv);
  MFB_CHECK_ARG(qkv && wq && wk && positions && freqs && q && k && v, "NULL q/k norm + rope argument");
  const long long items = (long long)M * (H + 2 * Hk);
  const int grid = norm::grid_for(items, 32, 8);
  norm::qk_fwd_kernel<4><<<grid, 256, 0, (cudaStream_t)stream>>>(qkv, ld_qkv, wq, wk, positions, freqs, q, k, v,
                                                                 rstd_q, rstd_k, M, H, Hk, eps);
  MFB_LAUNCH_CHECK("q/k norm + rope fwd");
  return MFB_OK;
}

extern "C" int mfb_qknorm_rope_bwd(const uint16_t* qkv, int ld_qkv, const float* wq, const float* wk,
                                   const int32_t* positions, const float* freqs, const float* rstd_q,
                                   const float* rstd_k, const uint16_t* dq, const uint16_t* dk, const uint16_t* dv,
                                   uint16_t* dqkv, float* dwq, float* dwk, int accumulate, int M, int H, int Hk,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  MFB_CHECK_ARG(M > 0 && H > 0 && Hk > 0 && ld_qkv >= (H + 2 * Hk) * 64 && ld_qkv % 8 == 0,
                "q/k norm + rope bwd: bad shape (M=%d H=%d Hk=%d ld=%d)", M, H, Hk, ld_qkv);
  MFB_CHECK_ARG(qkv && wq && wk && positions && freqs && rstd_q && rstd_k && dq && dk && dv && dqkv && dwq && dwk,
                "NULL q/k norm + rope bwd argument");
  const long long items = (long long)M * (H + 2 * Hk);
  const int grid = norm::grid_for(items, 32 * 8, norm::BWD_BLOCKS_PER_SM);
  MFB_CHECK_ARG(workspace && workspace_bytes >= sizeof(float) * 128 * (size_t)grid,
                "q/k norm + rope bwd workspace needs %zu bytes", sizeof(float) * 128 * (size_t)grid);
  float* partial = static_cast<float*>(workspace);
  cudaStream_t s = (cudaStream_t)stream;
  norm::qk_bwd_kernel<<<grid, 256, 0, s>>>(qkv, ld_qkv, wq, wk, positions, freqs, rstd_q, rstd_k, dq, dk, dv, dqkv,
                                           partial, M, H, Hk);
  MFB_LAUNCH_CHECK("q/k norm + rope bwd");
  // Columns 0..63 of each block's partial are wq's, 64..127 wk's.
  norm::colsum_kernel<<<1, 64, 0, s>>>(partial, grid, 64, 128, dwq, accumulate);
  MFB_LAUNCH_CHECK("q norm dweight");
  norm::colsum_kernel<<<1, 64, 0, s>>>(partial + 64, grid, 64, 128, dwk, accumulate);
  MFB_LAUNCH_CHECK("k norm dweight");
  return MFB_OK;
}
