// Encoder-step glue kernels: frozen embedding gather, the gated centered
// short convolution (forward and backward), and the token classification
// head with its summed cross-entropy (forward and backward in one pass).
//
// Embedding: encode() reads params["lfm2.embed_tokens.weight"][ids] and casts
// to bf16 (src/minifield_training/models/lfm2_5/encoder.py:231); JAX clamps
// out-of-range gather indices, so ids are clamped to [0, V).
//
// Convolution branch (encoder.py:76-86, layers/convolution.py:29-37,
// kernels/bidirectional.py:38-58): the in-projection output splits into
// b, c, values (thirds of the row); gated = b * values (bf16);
// conv[t] = sum over taps i = 0, 1, 2 of gated[t + i - 1] * bf16(taps[:, i]),
// each tap product rounded to bf16, zeroed unless the neighbour is in the
// token's own nonzero segment (row edges count as padding), and accumulated
// in bf16 in tap order; mixed = c * conv (bf16).
//
// Layout: rows of the packed [B*T] token axis; a thread owns one 8-channel
// (16-byte) chunk and walks TOK consecutive tokens, keeping a three-row
// window in registers, so each row is read once plus a one-row halo per group.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace mfb {
namespace enc {

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

// ---- embedding gather -------------------------------------------------------
__global__ void embed_kernel(const float* __restrict__ table, const int32_t* __restrict__ ids, uint16_t* __restrict__ out,
                             long long M, int C, int V) {
  const int chunks = C / 8;
  const long long total = M * chunks;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / chunks;
    const int ch = (int)(i % chunks);
    const int id = min(max(ids[row], 0), V - 1);
    const float4 a = *reinterpret_cast<const float4*>(table + (long long)id * C + ch * 8);
    const float4 b = *reinterpret_cast<const float4*>(table + (long long)id * C + ch * 8 + 4);
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    *reinterpret_cast<uint4*>(out + row * C + ch * 8) = pack8(f);
  }
}

// ---- gated centered convolution ----------------------------------------------
constexpr int TOK = 32;  // tokens walked per thread

struct Row {
  float b[8], c[8], x[8];
};

__device__ __forceinline__ void load_row(const uint16_t* bcx, int C, long long row, int ch, Row& r) {
  const uint16_t* base = bcx + row * 3 * C + ch * 8;
  unpack8(*reinterpret_cast<const uint4*>(base), r.b);
  unpack8(*reinterpret_cast<const uint4*>(base + C), r.c);
  unpack8(*reinterpret_cast<const uint4*>(base + 2 * C), r.x);
}

// Tap contribution in the reference's rounding order for token t from neighbour p.
__device__ __forceinline__ void conv_at(const float* gm, const float* g0, const float* gp, const float* tb, bool sm,
                                        bool s0, bool sp, float* out) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float t0 = sm ? bf(gm[e] * tb[e * 3 + 0]) : 0.f;
    const float t1 = s0 ? bf(g0[e] * tb[e * 3 + 1]) : 0.f;
    const float t2 = sp ? bf(gp[e] * tb[e * 3 + 2]) : 0.f;
    out[e] = bf(bf(t0 + t1) + t2);
  }
}

// One decode step of the causal gated short convolution
// (kernels/convolution.py:82-111 via layers/convolution.py:153-178): window =
// [history oldest .. newest, b * values] of one token per row, mixed = c *
// sum_k window_k * tap_k (taps rounded to bf16, each product and partial sum
// rounded as in conv_at), and the history shifts by one with this step's
// gated input. In place on the history: every element is read before it is
// written by the same thread.
__global__ void conv_step_kernel(const uint16_t* __restrict__ bcx, const float* __restrict__ taps,
                                 uint16_t* __restrict__ hist, uint16_t* __restrict__ mixed, int B, int C) {
  allow_dependents();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * C) return;
  const int b = (int)(i / C), ch = (int)(i % C);
  auto ld = [](const uint16_t* p) { return __bfloat162float(__ushort_as_bfloat16(*p)); };
  const uint16_t* row = bcx + (long long)b * 3 * C;
  const float g = bf(ld(row + ch) * ld(row + 2 * C + ch));
  uint16_t* h = hist + (long long)b * 2 * C + ch;
  const float h0 = ld(h), h1 = ld(h + C);
  const float t0 = bf(h0 * bf(taps[ch * 3 + 0])), t1 = bf(h1 * bf(taps[ch * 3 + 1]));
  const float t2 = bf(g * bf(taps[ch * 3 + 2]));
  const float acc = bf(bf(t0 + t1) + t2);
  mixed[i] = __bfloat16_as_ushort(__float2bfloat16_rn(ld(row + C + ch) * acc));
  h[0] = h[C];
  h[C] = __bfloat16_as_ushort(__float2bfloat16_rn(g));
}

// Causal gated short convolution over a whole prompt of T tokens per row
// (kernels/convolution.py:7-22 for a zero history, :82-111 with one), plus the
// continuation history of layers/convolution.py:77-101 (state_tail at the row's
// full length: the last two gated inputs, zeros or the incoming history where
// the row is shorter). One thread per (row, chunk of CAUSAL_TOK tokens,
// channel): channels are the fastest index, so a warp reads 64 contiguous bytes
// of each of b, c and values per token. Rounding as conv_step_kernel.
constexpr int CAUSAL_TOK = 32;

__global__ void conv_causal_kernel(const uint16_t* __restrict__ bcx, const float* __restrict__ taps,
                                   const uint16_t* __restrict__ hist_in, uint16_t* __restrict__ hist_out,
                                   uint16_t* __restrict__ mixed, int B, int T, int C) {
  const int chunks = (T + CAUSAL_TOK - 1) / CAUSAL_TOK;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * chunks * C) return;
  const int ch = (int)(i % C);
  const long long bk = i / C;
  const int k = (int)(bk % chunks), b = (int)(bk / chunks);
  auto ld = [](const uint16_t* p) { return __bfloat162float(__ushort_as_bfloat16(*p)); };
  const uint16_t* rows = bcx + (long long)b * T * 3 * C;
  // Gated input at token t of this row; t in {-2, -1} reads the incoming history.
  auto gated = [&](int t) -> float {
    if (t >= 0) return bf(ld(rows + (long long)t * 3 * C + ch) * ld(rows + (long long)t * 3 * C + 2 * C + ch));
    return hist_in ? ld(hist_in + ((long long)b * 2 + 2 + t) * C + ch) : 0.f;
  };
  const float w0 = bf(taps[ch * 3 + 0]), w1 = bf(taps[ch * 3 + 1]), w2 = bf(taps[ch * 3 + 2]);
  const int t0 = k * CAUSAL_TOK, t1 = min(T, t0 + CAUSAL_TOK);
  float h0 = gated(t0 - 2), h1 = gated(t0 - 1);
  for (int t = t0; t < t1; ++t) {
    const float g = gated(t);
    const float acc = bf(bf(bf(h0 * w0) + bf(h1 * w1)) + bf(g * w2));
    mixed[((long long)b * T + t) * C + ch] =
        __bfloat16_as_ushort(__float2bfloat16_rn(ld(rows + (long long)t * 3 * C + C + ch) * acc));
    h0 = h1;
    h1 = g;
  }
  if (hist_out && t1 == T) {
    hist_out[(long long)b * 2 * C + ch] = __bfloat16_as_ushort(__float2bfloat16_rn(h0));
    hist_out[((long long)b * 2 + 1) * C + ch] = __bfloat16_as_ushort(__float2bfloat16_rn(h1));
  }
}

__global__ void __launch_bounds__(128) conv_fwd_kernel(const uint16_t* __restrict__ bcx, const float* __restrict__ taps,
                                                       const int32_t* __restrict__ seg, uint16_t* __restrict__ mixed,
                                                       long long M, int T, int C) {
  const int chunks = C / 8;
  const long long groups = (M + TOK - 1) / TOK;
  for (long long w = blockIdx.x * (long long)blockDim.x + threadIdx.x; w < groups * chunks;
       w += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(w % chunks);
    const long long t0 = (w / chunks) * TOK;
    float tb[24];
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
      for (int i = 0; i < 3; ++i) tb[e * 3 + i] = bf(taps[(ch * 8 + e) * 3 + i]);
    // Window: gated at t-1, t, t+1 and their segment ids.
    float gm[8] = {0}, g0[8], gp[8] = {0};
    Row cur, nxt;
    int sm_id = 0, s0_id, sp_id = 0;
    const bool has_prev = (t0 % T) != 0;
    if (has_prev) {
      Row prev;
      load_row(bcx, C, t0 - 1, ch, prev);
#pragma unroll
      for (int e = 0; e < 8; ++e) gm[e] = bf(prev.b[e] * prev.x[e]);
      sm_id = seg[t0 - 1];
    }
    load_row(bcx, C, t0, ch, cur);
#pragma unroll
    for (int e = 0; e < 8; ++e) g0[e] = bf(cur.b[e] * cur.x[e]);
    s0_id = seg[t0];
    for (int k = 0; k < TOK && t0 + k < M; ++k) {
      const long long t = t0 + k;
      const bool first = (t % T) == 0, last = (t % T) == T - 1 || t + 1 >= M;
      // The next row is loaded even across a row end: it is the next token's
      // own row; `last` only masks it as a neighbour.
      if (t + 1 < M) {
        load_row(bcx, C, t + 1, ch, nxt);
#pragma unroll
        for (int e = 0; e < 8; ++e) gp[e] = bf(nxt.b[e] * nxt.x[e]);
        sp_id = seg[t + 1];
      }
      const bool live = s0_id != 0;
      float conv[8], o[8];
      conv_at(gm, g0, gp, tb, live && !first && sm_id == s0_id, live, live && !last && sp_id == s0_id, conv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = bf(cur.c[e] * conv[e]);
      *reinterpret_cast<uint4*>(mixed + t * C + ch * 8) = pack8(o);
#pragma unroll
      for (int e = 0; e < 8; ++e) gm[e] = g0[e], g0[e] = gp[e];
      cur = nxt;
      sm_id = s0_id;
      s0_id = sp_id;
    }
  }
}

// Backward: d_conv[t] = d_mixed[t] * c[t]; d_c[t] = d_mixed[t] * conv[t];
// d_gated[p] = sum_i d_conv[p - i + 1] * tap_i * same(p, p - i + 1);
// d_b = d_gated * values, d_values = d_gated * b; d_tap_i += d_conv[t] * gated[t + i - 1] * same.
__global__ void __launch_bounds__(128) conv_bwd_kernel(const uint16_t* __restrict__ bcx, const float* __restrict__ taps,
                                                       const int32_t* __restrict__ seg,
                                                       const uint16_t* __restrict__ dmixed, uint16_t* __restrict__ dbcx,
                                                       float* __restrict__ partial, long long M, int T, int C) {
  const int chunks = C / 8;
  const long long groups = (M + TOK - 1) / TOK;
  float acc[24];
#pragma unroll
  for (int j = 0; j < 24; ++j) acc[j] = 0.f;
  // Blocks own fixed channel chunks (blockDim.x == chunks or a divisor) so the
  // tap partials of a thread stay in one column range.
  const int ch = threadIdx.x % chunks;
  for (long long gidx = blockIdx.x * (long long)(blockDim.x / chunks) + threadIdx.x / chunks; gidx < groups;
       gidx += (long long)gridDim.x * (blockDim.x / chunks)) {
    const long long t0 = gidx * TOK;
    float tb[24];
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
      for (int i = 0; i < 3; ++i) tb[e * 3 + i] = bf(taps[(ch * 8 + e) * 3 + i]);
    // Window rows t-1, t, t+1: gated, d_conv, segment ids.
    float gm[8] = {0}, g0[8], gp[8] = {0}, dcm[8] = {0}, dc0[8], dcp[8] = {0};
    Row cur, nxt;
    int sm_id = 0, s0_id, sp_id = 0;
    if ((t0 % T) != 0) {
      Row prev;
      float dmv[8];
      load_row(bcx, C, t0 - 1, ch, prev);
      unpack8(*reinterpret_cast<const uint4*>(dmixed + (t0 - 1) * C + ch * 8), dmv);
#pragma unroll
      for (int e = 0; e < 8; ++e) gm[e] = bf(prev.b[e] * prev.x[e]), dcm[e] = dmv[e] * prev.c[e];
      sm_id = seg[t0 - 1];
    }
    {
      float dmv[8];
      load_row(bcx, C, t0, ch, cur);
      unpack8(*reinterpret_cast<const uint4*>(dmixed + t0 * C + ch * 8), dmv);
#pragma unroll
      for (int e = 0; e < 8; ++e) g0[e] = bf(cur.b[e] * cur.x[e]), dc0[e] = dmv[e] * cur.c[e];
      s0_id = seg[t0];
    }
    for (int k = 0; k < TOK && t0 + k < M; ++k) {
      const long long t = t0 + k;
      const bool first = (t % T) == 0, last = (t % T) == T - 1 || t + 1 >= M;
      float dmv0[8];
      unpack8(*reinterpret_cast<const uint4*>(dmixed + t * C + ch * 8), dmv0);
      if (t + 1 < M) {  // the next token's own row, masked as a neighbour when `last`
        float dmv[8];
        load_row(bcx, C, t + 1, ch, nxt);
        unpack8(*reinterpret_cast<const uint4*>(dmixed + (t + 1) * C + ch * 8), dmv);
#pragma unroll
        for (int e = 0; e < 8; ++e) gp[e] = bf(nxt.b[e] * nxt.x[e]), dcp[e] = dmv[e] * nxt.c[e];
        sp_id = seg[t + 1];
      }
      // Taps seen by token t (its own validity) and by its neighbours (theirs).
      const bool live0 = s0_id != 0;
      const bool use_m = live0 && !first && sm_id == s0_id;  // t reads t-1
      const bool use_p = live0 && !last && sp_id == s0_id;   // t reads t+1
      const bool m_reads = !first && sm_id != 0 && sm_id == s0_id;  // t-1 reads t via tap 2
      const bool p_reads = !last && sp_id != 0 && sp_id == s0_id;   // t+1 reads t via tap 0
      float conv[8], dc[8], dg[8];
      conv_at(gm, g0, gp, tb, use_m, live0, use_p, conv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        dc[e] = dmv0[e] * conv[e];
        dg[e] = (live0 ? dc0[e] * tb[e * 3 + 1] : 0.f) + (m_reads ? dcm[e] * tb[e * 3 + 2] : 0.f) +
                (p_reads ? dcp[e] * tb[e * 3 + 0] : 0.f);
        if (use_m) acc[e * 3 + 0] = fmaf(dc0[e], gm[e], acc[e * 3 + 0]);
        if (live0) acc[e * 3 + 1] = fmaf(dc0[e], g0[e], acc[e * 3 + 1]);
        if (use_p) acc[e * 3 + 2] = fmaf(dc0[e], gp[e], acc[e * 3 + 2]);
      }
      float db[8], dx[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) db[e] = dg[e] * cur.x[e], dx[e] = dg[e] * cur.b[e];
      uint16_t* out = dbcx + t * 3 * C + ch * 8;
      *reinterpret_cast<uint4*>(out) = pack8(db);
      *reinterpret_cast<uint4*>(out + C) = pack8(dc);
      *reinterpret_cast<uint4*>(out + 2 * C) = pack8(dx);
#pragma unroll
      for (int e = 0; e < 8; ++e) gm[e] = g0[e], g0[e] = gp[e], dcm[e] = dc0[e], dc0[e] = dcp[e];
      cur = nxt;
      sm_id = s0_id;
      s0_id = sp_id;
    }
  }
  // Per-block tap partials [C][3]: threads with the same chunk add up via shared memory.
  __shared__ float sacc[128][24];
#pragma unroll
  for (int j = 0; j < 24; ++j) sacc[threadIdx.x][j] = acc[j];
  __syncthreads();
  for (int idx = threadIdx.x; idx < chunks * 24; idx += blockDim.x) {
    const int c = idx / 24, j = idx % 24;
    float t = 0.f;
    for (int k = c; k < (int)blockDim.x; k += chunks) t += sacc[k][j];
    partial[(long long)blockIdx.x * C * 3 + c * 24 + j] = t;
  }
}

__global__ void colsum_kernel(const float* __restrict__ partial, int nblocks, int n, float* __restrict__ out,
                              int accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  float t = 0.f;
  for (int b = 0; b < nblocks; ++b) t += partial[(long long)b * n + c];
  out[c] = accumulate ? out[c] + t : t;
}

// ---- classification head + cross-entropy ---------------------------------------
// One warp per token row of C = 1024 (4 vectors per lane); K <= 4 classes.
// logits = bf16(e . bf16(W_k)); loss += lse(logits) - logits[y] on valid rows;
// d_logits = bf16((softmax - onehot) * valid); d_e = bf16(sum_k d_logit_k bf16(W_k));
// partial dW_k[c] += d_logit_k * e[c].
template <int K>
__global__ void __launch_bounds__(256) head_kernel(const uint16_t* __restrict__ e, const float* __restrict__ w,
                                                   const int32_t* __restrict__ labels,
                                                   const int32_t* __restrict__ valid, uint16_t* __restrict__ de,
                                                   float* __restrict__ partial_w, float* __restrict__ partial_loss,
                                                   int M, int C) {
  constexpr int V = 4;  // C == 1024
  __shared__ float sred[8][2];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float wb[K][V][8], acc[K][V][8];
#pragma unroll
  for (int k = 0; k < K; ++k)
#pragma unroll
    for (int j = 0; j < V; ++j)
#pragma unroll
      for (int q = 0; q < 8; ++q) wb[k][j][q] = bf(w[k * C + (j * 32 + lane) * 8 + q]), acc[k][j][q] = 0.f;
  float loss = 0.f, count = 0.f;
  for (int row = blockIdx.x * 8 + wid; row < M; row += gridDim.x * 8) {
    float x[V][8];
    float dot[K];
#pragma unroll
    for (int k = 0; k < K; ++k) dot[k] = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      unpack8(*reinterpret_cast<const uint4*>(e + (long long)row * C + (j * 32 + lane) * 8), x[j]);
#pragma unroll
      for (int k = 0; k < K; ++k)
#pragma unroll
        for (int q = 0; q < 8; ++q) dot[k] = fmaf(x[j][q], wb[k][j][q], dot[k]);
    }
    float lg[K], mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < K; ++k) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot[k] += __shfl_xor_sync(0xffffffffu, dot[k], o);
      lg[k] = bf(dot[k]);
      mx = fmaxf(mx, lg[k]);
    }
    float se = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) se += expf(lg[k] - mx);
    const int y = min(max(labels[row], 0), K - 1);
    const bool ok = valid[row] != 0;
    float dl[K];
#pragma unroll
    for (int k = 0; k < K; ++k) dl[k] = ok ? bf(expf(lg[k] - mx) / se - (k == y ? 1.f : 0.f)) : 0.f;
    if (ok) {
      loss += mx + logf(se) - lg[y];
      count += 1.f;
    }
#pragma unroll
    for (int j = 0; j < V; ++j) {
      float o[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float t = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) {
          t = fmaf(dl[k], wb[k][j][q], t);
          acc[k][j][q] = fmaf(dl[k], x[j][q], acc[k][j][q]);
        }
        o[q] = t;
      }
      *reinterpret_cast<uint4*>(de + (long long)row * C + (j * 32 + lane) * 8) = pack8(o);
    }
  }
  // Reduce the dW accumulators across the 8 warps column by column.
  __shared__ float scol[K][1024];
  for (int idx = threadIdx.x; idx < K * C; idx += 256) scol[idx / C][idx % C] = 0.f;
  __syncthreads();
  for (int wv = 0; wv < 8; ++wv) {
    if (wid == wv) {
#pragma unroll
      for (int k = 0; k < K; ++k)
#pragma unroll
        for (int j = 0; j < V; ++j)
#pragma unroll
          for (int q = 0; q < 8; ++q) scol[k][(j * 32 + lane) * 8 + q] += acc[k][j][q];
    }
    __syncthreads();
  }
  for (int idx = threadIdx.x; idx < K * C; idx += 256)
    partial_w[(long long)blockIdx.x * K * C + idx] = scol[idx / C][idx % C];
  if (lane == 0) sred[wid][0] = loss, sred[wid][1] = count;
  __syncthreads();
  if (threadIdx.x == 0) {
    float l = 0.f, c = 0.f;
    for (int k = 0; k < 8; ++k) l += sred[k][0], c += sred[k][1];
    partial_loss[2 * blockIdx.x] = l;
    partial_loss[2 * blockIdx.x + 1] = c;
  }
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

constexpr int CONV_BWD_BLOCKS_PER_SM = 2;
constexpr int HEAD_BLOCKS_PER_SM = 1;

}  // namespace enc
}  // namespace mfb

using namespace mfb;

extern "C" int mfb_embed_gather(const float* table, const int32_t* ids, uint16_t* out, long long M, int C, int V,
                                void* stream) {
  MFB_CHECK_ARG(M > 0 && C > 0 && C % 8 == 0 && V > 0, "embedding gather: bad shape (M=%lld C=%d V=%d)", M, C, V);
  MFB_CHECK_ARG(table && ids && out && ((uintptr_t)table & 15) == 0, "embedding gather: NULL or unaligned argument");
  const int grid = 8 * enc::sm_count();
  enc::embed_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(table, ids, out, M, C, V);
  MFB_LAUNCH_CHECK("embedding gather");
  return MFB_OK;
}

extern "C" int mfb_conv_fwd(const uint16_t* bcx, const float* taps, const int32_t* segment_ids, uint16_t* mixed,
                            long long M, int T, int C, void* stream) {
  MFB_CHECK_ARG(M > 0 && T > 0 && M % T == 0 && C > 0 && C % 8 == 0 && C <= 8 * 128,
                "gated conv: bad shape (M=%lld T=%d C=%d)", M, T, C);
  MFB_CHECK_ARG(bcx && taps && segment_ids && mixed, "NULL gated conv argument");
  const long long work = (M + enc::TOK - 1) / enc::TOK * (C / 8);
  const int grid = (int)std::min<long long>((work + 127) / 128, 16LL * enc::sm_count());
  enc::conv_fwd_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>(bcx, taps, segment_ids, mixed, M, T, C);
  MFB_LAUNCH_CHECK("gated conv fwd");
  return MFB_OK;
}

extern "C" int mfb_conv_step(const uint16_t* bcx, const float* taps, uint16_t* history, uint16_t* mixed, int B,
                             int C, void* stream) {
  MFB_CHECK_ARG(B > 0 && C > 0, "conv step: bad shape (B=%d C=%d)", B, C);
  MFB_CHECK_ARG(bcx && taps && history && mixed, "NULL conv step argument");
  const long long n = (long long)B * C;
  enc::conv_step_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(bcx, taps, history, mixed, B,
                                                                                        C);
  MFB_LAUNCH_CHECK("conv step");
  return MFB_OK;
}

extern "C" int mfb_conv_causal(const uint16_t* bcx, const float* taps, const uint16_t* history_in,
                               uint16_t* history_out, uint16_t* mixed, int B, int T, int C, void* stream) {
  MFB_CHECK_ARG(B > 0 && T > 0 && C > 0, "causal conv: bad shape (B=%d T=%d C=%d)", B, T, C);
  MFB_CHECK_ARG(bcx && taps && mixed, "NULL causal conv argument");
  MFB_CHECK_ARG(history_out == nullptr || history_out != history_in,
                "causal conv: history_out must not alias history_in");
  const long long n = (long long)B * ((T + enc::CAUSAL_TOK - 1) / enc::CAUSAL_TOK) * C;
  enc::conv_causal_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      bcx, taps, history_in, history_out, mixed, B, T, C);
  MFB_LAUNCH_CHECK("causal conv");
  return MFB_OK;
}

extern "C" size_t mfb_encoder_workspace_size(int C, int classes) {
  const size_t conv = sizeof(float) * (size_t)enc::CONV_BWD_BLOCKS_PER_SM * 160 * 3 * (size_t)C;
  const size_t head = sizeof(float) * (size_t)enc::HEAD_BLOCKS_PER_SM * 160 * ((size_t)classes * C + 2);
  return std::max(conv, head);
}

extern "C" int mfb_conv_bwd(const uint16_t* bcx, const float* taps, const int32_t* segment_ids, const uint16_t* dmixed,
                            uint16_t* dbcx, float* dtaps, int accumulate, long long M, int T, int C, void* workspace,
                            size_t workspace_bytes, void* stream) {
  MFB_CHECK_ARG(M > 0 && T > 0 && M % T == 0 && C > 0 && C % 8 == 0 && C / 8 <= 128 && 128 % (C / 8) == 0,
                "gated conv bwd: bad shape (M=%lld T=%d C=%d)", M, T, C);
  MFB_CHECK_ARG(bcx && taps && segment_ids && dmixed && dbcx && dtaps, "NULL gated conv bwd argument");
  const int grid = enc::CONV_BWD_BLOCKS_PER_SM * enc::sm_count();
  MFB_CHECK_ARG(workspace && workspace_bytes >= sizeof(float) * (size_t)grid * 3 * C,
                "gated conv bwd workspace needs %zu bytes", sizeof(float) * (size_t)grid * 3 * C);
  float* partial = static_cast<float*>(workspace);
  cudaStream_t s = (cudaStream_t)stream;
  enc::conv_bwd_kernel<<<grid, 128, 0, s>>>(bcx, taps, segment_ids, dmixed, dbcx, partial, M, T, C);
  MFB_LAUNCH_CHECK("gated conv bwd");
  enc::colsum_kernel<<<(3 * C + 255) / 256, 256, 0, s>>>(partial, grid, 3 * C, dtaps, accumulate);
  MFB_LAUNCH_CHECK("gated conv dtaps");
  return MFB_OK;
}

extern "C" int mfb_head_loss(const uint16_t* encoded, const float* weight, const int32_t* labels, const int32_t* valid,
                             uint16_t* d_encoded, float* d_weight, float* loss_count, int M, int C, int classes,
                             void* workspace, size_t workspace_bytes, void* stream) {
  MFB_CHECK_ARG(M > 0 && C == 1024 && classes >= 1 && classes <= 4, "head: supports C=1024 and 1..4 classes (C=%d K=%d)",
                C, classes);
  MFB_CHECK_ARG(encoded && weight && labels && valid && d_encoded && d_weight && loss_count, "NULL head argument");
  const int grid = enc::HEAD_BLOCKS_PER_SM * enc::sm_count();
  const size_t need = sizeof(float) * (size_t)grid * ((size_t)classes * C + 2);
  MFB_CHECK_ARG(workspace && workspace_bytes >= need, "head workspace needs %zu bytes", need);
  float* pw = static_cast<float*>(workspace);
  float* pl = pw + (size_t)grid * classes * C;
  cudaStream_t s = (cudaStream_t)stream;
  switch (classes) {
    case 1: enc::head_kernel<1><<<grid, 256, 0, s>>>(encoded, weight, labels, valid, d_encoded, pw, pl, M, C); break;
    case 2: enc::head_kernel<2><<<grid, 256, 0, s>>>(encoded, weight, labels, valid, d_encoded, pw, pl, M, C); break;
    case 3: enc::head_kernel<3><<<grid, 256, 0, s>>>(encoded, weight, labels, valid, d_encoded, pw, pl, M, C); break;
    default: enc::head_kernel<4><<<grid, 256, 0, s>>>(encoded, weight, labels, valid, d_encoded, pw, pl, M, C); break;
  }
  MFB_LAUNCH_CHECK("head");
  enc::colsum_kernel<<<(classes * C + 255) / 256, 256, 0, s>>>(pw, grid, classes * C, d_weight, 0);
  MFB_LAUNCH_CHECK("head dweight");
  enc::colsum_kernel<<<1, 32, 0, s>>>(pl, grid, 2, loss_count, 0);
  MFB_LAUNCH_CHECK("head loss");
  return MFB_OK;
}
