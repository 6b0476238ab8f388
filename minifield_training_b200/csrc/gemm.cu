// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// C[M,N] = alpha * A[M,K] . B[N,K]^T (optionally times a uint8 mask), fp32
// accumulation in TMEM, bf16 or fp32 output. This is full_linear
// (src/minifield_training/kernels/linear.py:7-13: x @ W.astype(bf16).T) and the
// two products of its backward, dX = dY W and dW = dY^T X; with the QAT STE
// mask fused into the weight-gradient epilogue (the STE of
// strategies/quantization.py:114-126).
//
// Each operand may be K-major (stored [rows, K]) or MN-major (stored
// [K, rows]); both are loaded by TMA with 128-byte swizzle and described to
// the tensor core without any transpose pass:
//   K-major : box {64 K, rows}, 8-row groups 1024 B apart (SBO), K steps of
//             16 elements advance the start address by 32 B inside the atom.
//   MN-major: boxes {64 rows, 64 K} placed 8192 B apart (LBO), 8-K-row groups
//             1024 B apart (SBO), K steps advance by 2048 B.
//
// Persistent, warp-specialised CTA (one per SM, 320 threads):
//   warp 0     TMA producer over a shared-memory stage ring,
//   warp 1     TMEM allocator + single-thread tcgen05.mma issuer,
//   warps 2-9  epilogue, two warps per TMEM lane quarter each taking half of
//              the tile's columns: tcgen05.ld of the CTA's 128x256 fp32
//              accumulator, scale, mask, convert and store.
// Two TMEM accumulators (2 x 256 columns) let the epilogue of one tile overlap
// the main loop of the next. Every mbarrier wait is bounded; a timeout writes a
// device status word that the host reads back (no trap, no endless spin).
//
// Products with more than 128 output rows run on CTA pairs (clusters of two,
// tcgen05 cta_group::2): a pair owns a 256x256 output tile, each CTA loads its
// 128 A rows and 128 of the 256 B rows of a k-block (32 KB per stage, six
// stages) into its own shared memory, and the even CTA issues one M=256 MMA per
// 16-deep step that reads both CTAs' halves and accumulates each CTA's 128 rows
// in that CTA's TMEM. Per 128x256x64 of work a CTA then streams 32 KB from L2
// instead of 48 KB (a lone CTA loads all 256 B rows, four 48 KB stages), which
// is what bounds the single-CTA main loop. Loads complete on the even CTA's
// stage barrier; the MMA commits are multicast to both CTAs' stage-empty and
// accumulator-full barriers; the odd CTA's epilogue releases an accumulator by
// a remote arrive. No load is multicast.
//
// SwiGLU epilogues (layers/feed_forward.py:24-35): in the gate|up projection
// (EPI_SWIGLU_FWD) each 256-wide B tile is the 128 gate rows and the 128
// matching up rows of the fused [gate; up] weight (two 128-row TMA boxes), so
// the epilogue holds gate and up of the same 128 channels and writes gu
// (bf16, the saved activation) and h = silu(gate) * up in one pass. In the
// down projection's input gradient (EPI_SWIGLU_BWD) the epilogue rounds the
// dH tile to bf16, reads gate and up of its channels from gu and writes
// dGU = [dH * up * silu'(gate), dH * silu(gate)]; dH is never stored.
//
// Products of at most 64 rows without a mask (the decode step's [batch, C]
// projections) run swapped: D = B . A^T, the weight rows on the MMA's 128-row
// side and the batch as a 64-wide N tile, D stored transposed into C; the
// weights are the operand loaded ahead of a programmatic-dependency wait.
//
// Split-K, when a caller-owned workspace is given and the output tiles fill
// the GPU poorly: deep decode projections (w2) and the weight gradients (a
// few 256x256 pair tiles, K = the token count).
// The K range is cut into up to 16 slices (choose_split); each (tile, slice)
// is a work item that writes its FP32 partial [M, N] to the workspace, and
// splitk_reduce_kernel sums the slices in slice order (deterministic), scales,
// applies the STE mask and converts.
#include <cudaTypedefs.h>

#include <algorithm>

#include "tc.cuh"

namespace mfb {
namespace gemm {

// Device status word of the GEMM kernels on each device (0 = ok; otherwise the
// id of the bounded wait that gave up). Read and cleared by mfb_gemm_status.
__device__ int g_status;

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter, each storing half of a tile's columns
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int A_BYTES = BM * BK * 2;
constexpr int EPI_PLAIN = 0, EPI_SWIGLU_FWD = 1, EPI_SWIGLU_BWD = 2;

struct Args {
  void* C;
  const uint8_t* mask;
  long long ldc;
  int M, N, K;
  int out_f32;
  int a_mn, b_mn;
  int num_m, num_n, num_k;
  int vec_ok;  // C rows 16-byte aligned: vector stores
  float alpha;
  int k_split, kb_per;  // K slices and k-blocks per slice (1, num_k without split-K)
  float* partial;       // [k_split, M, N] FP32 partials when k_split > 1
  int epi;              // EPI_*: plain store or a SwiGLU epilogue
  int n_fast;           // work order: n block fastest (tiles sharing A rows run together)
  int swapped;          // the product runs as D = B . A^T (weights as the MMA's M side): D[r][s] is
                        // stored at C[s * ldc + r], and the weights (A here) stream before the
                        // programmatic-dependency wait
  int F;                // SwiGLU width (gate and up channels each)
  __nv_bfloat16* h;     // EPI_SWIGLU_FWD: h [M, F], row stride F
  const __nv_bfloat16* gu;  // EPI_SWIGLU_BWD: gu [M, 2F] read by the epilogue
};

// Logistic sigmoid in the SwiGLU epilogues: the hardware exp2 and reciprocal
// (a few ulp of FP32, far below the bf16 rounding of every value it feeds).
__device__ __forceinline__ float silu_sigmoid(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

__device__ __forceinline__ void unpack8_bf16(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

__device__ __forceinline__ void store32_bf16(__nv_bfloat16* dst, const float* v) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 o;
    o.x = pack_bf16(v[8 * i], v[8 * i + 1]);
    o.y = pack_bf16(v[8 * i + 2], v[8 * i + 3]);
    o.z = pack_bf16(v[8 * i + 4], v[8 * i + 5]);
    o.w = pack_bf16(v[8 * i + 6], v[8 * i + 7]);
    reinterpret_cast<uint4*>(dst)[i] = o;
  }
}

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// EPI_SWIGLU_FWD, one row and 32 channels: gate and up accumulators in, gu
// (gate at column c, up at F + c) and h out, each value rounded to bf16 where
// the reference's bf16 graph rounds it (full_linear's output, then the product).
__device__ __forceinline__ void swiglu_fwd_chunk(const Args& a, int row, int c, const uint32_t* g32,
                                                 const uint32_t* u32) {
  float g[32], u[32], h[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    g[i] = round_bf16(__uint_as_float(g32[i]) * a.alpha);
    u[i] = round_bf16(__uint_as_float(u32[i]) * a.alpha);
    h[i] = g[i] * silu_sigmoid(g[i]) * u[i];
  }
  __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)row * a.ldc;
  store32_bf16(gu + c, g);
  store32_bf16(gu + a.F + c, u);
  store32_bf16(a.h + (long long)row * a.F + c, h);
}

// EPI_SWIGLU_BWD: gate and up of one row's 32 channels (loaded a chunk ahead).
struct GuChunk {
  uint4 g[4], u[4];
};
__device__ __forceinline__ void load_gu(const Args& a, int row, int c, GuChunk& out) {
  const uint4* gp = reinterpret_cast<const uint4*>(a.gu + (long long)row * 2 * a.F + c);
  const uint4* up = reinterpret_cast<const uint4*>(a.gu + (long long)row * 2 * a.F + a.F + c);
#pragma unroll
  for (int i = 0; i < 4; ++i) out.g[i] = gp[i], out.u[i] = up[i];
}

// EPI_SWIGLU_BWD, one row and 32 channels: dH accumulator and gate/up in, dGU out.
__device__ __forceinline__ void swiglu_bwd_chunk(const Args& a, int row, int c, const uint32_t* d32,
                                                 const GuChunk& in) {
  float g[32], u[32], dg[32], du[32];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    unpack8_bf16(in.g[i], g + 8 * i);
    unpack8_bf16(in.u[i], u + 8 * i);
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float d = round_bf16(__uint_as_float(d32[i]) * a.alpha);
    const float sg = silu_sigmoid(g[i]);
    du[i] = d * g[i] * sg;
    dg[i] = d * u[i] * sg * (1.f + g[i] * (1.f - sg));
  }
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)row * a.ldc;
  store32_bf16(out + c, dg);
  store32_bf16(out + a.F + c, du);
}

// Work item -> (m block, n block, first and end k-block). Consecutive items
// run at the same time on neighbouring SMs, so the fastest-varying block index
// decides which operand they share through L2: m fastest shares a B panel, n
// fastest an A panel. The host puts the larger operand's panels in common, so
// that operand streams from HBM once instead of once per block of the other
// dimension.
struct Item {
  int mb, nb, kb0, kb1;
};
__device__ __forceinline__ Item item_of(const Args& a, int tile) {
  const int mn = tile % (a.num_m * a.num_n), ks = tile / (a.num_m * a.num_n);
  Item it;
  if (a.n_fast) {
    it.nb = mn % a.num_n;
    it.mb = mn / a.num_n;
  } else {
    it.mb = mn % a.num_m;
    it.nb = mn / a.num_m;
  }
  it.kb0 = ks * a.kb_per;
  it.kb1 = min(a.num_k, it.kb0 + a.kb_per);
  return it;
}

// Raw FP32 partial of 32 columns of one row for split-K.
__device__ __forceinline__ void store_partial(const Args& a, int ks, int row, int col0, const uint32_t* r) {
  float* c = a.partial + ((long long)ks * a.M + row) * a.N + col0;
  if (col0 + 32 <= a.N && (a.N & 3) == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      reinterpret_cast<float4*>(c)[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                                    __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
  } else {
    for (int i = 0; i < 32; ++i)
      if (col0 + i < a.N) c[i] = __uint_as_float(r[i]);
  }
}

// C = alpha * sum over slices of the partials, slice 0 first, times the
// uint8 mask [M, N] when given (as store_chunk applies it). One thread per 4
// consecutive columns when N % 4 == 0 (float4 partial loads, issued ahead of
// the in-order adds), else one per element.
template <bool VEC4>
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int k_split, int M, int N, void* C,
                                     long long ldc, int out_f32, float alpha, const uint8_t* __restrict__ mask,
                                     int trans) {
  const int per = VEC4 ? 4 : 1, cols = N / per;
  const long long total = (long long)M * cols, slice = (long long)M * N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i / cols), col = (int)(i - (long long)row * cols) * per;
    const float* p = partial + (long long)row * N + col;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int ks = 0; ks < k_split; ++ks) {
      if (VEC4) {
        const float4 v = *reinterpret_cast<const float4*>(p + ks * slice);
        acc[0] += v.x;
        acc[1] += v.y;
        acc[2] += v.z;
        acc[3] += v.w;
      } else {
        acc[0] += p[ks * slice];
      }
    }
    float mk[4] = {1.f, 1.f, 1.f, 1.f};
    if (mask) {
      if (VEC4) {
        const uchar4 m4 = *reinterpret_cast<const uchar4*>(mask + (long long)row * N + col);
        mk[0] = m4.x, mk[1] = m4.y, mk[2] = m4.z, mk[3] = m4.w;
      } else {
        mk[0] = mask[(long long)row * N + col];
      }
    }
#pragma unroll
    for (int e = 0; e < per; ++e) {
      const float v = acc[e] * alpha * mk[e];
      // Swapped products (trans): partial element (row, col) is C's (col, row).
      const long long at = trans ? (long long)(col + e) * ldc + row : row * ldc + col + e;
      if (out_f32)
        reinterpret_cast<float*>(C)[at] = v;
      else
        reinterpret_cast<__nv_bfloat16*>(C)[at] = __float2bfloat16_rn(v);
    }
  }
}

// Swapped products: D[row][col0 + i] goes to C[(col0 + i) * ldc + row]; a
// warp's lanes hold consecutive rows, so each store instruction writes one
// contiguous run of C.
__device__ __forceinline__ void store_chunk_t(const Args& a, int row, int col0, const uint32_t* r) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int col = col0 + i;
    if (col < a.N) {
      const float v = __uint_as_float(r[i]) * a.alpha;
      if (a.out_f32)
        reinterpret_cast<float*>(a.C)[(long long)col * a.ldc + row] = v;
      else
        reinterpret_cast<__nv_bfloat16*>(a.C)[(long long)col * a.ldc + row] = __float2bfloat16_rn(v);
    }
  }
}

__device__ __forceinline__ void store_chunk(const Args& a, int row, int col0, const uint32_t* r) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * a.alpha;
  const bool full = col0 + 32 <= a.N;
  const bool vec = full && a.vec_ok;
  if (a.mask) {
    const uint8_t* mrow = a.mask + (long long)row * a.N + col0;
    if (full && (a.N & 15) == 0) {
      const uint4 m0 = *reinterpret_cast<const uint4*>(mrow);
      const uint4 m1 = *reinterpret_cast<const uint4*>(mrow + 16);
      const uint8_t* mb0 = reinterpret_cast<const uint8_t*>(&m0);
      const uint8_t* mb1 = reinterpret_cast<const uint8_t*>(&m1);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[i] *= (float)mb0[i];
        v[16 + i] *= (float)mb1[i];
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < a.N) v[i] *= (float)mrow[i];
    }
  }
  if (a.out_f32) {
    float* c = reinterpret_cast<float*>(a.C) + (long long)row * a.ldc + col0;
    if (vec) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4*>(c)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < a.N) c[i] = v[i];
    }
  } else {
    __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)row * a.ldc + col0;
    if (vec) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 o;
        o.x = pack_bf16(v[8 * i], v[8 * i + 1]);
        o.y = pack_bf16(v[8 * i + 2], v[8 * i + 3]);
        o.z = pack_bf16(v[8 * i + 4], v[8 * i + 5]);
        o.w = pack_bf16(v[8 * i + 6], v[8 * i + 7]);
        reinterpret_cast<uint4*>(c)[i] = o;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < a.N) c[i] = __float2bfloat16_rn(v[i]);
    }
  }
}

// Shape of one CTA's share of the work. A CTA always owns 128 accumulator rows
// and the tile's 256 columns; alone it loads all 256 B rows of a k-block, in a
// pair (PAIR) it loads its 128 of them and the pair MMA (M = 256) reads both
// halves, so each CTA streams 32 KB instead of 48 KB per 128x256x64 step.
// A pair with a SwiGLU epilogue stages its epilogue through shared memory
// (STAGED): each epilogue warp owns a ring of RING slots of SLOT bytes, one
// 32-row x 32-column chunk per slot (64-byte swizzled bf16 boxes moved by TMA),
// and the main loop keeps four stages to make room.
// TN: the tile's N (256; 64 for swapped products, whose N is a handful of
// activation rows, with more stages for the weight stream).
template <bool PAIR, int EPI, int TN = BN>
struct Shape {
  static constexpr bool STAGED = PAIR && EPI != EPI_PLAIN;
  static constexpr int B_ROWS = PAIR ? TN / 2 : TN;
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = PAIR ? (STAGED ? 4 : 6) : (TN == BN ? 4 : 8);
  static constexpr int TMEM_COLS = 2 * TN;
  // SwiGLU backward: gate and up boxes in, overwritten in place by dGate and
  // dUp (two 2 KB boxes); forward: gate, up and h out (three boxes).
  static constexpr int RING = EPI == EPI_SWIGLU_BWD ? 3 : 2;
  static constexpr int SLOT = EPI == EPI_SWIGLU_BWD ? 4096 : 6144;
  static constexpr int RING_BYTES = STAGED ? EPI_WARPS * RING * SLOT : 0;
  static constexpr int TAIL = 512;  // mbarriers and the TMEM address slot
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + RING_BYTES + TAIL;
  static_assert(8 * (2 * STAGES + 6 + EPI_WARPS * RING) + 4 <= TAIL, "barriers and the TMEM slot fit the tail");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

// Byte offset of 16-byte piece j of row r in a 32 x 32 bf16 box with 64-byte
// rows and 64-byte swizzle (piece index XOR bits 7-8 of the row's address):
// a warp whose lanes each own one row touches every bank once per 8 lanes.
__device__ __forceinline__ int sw64(int r, int j) { return r * 64 + ((j ^ ((r >> 1) & 3)) << 4); }

__device__ __forceinline__ void box_store32(uint8_t* box, int r, const float* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 o;
    o.x = pack_bf16(v[8 * j], v[8 * j + 1]);
    o.y = pack_bf16(v[8 * j + 2], v[8 * j + 3]);
    o.z = pack_bf16(v[8 * j + 4], v[8 * j + 5]);
    o.w = pack_bf16(v[8 * j + 6], v[8 * j + 7]);
    *reinterpret_cast<uint4*>(box + sw64(r, j)) = o;
  }
}
__device__ __forceinline__ void box_load32(const uint8_t* box, int r, float* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j) unpack8_bf16(*reinterpret_cast<const uint4*>(box + sw64(r, j)), v + 8 * j);
}

// Staged EPI_SWIGLU_FWD for one row r of a chunk: gate, up and h into the
// slot's three boxes (same rounding as swiglu_fwd_chunk; the SwiGLU products
// are unscaled, alpha = 1).
__device__ __forceinline__ void swiglu_fwd_box(const uint32_t* g32, const uint32_t* u32, uint8_t* slot, int r) {
  float g[32], u[32], h[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    g[i] = round_bf16(__uint_as_float(g32[i]));
    u[i] = round_bf16(__uint_as_float(u32[i]));
    h[i] = g[i] * silu_sigmoid(g[i]) * u[i];
  }
  box_store32(slot, r, g);
  box_store32(slot + 2048, r, u);
  box_store32(slot + 4096, r, h);
}

// Staged EPI_SWIGLU_BWD for one row r of a chunk: gate and up read from the
// slot, dGate and dUp written over them (same math as swiglu_bwd_chunk, alpha = 1).
__device__ __forceinline__ void swiglu_bwd_box(const uint32_t* d32, uint8_t* slot, int r) {
  float g[32], u[32], dg[32], du[32];
  box_load32(slot, r, g);
  box_load32(slot + 2048, r, u);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float d = round_bf16(__uint_as_float(d32[i]));
    const float sg = silu_sigmoid(g[i]);
    du[i] = d * g[i] * sg;
    dg[i] = d * u[i] * sg * (1.f + g[i] * (1.f - sg));
  }
  box_store32(slot, r, dg);
  box_store32(slot + 2048, r, du);
}

// te0 / te1: the staged epilogue's tensor maps (SwiGLU backward: gu loaded,
// dGU stored; forward: gu and h stored); unused otherwise.
template <bool PAIR, int EPI, int TN = BN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                const __grid_constant__ CUtensorMap te0, const __grid_constant__ CUtensorMap te1, Args args) {
  using S = Shape<PAIR, EPI, TN>;
  constexpr int TMEM_COLS = S::TMEM_COLS;
  constexpr int STAGES = S::STAGES, STAGE_BYTES = S::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  // Offset from the __shared__ array itself so accesses keep the shared state space.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t ring = sbase + STAGES * STAGE_BYTES;  // staged epilogue slots (STAGED only)
  const uint32_t bars = ring + S::RING_BYTES;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bars + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bars + 8u * (2 * STAGES + 2 + a); };
  const uint32_t done_bar = bars + 8u * (2 * STAGES + 4);
  // One slot-full barrier per ring slot of each epilogue warp (STAGED).
  auto slot_bar = [&](int ew, int b) { return bars + 8u * (2 * STAGES + 6 + ew * S::RING + b); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + STAGES * STAGE_BYTES + S::RING_BYTES +
                                                    8 * (2 * STAGES + 6 + EPI_WARPS * S::RING));

  // In a pair, rank 0 issues the MMAs and owns the stage-full and
  // accumulator-empty barriers both CTAs signal; work is walked per pair.
  const uint32_t rank = PAIR ? tc::cluster_ctarank() : 0u;
  const int unit = PAIR ? (int)tc::cluster_id_x() : (int)blockIdx.x;
  const int units = PAIR ? (int)tc::cluster_count_x() : (int)gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(full_bar(s), 1);
      tc::mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(tfull_bar(a), 1);
      tc::mbar_init(tempty_bar(a), (PAIR ? 2 : 1) * EPI_WARPS);  // one arrival per epilogue warp
    }
    tc::mbar_init(done_bar, 1);
    if (S::STAGED)
      for (int i = 0; i < EPI_WARPS * S::RING; ++i) tc::mbar_init(slot_bar(0, i), 1);
    tc::mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tc::tma_prefetch_desc(&ta);
    tc::tma_prefetch_desc(&tb);
  }
  if (warp == 1) {
    if (PAIR) {
      tc::tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
      tc::tmem_relinquish_pair();
    } else {
      tc::tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
      tc::tmem_relinquish();
    }
  }
  tc::tc_fence_before();
  if (PAIR)
    tc::cluster_sync();  // the peer's barriers are initialised before any load signals them
  else
    __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int num_tiles = args.num_m * args.num_n * args.k_split;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // Loads signal the leader's stage-full barrier; only the leader expects
      // the bytes (both CTAs' loads) and arrives.
      auto full_target = [&](int s) { return PAIR ? tc::mapa_shared(full_bar(s), 0) : full_bar(s); };
      auto load = [&](uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
        if (PAIR)
          tc::tma_load_2d_pair(dst, map, x, y, bar);
        else
          tc::tma_load_2d(dst, map, x, y, bar);
      };
      auto expect = [&](int s) {
        if (rank == 0) tc::mbar_expect_tx(full_bar(s), (PAIR ? 2 : 1) * STAGE_BYTES);
      };
      // This CTA's B rows of one stage: rows nb*TN + rank*B_ROWS.. (K-major
      // box or MN-major 64-row boxes), or for the SwiGLU forward the 128 gate
      // and the 128 up rows of channel block nb (alone: two boxes; in a pair
      // rank 0 loads the gate rows and rank 1 the up rows, so the accumulator
      // columns are gate | up either way).
      auto load_b = [&](uint32_t sb, int kb, int nb, uint32_t bar) {
        if (EPI == EPI_SWIGLU_FWD) {
          if (PAIR) {
            load(sb, &tb, kb * BK, (int)rank * args.F + nb * (TN / 2), bar);
          } else {
            load(sb, &tb, kb * BK, nb * (TN / 2), bar);
            load(sb + (TN / 2) * 128, &tb, kb * BK, args.F + nb * (TN / 2), bar);
          }
        } else if (!args.b_mn) {
          load(sb, &tb, kb * BK, nb * TN + (int)rank * S::B_ROWS, bar);
        } else {
#pragma unroll
          for (int j = 0; j < S::B_ROWS / 64; ++j)
            load(sb + j * 8192, &tb, nb * TN + (int)rank * S::B_ROWS + 64 * j, kb * BK, bar);
        }
      };
      auto load_a = [&](uint32_t sa, int kb, int mb, uint32_t bar) {
        if (!args.a_mn) {
          load(sa, &ta, kb * BK, mb * BM, bar);
        } else {
#pragma unroll
          for (int i = 0; i < BM / 64; ++i) load(sa + i * 8192, &ta, mb * BM + 64 * i, kb * BK, bar);
        }
      };
      // The weights (B; A of a swapped product) of the first tile's first
      // stages load before the dependency wait: a GEMM launched as a
      // programmatic dependent streams them while the previous kernel
      // finishes. The activations, and everything this grid writes, come
      // after the wait.
      const bool w_is_a = args.swapped != 0;
      int pre = 0;
      if (unit < num_tiles) {
        const Item it = item_of(args, unit);
        pre = min(STAGES, it.kb1 - it.kb0);
        for (int i = 0; i < pre; ++i) {
          expect(i);
          const uint32_t sa = sbase + i * STAGE_BYTES;
          if (w_is_a)
            load_a(sa, it.kb0 + i, it.mb * (PAIR ? 2 : 1) + (int)rank, full_target(i));
          else
            load_b(sa + A_BYTES, it.kb0 + i, it.nb, full_target(i));
        }
      }
      wait_prerequisites();
      for (int tile = unit; ok && tile < num_tiles; tile += units) {
        const Item it = item_of(args, tile);
        const int mb = it.mb * (PAIR ? 2 : 1) + (int)rank, nb = it.nb;
        for (int kb = it.kb0; kb < it.kb1; ++kb) {
          const bool early = tile == unit && kb - it.kb0 < pre;  // weights already in flight
          if (!early) {
            if (!tc::mbar_wait(empty_bar(stage), phase ^ 1, &g_status, 1)) {
              ok = false;
              break;
            }
            expect(stage);
          }
          const uint32_t sa = sbase + stage * STAGE_BYTES, sb = sa + A_BYTES, bar = full_target(stage);
          if (!early || !w_is_a) load_a(sa, kb, mb, bar);
          if (!early || w_is_a) load_b(sb, kb, nb, bar);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // The whole warp runs the issue loop (converged); one elected lane issues.
    // In a pair only rank 0 issues.
    if (rank == 0) {
      const uint32_t idesc = tc::idesc_bf16_f32(PAIR ? 2 * BM : BM, TN, args.a_mn, args.b_mn);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = unit; ok && tile < num_tiles; tile += units) {
        if (!tc::mbar_wait_w(tempty_bar(acc), acc_phase ^ 1, &g_status, 2)) break;
        tc::tc_fence_after();
        const uint32_t d = tmem + acc * TN;
        const Item it = item_of(args, tile);
        for (int kb = it.kb0; kb < it.kb1; ++kb) {
          if (!tc::mbar_wait_w(full_bar(stage), phase, &g_status, 3)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t sa = sbase + stage * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = args.a_mn ? tc::smem_desc_sw128(sa + k * 2048, 8192, 1024)
                                          : tc::smem_desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = args.b_mn ? tc::smem_desc_sw128(sb + k * 2048, 8192, 1024)
                                          : tc::smem_desc_sw128(sb + k * 32, 16, 1024);
            const uint32_t accumulate = (kb != it.kb0 || k != 0) ? 1u : 0u;
            if (PAIR)
              tc::mma_bf16_pair_w(d, ad, bd, idesc, accumulate);
            else
              tc::mma_bf16_w(d, ad, bd, idesc, accumulate);
          }
          if (PAIR)
            tc::mma_commit_pair_both_w(empty_bar(stage));
          else
            tc::mma_commit_w(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (PAIR)
          tc::mma_commit_pair_both_w(tfull_bar(acc));
        else
          tc::mma_commit_w(tfull_bar(acc));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // Drain: every MMA issued above has completed before TMEM is freed.
      if (PAIR)
        tc::mma_commit_pair_w(done_bar);
      else
        tc::mma_commit_w(done_bar);
      tc::mbar_wait_w(done_bar, 0, &g_status, 4);
    }
  } else if constexpr (S::STAGED) {
    // Staged SwiGLU epilogue. This warp's region of each tile is 32 rows
    // (TMEM lane quarter q) x half of the columns, walked in 32-column chunks;
    // chunk i of the warp's whole sequence uses ring slot i % RING. Lane 0
    // issues the TMA ops and commits one bulk group per chunk (empty when the
    // chunk lies past M), so "group of chunk i - k done" is a fixed count.
    constexpr int RING = S::RING, SLOT = S::SLOT;
    constexpr int CH = EPI == EPI_SWIGLU_BWD ? 4 : 2;  // chunks per tile per warp
    const int q = warp & 3, half = (warp - 2) >> 2, ew = warp - 2;
    const uint32_t my_ring = ring + ew * RING * SLOT;
    uint8_t* my_ring_p = smem + STAGES * STAGE_BYTES + ew * RING * SLOT;
    // Output column (backward: dH column; forward: channel) of chunk c of a tile.
    auto chunk_col = [&](const Item& it, int c) {
      return EPI == EPI_SWIGLU_BWD ? it.nb * TN + half * 128 + c * 32 : it.nb * (TN / 2) + half * 64 + c * 32;
    };
    auto chunk_row0 = [&](const Item& it) { return (it.mb * 2 + (int)rank) * BM + q * 32; };
    uint32_t loaded = 0, slot_phase = 0;  // per slot: a gu load in flight; its barrier parity
    // SwiGLU backward: gate|up loads run RING - 1 chunks ahead of the math.
    // The load cursor walks the same chunk sequence; a tile's coordinates are
    // decoded once, when the cursor enters it.
    int ld_j = 0, ld_c = 0, ld_tile = unit, ld_row0 = 0, ld_col0 = 0;
    auto ld_enter = [&]() {
      if (ld_tile < num_tiles) {
        const Item it = item_of(args, ld_tile);
        ld_row0 = chunk_row0(it);
        ld_col0 = chunk_col(it, 0);
      }
    };
    ld_enter();
    // The load of the cursor's chunk (every lane tracks it; lane 0 issues it).
    auto issue_next_load = [&]() {
      const int j = ld_j++, tile = ld_tile, row0 = ld_row0, col = ld_col0 + ld_c * 32;
      if (++ld_c == CH) {
        ld_c = 0;
        ld_tile += units;
        ld_enter();
      }
      if (tile >= num_tiles || row0 >= args.M || col >= args.F) return;
      const int b = j % RING;
      loaded |= 1u << b;
      if (lane == 0) {
        tc::mbar_expect_tx(slot_bar(ew, b), 2 * 2048);
        tc::tma_load_2d(my_ring + b * SLOT, &te0, col, row0, slot_bar(ew, b));
        tc::tma_load_2d(my_ring + b * SLOT + 2048, &te0, args.F + col, row0, slot_bar(ew, b));
      }
    };
    if (EPI == EPI_SWIGLU_BWD) {
      wait_prerequisites();  // gu comes from an earlier kernel
      for (int j = 0; j < RING - 1; ++j) issue_next_load();
    }
    int acc = 0, i = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int tile = unit; ok && tile < num_tiles; tile += units) {
      const Item it = item_of(args, tile);
      const int row0 = chunk_row0(it);
      if (!tc::mbar_wait_w(tfull_bar(acc), acc_phase, &g_status, 5)) break;
      tc::tc_fence_after();
      const uint32_t tacc = tmem + ((uint32_t)(q * 32) << 16) + acc * TN;
#pragma unroll 1
      for (int c = 0; c < CH; ++c, ++i) {
        const int col = chunk_col(it, c), b = i % RING;
        const bool live = row0 < args.M && col < args.F;
        uint8_t* slot_p = my_ring_p + b * SLOT;
        const uint32_t slot = my_ring + b * SLOT;
        if (EPI == EPI_SWIGLU_BWD) {
          uint32_t r[32];
          tc::tmem_ld_32x32b_x32(tacc + half * 128 + c * 32, r);
          tc::tmem_ld_wait();
          if (live && ok) {
            if (tc::mbar_wait_w(slot_bar(ew, b), (slot_phase >> b) & 1, &g_status, 6)) {
              slot_phase ^= 1u << b;
              loaded &= ~(1u << b);
              swiglu_bwd_box(r, slot_p, lane);
              tc::fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tc::tma_store_2d(&te1, slot, col, row0);
                tc::tma_store_2d(&te1, slot + 2048, args.F + col, row0);
              }
            } else {
              ok = false;
            }
          }
          if (lane == 0) {
            tc::bulk_commit_group();
            tc::bulk_wait_group_read<1>();  // chunk i - 1's stores have left its slot
          }
          __syncwarp();
          if (ok) issue_next_load();  // chunk i + RING - 1, into chunk i - 1's slot
        } else {
          uint32_t g[32], u[32];
          tc::tmem_ld_32x32b_x32(tacc + half * 64 + c * 32, g);
          tc::tmem_ld_32x32b_x32(tacc + TN / 2 + half * 64 + c * 32, u);
          tc::tmem_ld_wait();
          if (lane == 0) tc::bulk_wait_group_read<RING - 1>();  // chunk i - RING's stores have left this slot
          __syncwarp();
          if (live) {
            swiglu_fwd_box(g, u, slot_p, lane);
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tc::tma_store_2d(&te0, slot, col, row0);
              tc::tma_store_2d(&te0, slot + 2048, args.F + col, row0);
              tc::tma_store_2d(&te1, slot + 4096, col, row0);
            }
          }
          if (lane == 0) tc::bulk_commit_group();
        }
      }
      // This warp's TMEM reads of the tile are done: one (remote) arrival on
      // the leader's accumulator-empty barrier.
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cluster(tc::mapa_shared(tempty_bar(acc), 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    // Unwind: loads still in flight (only after a timeout) land before exit,
    // and every store has completed.
    for (int b = 0; b < RING; ++b)
      if (loaded & (1u << b)) tc::mbar_wait_w(slot_bar(ew, b), (slot_phase >> b) & 1, &g_status, 7);
    if (lane == 0) tc::bulk_wait_group0();
    __syncwarp();
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // which half of the tile's columns this warp stores
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = unit; tile < num_tiles; tile += units) {
      const Item it = item_of(args, tile);
      const int mb = it.mb * (PAIR ? 2 : 1) + (int)rank, nb = it.nb, ks = tile / (args.num_m * args.num_n);
      if (!tc::mbar_wait_w(tfull_bar(acc), acc_phase, &g_status, 5)) break;
      tc::tc_fence_after();
      const int row = mb * BM + q * 32 + lane;
      const uint32_t tacc = tmem + ((uint32_t)(q * 32) << 16) + acc * TN;
      if (EPI == EPI_SWIGLU_FWD) {
#pragma unroll 1
        for (int ch = half * (TN / 128); ch < (half + 1) * (TN / 128); ++ch) {  // gate ch*32.., up TN/2 + ch*32..
          uint32_t g[32], u[32];
          tc::tmem_ld_32x32b_x32(tacc + ch * 32, g);
          tc::tmem_ld_32x32b_x32(tacc + TN / 2 + ch * 32, u);
          tc::tmem_ld_wait();
          if (row < args.M) swiglu_fwd_chunk(args, row, nb * (TN / 2) + ch * 32, g, u);
        }
      } else if (EPI == EPI_SWIGLU_BWD) {
        const int ch0 = half * (TN / 64), ch1 = ch0 + TN / 64;
        GuChunk cur, next;
        if (row < args.M && nb * TN + ch0 * 32 < args.N) load_gu(args, row, nb * TN + ch0 * 32, cur);
#pragma unroll 1
        for (int ch = ch0; ch < ch1; ++ch) {
          uint32_t r[32];
          tc::tmem_ld_32x32b_x32(tacc + ch * 32, r);
          const int col0 = nb * TN + ch * 32;
          if (ch + 1 < ch1 && row < args.M && col0 + 32 < args.N) load_gu(args, row, col0 + 32, next);
          tc::tmem_ld_wait();
          if (row < args.M && col0 < args.N) swiglu_bwd_chunk(args, row, col0, r, cur);
          cur = next;
        }
      } else {
#pragma unroll 1
        for (int ch = half * (TN / 64); ch < (half + 1) * (TN / 64); ++ch) {
          uint32_t r[32];
          tc::tmem_ld_32x32b_x32(tacc + ch * 32, r);
          tc::tmem_ld_wait();
          const int col0 = nb * TN + ch * 32;
          if (row < args.M && col0 < args.N) {
            if (args.k_split > 1)
              store_partial(args, ks, row, col0, r);
            else if (args.swapped)
              store_chunk_t(args, row, col0, r);
            else
              store_chunk(args, row, col0, r);
          }
        }
      }
      // This warp's TMEM reads are done: one arrival on the leader's
      // accumulator-empty barrier (remote for the peer of a pair).
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR)
          tc::mbar_arrive_cluster(tc::mapa_shared(tempty_bar(acc), 0));
        else
          tc::mbar_arrive(tempty_bar(acc));
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  // Both CTAs of a pair stay resident until every MMA, load and remote
  // arrival of the pair is done; then each frees its TMEM.
  tc::tc_fence_before();
  if (PAIR)
    tc::cluster_sync();
  else
    __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    if (PAIR)
      tc::tmem_dealloc_pair(tmem, TMEM_COLS);
    else
      tc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace gemm

namespace tc {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                   uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return set_error(MFB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MFB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MFB_OK;
}

int make_tmap_bf16_box32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld) {
  auto fn = encode_fn();
  if (!fn) return set_error(MFB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MFB_ERR_CUDA, "cuTensorMapEncodeTiled (32x32 box) failed (%d)", (int)r);
  return MFB_OK;
}

int make_tmap_bf16_heads(CUtensorMap* map, const void* base, uint64_t rows, int heads, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(MFB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[3] = {64, rows, (cuuint64_t)heads};
  cuuint64_t strides[2] = {(cuuint64_t)heads * 128, 128};
  cuuint32_t box[3] = {64, box_rows, (cuuint32_t)heads};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MFB_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return MFB_OK;
}

int make_tmap_f32_rows_heads(CUtensorMap* map, const void* base, int heads, uint64_t T, uint64_t batch,
                             uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(MFB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[4] = {64, (cuuint64_t)heads, T, batch};
  cuuint64_t strides[3] = {256, (cuuint64_t)heads * 256, T * (cuuint64_t)heads * 256};
  cuuint32_t box[4] = {32, 1, box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MFB_ERR_CUDA, "cuTensorMapEncodeTiled (4-D f32) failed (%d)", (int)r);
  return MFB_OK;
}

}  // namespace tc
}  // namespace mfb

using namespace mfb;

namespace {
int sm_count(int dev) {
  static int counts[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!counts[dev]) cudaDeviceGetAttribute(&counts[dev], cudaDevAttrMultiProcessorCount, dev);
  return counts[dev] ? counts[dev] : 148;
}
}  // namespace

namespace {
int pair_clusters(int dev);

// K slices for an (M, N, K) product, at most SPLIT_MAX.
//
// Products of more than 128 rows run on CTA pairs; there the slice count s
// minimises the modelled time ceil(tiles * s / pairs) / s (waves of one
// slice's work, in units of one full-K pair tile at ~0.5 us per 64-deep
// k-block) plus the partials' HBM traffic ((2s + 1) x M x N x 4 bytes at
// ~6 TB/s: written, read back, and the output) in the same units; a larger s
// must win by 3 %. This is what fills the GPU for the weight gradients, whose
// few output tiles (e.g. 1024 x 1024 = 16 pair tiles) run K = 65536 deep.
// Each slice keeps at least SPLIT_MIN_KB_PAIR k-blocks.
//
// Smaller products (the decode projections, single-CTA tiles): > 1 only when
// the tiles fill fewer than half the SMs and a tile is deep enough to be
// worth a reduce launch, slices of at least SPLIT_MIN_KB k-blocks, so the FP32
// partials stay well below the bf16 operand bytes a slice streams.
constexpr int SPLIT_MIN_KB = 4, SPLIT_MIN_KB_PAIR = 8, SPLIT_MAX = 16, SPLIT_MIN_TILE_KB = 30;
int choose_split(int M, int N, int K, int dev, int* kb_per, bool single = false) {
  const int num_k = cdiv(K, gemm::BK);
  *kb_per = num_k;
  const int pairs = M > gemm::BM && !single ? pair_clusters(dev) : 0;
  if (pairs > 0) {
    const int tiles = cdiv(M, 2 * gemm::BM) * cdiv(N, gemm::BN);
    const double tile_us = 0.5 * num_k, bytes = 4.0 * M * N;
    double best_t = 0.0;
    int best = 1;
    for (int s = 1; s <= SPLIT_MAX && (s == 1 || num_k / s >= SPLIT_MIN_KB_PAIR); ++s) {
      const double waves = (double)cdiv(tiles * s, pairs) / s;
      const double t = waves + (s > 1 ? (2.0 * s + 1.0) * bytes / 6.0e6 / tile_us : 0.0);
      if (s == 1 || t < 0.97 * best_t) {
        best_t = t;
        best = s;
      }
    }
    if (best == 1) return 1;
    *kb_per = cdiv(num_k, best);
    return cdiv(num_k, *kb_per);
  }
  const int sms = sm_count(dev);
  const int tiles = cdiv(M, gemm::BM) * cdiv(N, gemm::BN);
  // A tile that streams in a few microseconds (under SPLIT_MIN_TILE_KB
  // k-blocks, ~0.27 us each on one SM) is not split: the reduce launch would
  // cost more than the slices save.
  if (2 * tiles > sms || num_k < 2 * SPLIT_MIN_KB || num_k < SPLIT_MIN_TILE_KB) return 1;
  int split = std::min(std::min(num_k / SPLIT_MIN_KB, sms / tiles), SPLIT_MAX);
  *kb_per = cdiv(num_k, split);
  return cdiv(num_k, *kb_per);
}
}  // namespace

namespace {
// Products of at most SWAP_M rows without a mask (the decode step's [batch, C]
// projections) run swapped: D = B . A^T with the weights' rows on the MMA's
// 128-row side and the few activation rows as a SWAP_TN-wide N tile, stored
// transposed into C. The weight rows then fill the tiles (the unswapped tile
// would use 64 of its 128 rows) and the wide projections need no K split.
constexpr int SWAP_M = 64, SWAP_TN = 64;
bool swapped_shape(int M, const void* mask) { return M <= SWAP_M && mask == nullptr; }
}  // namespace

extern "C" size_t mfb_gemm_workspace_size(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  int dev = 0, kb_per = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  // The need of the unmasked product (swapped when M <= SWAP_M); a masked one
  // of so few rows may get fewer slices from it.
  const int split = M <= SWAP_M ? choose_split(N, M, K, dev, &kb_per, true) : choose_split(M, N, K, dev, &kb_per);
  return split > 1 ? sizeof(float) * (size_t)split * M * N : 0;
}

namespace {
// CTA pairs of the pair kernel the device keeps resident at once (0: pairs
// unavailable, run single CTAs). Cached per device.
int pair_clusters(int dev) {
  static int counts[64] = {0};
  if (dev < 0 || dev >= 64) return 0;
  if (counts[dev]) return counts[dev] > 0 ? counts[dev] : 0;
  int n = 0;
  // The largest pair configuration (a staged SwiGLU epilogue): one CTA per SM
  // for every pair configuration.
  auto kernel = gemm::gemm_kernel<true, gemm::EPI_SWIGLU_BWD>;
  constexpr int smem = gemm::Shape<true, gemm::EPI_SWIGLU_BWD>::SMEM;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * (sm_count(dev) / 2));
    cfg.blockDim = dim3(gemm::THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();  // a refused query leaves no sticky error behind
  counts[dev] = n > 0 ? n : -1;
  return n > 0 ? n : 0;
}

// Whether an M-row product runs on CTA pairs: at least two 128-row blocks of
// output and a device that co-schedules the pairs.
bool use_pair(int M, int dev) { return M > gemm::BM && pair_clusters(dev) > 0; }

// Launches gemm_kernel<PAIR, EPI> over a.num_m x a.num_n x a.k_split work
// items (a pair's 256 rows or a CTA's 128 per m block), one persistent CTA or
// CTA pair per SM or SM pair, optionally as a programmatic dependent launch.
template <bool PAIR, int EPI, int TN = gemm::BN>
int launch_kernel(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& te0, const CUtensorMap& te1,
                  const gemm::Args& a, bool pdl, cudaStream_t stream, const char* what) {
  int dev = 0;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  auto kernel = gemm::gemm_kernel<PAIR, EPI, TN>;
  constexpr int smem = gemm::Shape<PAIR, EPI, TN>::SMEM;
  MFB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int tiles = a.num_m * a.num_n * a.k_split;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (PAIR) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 2;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.gridDim = dim3(PAIR ? 2 * std::min(tiles, pair_clusters(dev)) : std::min(tiles, sm_count(dev)));
  cfg.blockDim = dim3(gemm::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  MFB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, ta, tb, te0, te1, a));
  MFB_LAUNCH_CHECK(what);
  return MFB_OK;
}

int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& te0, const CUtensorMap& te1,
                const gemm::Args& a, bool pair, bool pdl, cudaStream_t stream, const char* what) {
  switch (a.epi) {
    case gemm::EPI_SWIGLU_FWD:
      return pair ? launch_kernel<true, gemm::EPI_SWIGLU_FWD>(ta, tb, te0, te1, a, pdl, stream, what)
                  : launch_kernel<false, gemm::EPI_SWIGLU_FWD>(ta, tb, te0, te1, a, pdl, stream, what);
    case gemm::EPI_SWIGLU_BWD:
      return pair ? launch_kernel<true, gemm::EPI_SWIGLU_BWD>(ta, tb, te0, te1, a, pdl, stream, what)
                  : launch_kernel<false, gemm::EPI_SWIGLU_BWD>(ta, tb, te0, te1, a, pdl, stream, what);
    default:
      if (a.swapped) return launch_kernel<false, gemm::EPI_PLAIN, SWAP_TN>(ta, tb, te0, te1, a, pdl, stream, what);
      return pair ? launch_kernel<true, gemm::EPI_PLAIN>(ta, tb, te0, te1, a, pdl, stream, what)
                  : launch_kernel<false, gemm::EPI_PLAIN>(ta, tb, te0, te1, a, pdl, stream, what);
  }
}

// Tensor map of an A operand (K-major [M, K] or MN-major [K, M]).
int make_tmap_a(CUtensorMap* map, const void* A, int a_major, int lda, int M, int K) {
  if (a_major == MFB_MAJOR_K) return tc::make_tmap_bf16(map, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, gemm::BM);
  return tc::make_tmap_bf16(map, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, gemm::BK);
}
// Tensor map of a B operand (K-major [N, K]: boxes of a CTA's B rows; MN-major [K, N]: 64 x 64 boxes).
int make_tmap_b(CUtensorMap* map, const void* B, int b_major, int ldb, int N, int K, bool pair, int rows = 0) {
  if (b_major == MFB_MAJOR_K)
    return tc::make_tmap_bf16(map, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb,
                              rows ? rows
                                   : (pair ? gemm::Shape<true, gemm::EPI_PLAIN>::B_ROWS
                                           : gemm::Shape<false, gemm::EPI_PLAIN>::B_ROWS));
  return tc::make_tmap_bf16(map, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, gemm::BK);
}
}  // namespace

extern "C" int mfb_gemm_bf16(const uint16_t* A, int a_major, int lda, const uint16_t* B, int b_major, int ldb,
                             void* C, int ldc, int out_dtype, int M, int N, int K, float alpha, const uint8_t* mask,
                             void* stream) {
  return mfb_gemm_bf16_ws(A, a_major, lda, B, b_major, ldb, C, ldc, out_dtype, M, N, K, alpha, mask, 0, nullptr, 0,
                          stream);
}

extern "C" int mfb_gemm_bf16_ws(const uint16_t* A, int a_major, int lda, const uint16_t* B, int b_major, int ldb,
                                void* C, int ldc, int out_dtype, int M, int N, int K, float alpha,
                                const uint8_t* mask, int flags, void* workspace, size_t workspace_bytes,
                                void* stream) {
  MFB_CHECK_ARG((flags & ~MFB_GEMM_PDL) == 0, "unknown GEMM flags %d", flags);
  MFB_CHECK_ARG(!(flags & MFB_GEMM_PDL) || stream != nullptr,
                "MFB_GEMM_PDL needs a created stream, not the legacy default stream");
  MFB_CHECK_ARG(M > 0 && N > 0 && K > 0, "GEMM needs nonempty M/N/K (%d, %d, %d)", M, N, K);
  MFB_CHECK_ARG(A && B && C, "NULL operand");
  MFB_CHECK_ARG(a_major == MFB_MAJOR_K || a_major == MFB_MAJOR_MN, "bad a_major");
  MFB_CHECK_ARG(b_major == MFB_MAJOR_K || b_major == MFB_MAJOR_MN, "bad b_major");
  MFB_CHECK_ARG(out_dtype == MFB_DTYPE_BF16 || out_dtype == MFB_DTYPE_F32, "bad out_dtype");
  MFB_CHECK_ARG(lda % 8 == 0 && ldb % 8 == 0, "lda/ldb must be multiples of 8 elements (16-byte TMA strides)");
  MFB_CHECK_ARG(lda >= (a_major == MFB_MAJOR_K ? K : M) && ldb >= (b_major == MFB_MAJOR_K ? K : N), "ld too small");
  MFB_CHECK_ARG(ldc >= N, "ldc must be >= N");
  MFB_CHECK_ARG(((uintptr_t)A & 15) == 0 && ((uintptr_t)B & 15) == 0, "A and B must be 16-byte aligned (TMA)");
  int dev = 0;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  // The kernel computes D[KM, KN]: C itself, or C^T for a swapped product.
  const bool swap = swapped_shape(M, mask);
  const int KM = swap ? N : M, KN = swap ? M : N;
  const uint16_t* KA = swap ? B : A;
  const uint16_t* KB = swap ? A : B;
  const int ka_major = swap ? b_major : a_major, kb_major = swap ? a_major : b_major;
  const int klda = swap ? ldb : lda, kldb = swap ? lda : ldb;
  gemm::Args a{};
  a.C = C;
  a.mask = mask;
  a.ldc = ldc;
  a.M = KM;
  a.N = KN;
  a.K = K;
  a.out_f32 = out_dtype == MFB_DTYPE_F32;
  a.a_mn = ka_major == MFB_MAJOR_MN;
  a.b_mn = kb_major == MFB_MAJOR_MN;
  a.swapped = swap;
  a.num_n = cdiv(KN, swap ? SWAP_TN : gemm::BN);
  a.num_k = cdiv(K, gemm::BK);
  a.alpha = alpha;
  {
    const long long esize = out_dtype == MFB_DTYPE_F32 ? 4 : 2;
    a.vec_ok = ((uintptr_t)C % 16 == 0) && ((long long)ldc * esize) % 16 == 0;
  }
  a.k_split = 1;
  a.kb_per = a.num_k;
  a.partial = nullptr;
  if (workspace) {
    int kb_per = 0;
    int split = choose_split(KM, KN, K, dev, &kb_per, swap);
    const size_t slice = sizeof(float) * (size_t)M * N;
    if (split > 1 && workspace_bytes < slice * split) {  // a smaller workspace gets fewer slices
      split = (int)std::min<size_t>(split, workspace_bytes / slice);
      if (split > 1) {
        kb_per = cdiv(a.num_k, split);
        split = cdiv(a.num_k, kb_per);
      }
    }
    if (split > 1 && ((uintptr_t)workspace & 15) == 0) {
      a.k_split = split;
      a.kb_per = kb_per;
      a.partial = static_cast<float*>(workspace);
    }
  }
  const bool pair = !swap && use_pair(M, dev);
  a.num_m = cdiv(KM, pair ? 2 * gemm::BM : gemm::BM);
  a.n_fast = KM > KN;  // A (KM x K) is the larger operand
  CUtensorMap ta, tb;
  int st = make_tmap_a(&ta, KA, ka_major, klda, KM, K);
  if (st) return st;
  if ((st = make_tmap_b(&tb, KB, kb_major, kldb, KN, K, pair, swap ? SWAP_TN : 0))) return st;
  if ((st = launch_gemm(ta, tb, ta, ta, a, pair, (flags & MFB_GEMM_PDL) != 0, (cudaStream_t)stream,
                        "mfb_gemm_bf16")))
    return st;
  if (a.k_split > 1) {
    const bool vec4 = KN % 4 == 0 && ((uintptr_t)mask & 3) == 0;
    const long long total = (long long)KM * KN / (vec4 ? 4 : 1);
    const int blocks = (int)std::min<long long>((total + 255) / 256, 8LL * sm_count(dev));
    if (vec4)
      gemm::splitk_reduce_kernel<true><<<blocks, 256, 0, (cudaStream_t)stream>>>(a.partial, a.k_split, KM, KN, C,
                                                                                ldc, a.out_f32, alpha, mask, swap);
    else
      gemm::splitk_reduce_kernel<false><<<blocks, 256, 0, (cudaStream_t)stream>>>(a.partial, a.k_split, KM, KN, C,
                                                                                 ldc, a.out_f32, alpha, mask, swap);
    MFB_LAUNCH_CHECK("GEMM split-K reduce");
  }
  return MFB_OK;
}

namespace {
int check_swiglu_operands(const void* A, int a_major, int lda, int M, int F, int K) {
  MFB_CHECK_ARG(M > 0 && F > 0 && K > 0, "SwiGLU GEMM needs nonempty M/F/K (%d, %d, %d)", M, F, K);
  MFB_CHECK_ARG(A != nullptr, "NULL operand");
  MFB_CHECK_ARG(a_major == MFB_MAJOR_K || a_major == MFB_MAJOR_MN, "bad a_major");
  MFB_CHECK_ARG(lda % 8 == 0 && lda >= (a_major == MFB_MAJOR_K ? K : M), "lda must be a multiple of 8 and cover the operand");
  MFB_CHECK_ARG(((uintptr_t)A & 15) == 0, "A must be 16-byte aligned (TMA)");
  return MFB_OK;
}
}  // namespace

extern "C" int mfb_gemm_swiglu_fwd(const uint16_t* A, int a_major, int lda, const uint16_t* W13, int ldw, uint16_t* gu,
                                   uint16_t* h, int M, int F, int K, void* stream) {
  int st = check_swiglu_operands(A, a_major, lda, M, F, K);
  if (st) return st;
  MFB_CHECK_ARG(F % (gemm::BN / 2) == 0, "SwiGLU forward needs F a multiple of %d (F=%d)", gemm::BN / 2, F);
  MFB_CHECK_ARG(W13 && gu && h, "NULL SwiGLU buffer");
  MFB_CHECK_ARG(ldw % 8 == 0 && ldw >= K, "ldw must be a multiple of 8 and >= K");
  MFB_CHECK_ARG((((uintptr_t)W13 | (uintptr_t)gu | (uintptr_t)h) & 15) == 0, "W13, gu and h must be 16-byte aligned");
  int dev = 0;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  const bool pair = use_pair(M, dev);
  CUtensorMap ta, tb;
  if ((st = make_tmap_a(&ta, A, a_major, lda, M, K))) return st;
  if ((st = tc::make_tmap_bf16(&tb, W13, (uint64_t)K, (uint64_t)(2 * F), (uint64_t)ldw, gemm::BN / 2))) return st;
  gemm::Args a{};
  a.C = gu;
  a.ldc = 2LL * F;
  a.M = M;
  a.N = 2 * F;
  a.K = K;
  a.a_mn = a_major == MFB_MAJOR_MN;
  a.b_mn = 0;
  a.num_m = cdiv(M, pair ? 2 * gemm::BM : gemm::BM);
  a.num_n = F / (gemm::BN / 2);
  a.n_fast = M > 2 * F;
  a.num_k = cdiv(K, gemm::BK);
  a.k_split = 1;
  a.kb_per = a.num_k;
  a.alpha = 1.f;
  a.epi = gemm::EPI_SWIGLU_FWD;
  a.F = F;
  a.h = reinterpret_cast<__nv_bfloat16*>(h);
  CUtensorMap tgu = ta, th = ta;  // staged epilogue: gu and h stored by TMA
  if (pair && ((st = tc::make_tmap_bf16_box32(&tgu, gu, 2ull * F, (uint64_t)M, 2ull * F)) ||
               (st = tc::make_tmap_bf16_box32(&th, h, (uint64_t)F, (uint64_t)M, (uint64_t)F))))
    return st;
  return launch_gemm(ta, tb, tgu, th, a, pair, false, (cudaStream_t)stream, "mfb_gemm_swiglu_fwd");
}

extern "C" int mfb_gemm_swiglu_bwd(const uint16_t* dY, int a_major, int lda, const uint16_t* Wd, int b_major, int ldb,
                                   const uint16_t* gu, uint16_t* dgu, int M, int F, int K, void* stream) {
  int st = check_swiglu_operands(dY, a_major, lda, M, F, K);
  if (st) return st;
  MFB_CHECK_ARG(F % 32 == 0, "SwiGLU backward needs F a multiple of 32 (F=%d)", F);
  MFB_CHECK_ARG(Wd && gu && dgu, "NULL SwiGLU buffer");
  MFB_CHECK_ARG(b_major == MFB_MAJOR_K || b_major == MFB_MAJOR_MN, "bad b_major");
  MFB_CHECK_ARG(ldb % 8 == 0 && ldb >= (b_major == MFB_MAJOR_K ? K : F), "ldb must be a multiple of 8 and cover Wd");
  MFB_CHECK_ARG((((uintptr_t)Wd | (uintptr_t)gu | (uintptr_t)dgu) & 15) == 0, "Wd, gu and dgu must be 16-byte aligned");
  MFB_CHECK_ARG(gu != dgu, "dgu must not alias gu");
  int dev = 0;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  const bool pair = use_pair(M, dev);
  CUtensorMap ta, tb;
  if ((st = make_tmap_a(&ta, dY, a_major, lda, M, K))) return st;
  if ((st = make_tmap_b(&tb, Wd, b_major, ldb, F, K, pair))) return st;
  gemm::Args a{};
  a.C = dgu;
  a.ldc = 2LL * F;
  a.M = M;
  a.N = F;
  a.K = K;
  a.a_mn = a_major == MFB_MAJOR_MN;
  a.b_mn = b_major == MFB_MAJOR_MN;
  a.num_m = cdiv(M, pair ? 2 * gemm::BM : gemm::BM);
  a.num_n = cdiv(F, gemm::BN);
  a.n_fast = M > F;
  a.num_k = cdiv(K, gemm::BK);
  a.k_split = 1;
  a.kb_per = a.num_k;
  a.alpha = 1.f;
  a.epi = gemm::EPI_SWIGLU_BWD;
  a.F = F;
  a.gu = reinterpret_cast<const __nv_bfloat16*>(gu);
  CUtensorMap tgu = ta, tdgu = ta;  // staged epilogue: gu loaded and dGU stored by TMA
  if (pair && ((st = tc::make_tmap_bf16_box32(&tgu, gu, 2ull * F, (uint64_t)M, 2ull * F)) ||
               (st = tc::make_tmap_bf16_box32(&tdgu, dgu, 2ull * F, (uint64_t)M, 2ull * F))))
    return st;
  return launch_gemm(ta, tb, tgu, tdgu, a, pair, false, (cudaStream_t)stream, "mfb_gemm_swiglu_bwd");
}

// Reads and clears the GEMM kernels' device status word for the current
// device (nonzero: a bounded wait gave up; the value names which one).
extern "C" int mfb_gemm_status(int* code) {
  MFB_CHECK_ARG(code != nullptr, "code is NULL");
  *code = 0;
  MFB_CUDA_TRY(cudaMemcpyFromSymbol(code, gemm::g_status, sizeof(int)));
  if (*code) {
    const int zero = 0;
    MFB_CUDA_TRY(cudaMemcpyToSymbol(gemm::g_status, &zero, sizeof(int)));
  }
  return MFB_OK;
}
