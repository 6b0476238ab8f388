// Masked GQA flash attention, forward and backward, D = 64.
//
// Replaces the reference's _dense_attention (src/minifield_training/kernels/
// attention.py:12-34) for every mask shape -- causal + key mask, shared prefix,
// packed segments, bidirectional (kernels/bidirectional.py:7-35) and cached --
// through one (qid, kid, causal, offset, policy) encoding: pair (t, s) is valid
// iff qid[t] != 0, qid[t] == kid[s] and (!causal || s <= t + offset).
//
// Layout in HBM (the reference's "bthd" arrays): q/o/dq [B,T,H,D],
// k/v/dk/dv [B,S,Hk,D] bf16; lse [B,H,T] f32 (log2 domain).
//
// Work decomposition: per-64-block id ranges (min/max of nonzero ids,
// "uniform" flag) are built once per call; the tensor-core kernels combine
// them into 128 x 128 (query x key) tile tests, so tile pairs without any
// shared id -- and, when causal, pairs entirely above the diagonal -- are
// skipped before any load ("splash"-style block sparsity), and tiles whose ids
// are uniform and equal skip the per-element mask.
//
// Forward (attn_fwd_tc_kernel): CTA = (128 query rows, the two query heads of
// one KV head, batch row); the heads share every K/V tile (GQA reuse); S, P and
// O live in TMEM (tcgen05), the softmax is FP32 with exp2 and P is rounded to
// bf16 for the PV product (the reference casts probabilities to the query
// dtype, attention.py:31).
// Backward (attn_bwd_tc_kernel): CTA = (128 key rows, KV head, batch row);
// loops over the group's query heads and live query tiles, accumulates dK/dV
// in TMEM (no atomics for the GQA reduction) and dQ in FP32 with TMA tensor
// reduce-adds into the workspace.
#include <math.h>

#include "common.cuh"
#include "tc.cuh"

namespace mfb {
namespace attn {

constexpr int BQ = 64;
constexpr int BK = 64;
constexpr int HD = 64;
constexpr int kIntMax = 0x7fffffff;
constexpr int kIntMin = -0x7fffffff - 1;

struct Range {
  int lo, hi;   // min / max nonzero id in the block (lo > hi: no nonzero id)
  int full;     // all ids in range, equal and nonzero
  int pad;
};

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  float* lse;
  const __nv_bfloat16* d_o;
  float* dsum;
  float* uvec;
  float* dq_acc;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  const int* qid;
  const int* kid;
  const Range* qr;
  const Range* kr;
  const int* order;  // work items of the tensor-core kernel, longest first
  int B, T, S, H, Hk, G;
  int causal, offset, policy;
  int nqb, nkb;
  float scale, scale_log2;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}


// ---------------------------------------------------------------------------
// Id encoding from the reference's mask arguments.
// ---------------------------------------------------------------------------
__global__ void ids_kernel(int mode, const int* __restrict__ mask, const int* __restrict__ seg,
                           const int* __restrict__ aux, int* __restrict__ qid, int* __restrict__ kid, int B, int T,
                           int S, int P) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long nq = (long long)B * T, nk = (long long)B * S;
  if (i < nq) {
    int v = 1;
    if (mode == MFB_MASK_PACKED) {
      const int m = mask[i], sg = seg[i];
      v = (m > 0 && sg != 0) ? sg : 0;  // attention.py:97
    } else if (mode == MFB_MASK_BIDIR && seg != nullptr) {
      const int m = mask[i], sg = seg[i];
      v = (m != 0 && sg != 0) ? sg : 0;  // bidirectional.py:25
    }
    qid[i] = v;
  }
  if (i < nk) {
    const int b = (int)(i / S), s = (int)(i % S);
    int v;
    switch (mode) {
      case MFB_MASK_CAUSAL:
        v = mask[i] != 0;
        break;
      case MFB_MASK_PREFIX:
        v = s < P ? (aux[(long long)b * P + s] != 0) : (mask[(long long)b * T + (s - P)] != 0);
        break;
      case MFB_MASK_PACKED: {
        const int m = mask[i], sg = seg[i];
        v = (m > 0 && sg != 0) ? sg : 0;
        break;
      }
      case MFB_MASK_BIDIR: {
        const int m = mask[i];
        v = seg ? ((m != 0 && seg[i] != 0) ? seg[i] : 0) : (m != 0);
        break;
      }
      default:  // MFB_MASK_CACHED: slots below valid_length
        v = s < aux[b];
        break;
    }
    kid[i] = v;
  }
}

// Per-64-block id ranges for queries (z = 0) and keys (z = 1).
__global__ void ranges_kernel(const int* __restrict__ qid, const int* __restrict__ kid, Range* qr, Range* kr, int B,
                              int T, int S, int nqb, int nkb) {
  const int which = blockIdx.z;
  const int n = which ? S : T;
  const int nb = which ? nkb : nqb;
  const int blk = blockIdx.x, b = blockIdx.y;
  if (blk >= nb) return;
  const int* ids = which ? kid : qid;
  const int pos = blk * 64 + threadIdx.x;
  const int v = pos < n ? ids[(long long)b * n + pos] : 0;
  int lo = v != 0 ? v : kIntMax;
  int hi = v != 0 ? v : kIntMin;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  const int zero = __any_sync(0xffffffffu, v == 0) ? 1 : 0;
  __shared__ int sl[2], sh[2], sz[2];
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sl[w] = lo;
    sh[w] = hi;
    sz[w] = zero;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    Range r;
    r.lo = min(sl[0], sl[1]);
    r.hi = max(sh[0], sh[1]);
    r.full = (!sz[0] && !sz[1] && r.lo == r.hi) ? 1 : 0;
    r.pad = 0;
    (which ? kr : qr)[(long long)b * nb + blk] = r;
  }
}

// ---------------------------------------------------------------------------
// Backward.
// ---------------------------------------------------------------------------

// dsum[b,h,t] = sum_d dO * O; uniform-policy empty rows add dO/S to uvec[b,hk];
// and the row's FP32 dQ accumulator is zeroed for the main kernel's reductions.
// Blocks from `npre` on compute the per-64 id ranges instead (four 64-id
// blocks each, queries then keys: ranges_kernel's work), so that
// latency-bound work overlaps the bandwidth-bound pre-pass.
__global__ void __launch_bounds__(256) attn_bwd_pre_kernel(Params p, const int* __restrict__ qid,
                                                           const int* __restrict__ kid, int npre) {
  if (blockIdx.x >= npre) {
    __shared__ int sl[8], sh[8], sz[8];
    const int grp = threadIdx.x >> 6, half = (threadIdx.x >> 5) & 1;
    const int nqr = p.B * p.nqb, nr = nqr + p.B * p.nkb;
    const int rb = (blockIdx.x - npre) * 4 + grp;
    const bool keys = rb >= nqr;
    const int k = keys ? rb - nqr : rb, nb = keys ? p.nkb : p.nqb, n = keys ? p.S : p.T;
    const int b = k / nb, blk = k % nb;
    const int pos = blk * 64 + (threadIdx.x & 63);
    const int v = (rb < nr && pos < n) ? (keys ? kid : qid)[(long long)b * n + pos] : 0;
    int lo = v != 0 ? v : kIntMax;
    int hi = v != 0 ? v : kIntMin;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    const int zero = __any_sync(0xffffffffu, v == 0) ? 1 : 0;
    if ((threadIdx.x & 31) == 0) {
      sl[2 * grp + half] = lo;
      sh[2 * grp + half] = hi;
      sz[2 * grp + half] = zero;
    }
    __syncthreads();
    if ((threadIdx.x & 63) == 0 && rb < nr) {
      Range r;
      r.lo = min(sl[2 * grp], sl[2 * grp + 1]);
      r.hi = max(sh[2 * grp], sh[2 * grp + 1]);
      r.full = (!sz[2 * grp] && !sz[2 * grp + 1] && r.lo == r.hi) ? 1 : 0;
      r.pad = 0;
      const_cast<Range*>(keys ? p.kr : p.qr)[(long long)b * nb + blk] = r;
    }
    return;
  }
  const long long row = (long long)blockIdx.x * 32 + (threadIdx.x >> 3);  // (b, t, h) flattened as bthd rows
  const int sub = threadIdx.x & 7;
  const long long nrows = (long long)p.B * p.T * p.H;
  const bool ok = row < nrows;
  float acc = 0.f;
  uint4 dov = make_uint4(0, 0, 0, 0);
  if (ok) {
    float4* z = reinterpret_cast<float4*>(p.dq_acc + row * HD + sub * 8);
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    dov = *reinterpret_cast<const uint4*>(p.d_o + row * HD + sub * 8);
    const uint4 ov = *reinterpret_cast<const uint4*>(p.o + row * HD + sub * 8);
    const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&dov);
    const __nv_bfloat162* c = reinterpret_cast<const __nv_bfloat162*>(&ov);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = __bfloat1622float2(a[i]), fc = __bfloat1622float2(c[i]);
      acc += fa.x * fc.x + fa.y * fc.y;
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (ok) {
    const int h = (int)(row % p.H);
    const long long bt = row / p.H;
    const int t = (int)(bt % p.T), b = (int)(bt / p.T);
    const long long li = ((long long)b * p.H + h) * p.T + t;
    if (sub == 0) p.dsum[li] = acc;
    if (p.policy == MFB_EMPTY_UNIFORM && p.lse[li] == -INFINITY) {
      const int hk = h / p.G;
      const __nv_bfloat16* a = reinterpret_cast<const __nv_bfloat16*>(&dov);
      const float inv = 1.f / (float)p.S;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        atomicAdd(p.uvec + ((long long)b * p.Hk + hk) * HD + sub * 8 + i, __bfloat162float(a[i]) * inv);
    }
  }
}

__global__ void __launch_bounds__(256) dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq,
                                                         long long n4, float scale) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const float4 x = reinterpret_cast<const float4*>(acc)[i];
  uint2 o;
  o.x = pack_bf16(x.x * scale, x.y * scale);
  o.y = pack_bf16(x.z * scale, x.w * scale);
  reinterpret_cast<uint2*>(dq)[i] = o;
}

// ---------------------------------------------------------------------------
// Forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// CTA = (128 query rows, the two query heads of one GQA pair, batch row).
// Warp roles (320 threads):
//   warp 0      TMA producer: both Q tiles (thread 0, right after the barrier
//               set-up, so the load overlaps the prologue), then K/V tiles
//               through a 3-stage ring (128 keys x 64 dims, 128-byte swizzle);
//               all lanes stage each key tile's ids and run table.
//   warp 1      TMEM owner and MMA issuer (whole warp, one elected lane).
//   warps 2-5   softmax for query head h0, warps 6-9 for h0 + 1: one thread
//               per query row (TMEM lane quarter = warp % 4), reading its S row
//               with tcgen05.ld; at the end each warp's normalised O rows go
//               into its head's Q buffer and a whole tile leaves as one TMA
//               store per head (a partial tile stores rows).
// Per live key tile j and head g:
//   S_g = Q_g K_j^T           SS MMA, M=128 N=128 K=64 -> TMEM (128 columns)
//   softmax: the thread loads its 128-value S row with one wait, takes the
//   row max, and writes P_g = exp2(S * scale * log2e - M) back as bf16 pairs
//   into the first 64 columns of S_g (tcgen05.st). M is a lazily updated
//   reference max: it moves (and the thread rescales its O row and row sum in
//   TMEM) only when the running max exceeds it by more than 8 (P <= 256).
//   O_g += P_g V_j            TS MMA (A = P from TMEM, B = V MN-major) into a
//                             64-column accumulator.
// Masks: full tiles skip masking; otherwise warp 0 publishes the tile's runs of
// equal nonzero key ids (id, first, last); with at most 8 runs of distinct ids
// a row's valid keys are one interval, else the thread compares ids per key.
// The MMA order S_0(j), S_1(j), PV_0(j), S_0(j+1), PV_1(j), S_1(j+1), ... lets
// one head's softmax run while the other head's products are on the tensor
// core. TMEM: S_0 [0,128) O_0 [128,192) S_1 [256,384) O_1 [384,448).
// ---------------------------------------------------------------------------
__device__ int g_tc_status;

constexpr int TQ = 128, TK = 128;
constexpr int TF_HPB = 2;  // query heads per CTA: the two heads of a GQA pair share K/V
constexpr int TF_ST = 3;
constexpr int TF_THREADS = 320;
constexpr int TF_Q_OFF = 0;
constexpr int TF_K_OFF = 2 * 16384;
constexpr int TF_V_OFF = TF_K_OFF + TF_ST * 16384;
constexpr int TF_V_STRIDE = 16384;
// One constant "ones" MN atom (128 key rows x 64 columns, column 0 = 1.0;
// 16 KB) shared by every V stage: the PV product runs with N = 80 and each
// stage's B descriptor points its second MN atom here (LBO = ONES - V stage),
// so column 64 of O accumulates the row sum of P.
constexpr int TF_ONES_OFF = TF_V_OFF + TF_ST * TF_V_STRIDE;
constexpr int TF_KID_OFF = TF_ONES_OFF + 16384;
// Per stage: 128 key ids, then the run table (count, 8 x {id, first, last}).
constexpr int TF_KID_STRIDE = 128 + 32;
constexpr int TF_MAX_RUNS = 8;
constexpr int TF_LIST_OFF = TF_KID_OFF + TF_ST * TF_KID_STRIDE * 4;
constexpr int TF_MAX_TILES = 256;  // key tiles per row: S <= 32768
constexpr int TF_BAR_OFF = TF_LIST_OFF + (TF_MAX_TILES + 4) * 4;
constexpr int TF_ON = 80;  // PV product width: 64 value columns + the ones column block
constexpr int TF_SMEM = 1024 + TF_BAR_OFF + 256;

// 128-row tile range from the two 64-row block ranges it covers.
__device__ __forceinline__ Range range128(const Range* r, int nb64, int tile) {
  const Range a = r[2 * tile];
  Range out = a;
  if (2 * tile + 1 < nb64) {
    const Range c = r[2 * tile + 1];
    out.lo = min(a.lo, c.lo);
    out.hi = max(a.hi, c.hi);
    out.full = a.full && c.full && a.lo == c.lo;
  } else {
    out.full = 0;
  }
  return out;
}

__device__ __forceinline__ bool tile_live128(const Params& p, const Range& qr, const Range& kr, int q0, int s0) {
  if (p.causal && s0 > min(q0 + TQ - 1, p.T - 1) + p.offset) return false;
  return max(qr.lo, kr.lo) <= min(qr.hi, kr.hi);
}

__device__ __forceinline__ bool tile_full128(const Params& p, const Range& qr, const Range& kr, int q0, int s0) {
  if (!qr.full || !kr.full || qr.lo != kr.lo) return false;
  return !(p.causal && s0 + TK - 1 > q0 + p.offset);
}

// 10 warps: the sub-partitions holding 3 warps cap registers at 168 per thread.
__global__ void __launch_bounds__(TF_THREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to, Params p) {
  extern __shared__ uint8_t smem_raw[];
  // Offset from the __shared__ array itself so accesses keep the shared state space.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(smem);
  const uint32_t bars = sb + TF_BAR_OFF;
  const uint32_t q_full = bars;
  auto kv_full = [&](int s) { return bars + 8u * (1 + s); };
  auto kv_empty = [&](int s) { return bars + 8u * (1 + TF_ST + s); };
  auto s_full = [&](int g) { return bars + 8u * (1 + 2 * TF_ST + g); };
  auto p_full = [&](int g) { return bars + 8u * (3 + 2 * TF_ST + g); };
  auto o_full = [&](int g) { return bars + 8u * (5 + 2 * TF_ST + g); };
  const uint32_t done_bar = bars + 8u * (7 + 2 * TF_ST);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TF_BAR_OFF + 8 * (8 + 2 * TF_ST));
  int* kid_s = reinterpret_cast<int*>(smem + TF_KID_OFF);
  int* list = reinterpret_cast<int*>(smem + TF_LIST_OFF);  // [0] = count, then tile | full << 30

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work item (query tile, batch row) from the longest-first order; the head
  // pairs of one item are adjacent launches (they share K/V tiles in L2).
  const int hpairs = p.H / TF_HPB;
  const int item = p.order[blockIdx.x / hpairs];
  const int qt = item % cdiv(p.T, TQ), b = item / cdiv(p.T, TQ);
  const int h0 = (blockIdx.x % hpairs) * TF_HPB;
  const int hk = h0 / p.G;
  const int q0 = qt * TQ;
  const int nkt = cdiv(p.S, TK);
  const Range qrange = range128(p.qr + (long long)b * p.nqb, p.nqb, qt);
  const Range* krs = p.kr + (long long)b * p.nkb;
  int* status = &g_tc_status;

  if (threadIdx.x == 0) {
    tc::mbar_init(q_full, 1);
    for (int s = 0; s < TF_ST; ++s) {
      tc::mbar_init(kv_full(s), 1 + 32);
      tc::mbar_init(kv_empty(s), 1);
    }
    for (int g = 0; g < 2; ++g) {
      tc::mbar_init(s_full(g), 1);
      tc::mbar_init(p_full(g), 128);
      tc::mbar_init(o_full(g), 1);
    }
    tc::mbar_init(done_bar, 1);
    tc::mbar_fence_init();
    // Q does not depend on the live-tile list: its load overlaps the prologue.
    tc::mbar_expect_tx(q_full, 2 * 16384);
    tc::tma_load_2d(sb + TF_Q_OFF, &tq, h0 * 64, b * p.T + q0, q_full);
    tc::tma_load_2d(sb + TF_Q_OFF + 16384, &tq, (h0 + 1) * 64, b * p.T + q0, q_full);
  }
  if (warp == 0) {
    // Live key tiles of this query tile, in order, with their "no mask" flag.
    int count = 0;
    for (int base = 0; base < nkt; base += 32) {
      const int j = base + lane;
      bool live = false, full = false;
      if (j < nkt) {
        const Range kr = range128(krs, p.nkb, j);
        live = tile_live128(p, qrange, kr, q0, j * TK);
        full = live && tile_full128(p, qrange, kr, q0, j * TK);
      }
      const unsigned bal = __ballot_sync(0xffffffffu, live);
      if (live) list[1 + count + __popc(bal & ((1u << lane) - 1))] = j | (full ? 1 << 30 : 0);
      count += __popc(bal);
    }
    if (lane == 0) list[0] = count;
  } else if (warp == 1) {
    tc::tmem_alloc(smem_u32(tmem_slot), 512);
    tc::tmem_relinquish();
  } else {
    // The constant ones atom: column 0 of each of its 128 rows is 1.0.
    for (int i = threadIdx.x - 64; i < 128 * 8; i += TF_THREADS - 64) {
      const int row = i / 8, chunk = i % 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (chunk == (row & 7)) v.x = 0x3F80u;  // logical chunk 0 lands at physical chunk row % 8
      *reinterpret_cast<uint4*>(smem + TF_ONES_OFF + row * 128 + chunk * 16) = v;
    }
    tc::fence_proxy_async_smem();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = list[0];

  if (warp == 0) {
    if (lane == 0) {
      tc::tma_prefetch_desc(&tq);
      tc::tma_prefetch_desc(&tk);
      tc::tma_prefetch_desc(&tv);
    }
    for (int it = 0; it < ntiles; ++it) {
      const int j = list[1 + it] & 0xFFFF;
      const int st = it % TF_ST;
      const uint32_t ph = (it / TF_ST) & 1;
      if (!tc::mbar_wait(kv_empty(st), ph ^ 1, status, 11)) break;
      if (lane == 0) {
        tc::mbar_expect_tx(kv_full(st), 2 * 16384);
        tc::tma_load_2d(sb + TF_K_OFF + st * 16384, &tk, hk * 64, b * p.S + j * TK, kv_full(st));
        tc::tma_load_2d(sb + TF_V_OFF + st * TF_V_STRIDE, &tv, hk * 64, b * p.S + j * TK, kv_full(st));
      }
      // Key ids and their run table: (id, first, last) of each run of equal
      // nonzero ids; count -1 when an id recurs or there are more than 8 runs.
      int* kt = kid_s + st * TF_KID_STRIDE;
      int kv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int s = j * TK + 4 * lane + e;
        kv[e] = s < p.S ? p.kid[(long long)b * p.S + s] : 0;
        kt[4 * lane + e] = kv[e];
      }
      const int prev = __shfl_up_sync(0xffffffffu, kv[3], 1);
      const int next = __shfl_down_sync(0xffffffffu, kv[0], 1);
      unsigned sbits = 0, ebits = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int before = e == 0 ? (lane == 0 ? 0 : prev) : kv[e - 1];
        const int after = e == 3 ? (lane == 31 ? 0 : next) : kv[e + 1];
        if (kv[e] != 0 && (e + lane == 0 || before != kv[e])) sbits |= 1u << e;
        if (kv[e] != 0 && ((e == 3 && lane == 31) || after != kv[e])) ebits |= 1u << e;
      }
      const int ns = __popc(sbits), ne = __popc(ebits);
      int incl_s = ns, incl_e = ne;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int ys = __shfl_up_sync(0xffffffffu, incl_s, o), ye = __shfl_up_sync(0xffffffffu, incl_e, o);
        if (lane >= o) incl_s += ys, incl_e += ye;
      }
      const int total = __shfl_sync(0xffffffffu, incl_s, 31);
      int* rt = kt + 128;
      if (total <= TF_MAX_RUNS) {
        int is = incl_s - ns, ie = incl_e - ne;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (sbits & (1u << e)) {
            rt[1 + 3 * is] = kv[e];
            rt[2 + 3 * is] = 4 * lane + e;
            ++is;
          }
          if (ebits & (1u << e)) {
            rt[3 + 3 * ie] = 4 * lane + e;
            ++ie;
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        int cnt = total <= TF_MAX_RUNS ? total : -1;
        for (int a = 0; cnt > 0 && a < total; ++a)
          for (int c = a + 1; c < total; ++c)
            if (rt[1 + 3 * a] == rt[1 + 3 * c]) cnt = -1;
        rt[0] = cnt;
      }
      __syncwarp();
      tc::mbar_arrive(kv_full(st));
    }
  } else if (warp == 1) {
    // The whole warp runs the issue loop (converged); one elected lane issues.
    {
      const uint32_t idesc_s = tc::idesc_bf16_f32(128, 128, 0, 0);
      const uint32_t idesc_o = tc::idesc_bf16_f32(128, TF_ON, 0, 1);
      bool ok = tc::mbar_wait_w(q_full, 0, status, 13);
      tc::tc_fence_after();
      int it = 0, prev = -1;
      for (; ok && it < ntiles; ++it) {
        const int st = it % TF_ST;
        if (!(ok = tc::mbar_wait_w(kv_full(st), (it / TF_ST) & 1, status, 14))) break;
        tc::tc_fence_after();
        for (int g = 0; g < 2; ++g) {
          const uint32_t s_t = tmem + g * 256, o_t = tmem + g * 256 + 128;
          if (it > 0) {
            if (!(ok = tc::mbar_wait_w(p_full(g), (it - 1) & 1, status, 15))) break;
            tc::tc_fence_after();
            const uint32_t vb = sb + TF_V_OFF + prev * TF_V_STRIDE;
#pragma unroll
            for (int k = 0; k < TK / 16; ++k)
              tc::mma_bf16_ts_w(o_t, s_t + k * 8, tc::smem_desc_sw128(vb + k * 2048, TF_ONES_OFF - TF_V_OFF - prev * TF_V_STRIDE, 1024), idesc_o,
                              (it > 1 || k > 0) ? 1u : 0u);
          }
          const uint32_t qb_ = sb + TF_Q_OFF + g * 16384, kb_ = sb + TF_K_OFF + st * 16384;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc::mma_bf16_w(s_t, tc::smem_desc_sw128(qb_ + k * 32, 16, 1024), tc::smem_desc_sw128(kb_ + k * 32, 16, 1024),
                         idesc_s, k > 0 ? 1u : 0u);
          tc::mma_commit_w(s_full(g));
        }
        if (!ok) break;
        if (it > 0) tc::mma_commit_w(kv_empty(prev));
        prev = st;
      }
      if (ok && it > 0) {
        for (int g = 0; g < 2; ++g) {
          const uint32_t s_t = tmem + g * 256, o_t = tmem + g * 256 + 128;
          if (!tc::mbar_wait_w(p_full(g), (it - 1) & 1, status, 16)) break;
          tc::tc_fence_after();
          const uint32_t vb = sb + TF_V_OFF + prev * TF_V_STRIDE;
#pragma unroll
          for (int k = 0; k < TK / 16; ++k)
            tc::mma_bf16_ts_w(o_t, s_t + k * 8, tc::smem_desc_sw128(vb + k * 2048, TF_ONES_OFF - TF_V_OFF - prev * TF_V_STRIDE, 1024), idesc_o,
                            (it > 1 || k > 0) ? 1u : 0u);
          tc::mma_commit_w(o_full(g));
        }
      }
      tc::mma_commit_w(done_bar);
      tc::mbar_wait_w(done_bar, 0, status, 17);
    }
  } else {
    const int g = (warp - 2) >> 2, quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int t = q0 + r;
    const int h = h0 + g;
    const int qid_row = t < p.T ? p.qid[(long long)b * p.T + t] : 0;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_t = tmem + lane_off + g * 256, o_t = tmem + lane_off + g * 256 + 128;
    const float sl2 = p.scale_log2;
    float M = -INFINITY;  // reference max of the scaled logits (log2 domain)
    int it = 0;
    bool ok = true;
    for (; it < ntiles; ++it) {
      const int entry = list[1 + it];
      const int j = entry & 0xFFFF;
      const bool full = (entry >> 30) & 1;
      const int st = it % TF_ST;
      // Wait outcomes are made warp-uniform: the TMEM accesses below are
      // warp-collective.
      ok = tc::mbar_wait(s_full(g), it & 1, status, 18);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      ok = tc::mbar_wait(kv_full(st), (it / TF_ST) & 1, status, 19);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc::tc_fence_after();
      const int s0 = j * TK;
      uint32_t x[TK];
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::tmem_ld_32x32b_x32(s_t + c * 32, x + c * 32);
      tc::tmem_ld_wait();
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
      const uint32_t NEG = 0xFF800000u;  // -inf
      if (full) {
#pragma unroll
        for (int i = 0; i < TK; i += 4) {
          mx0 = fmaxf(mx0, __uint_as_float(x[i]));
          mx1 = fmaxf(mx1, __uint_as_float(x[i + 1]));
          mx2 = fmaxf(mx2, __uint_as_float(x[i + 2]));
          mx3 = fmaxf(mx3, __uint_as_float(x[i + 3]));
        }
      } else {
        const int* kt = kid_s + st * TF_KID_STRIDE;
        const int nr = kt[128];
        int lo = 1, hi = 0;
        if (nr >= 0) {
          for (int q = 0; q < nr; ++q)
            if (kt[129 + 3 * q] == qid_row) lo = kt[130 + 3 * q], hi = kt[131 + 3 * q];
        } else {
          lo = 0, hi = TK - 1;
        }
        if (p.causal) hi = min(hi, t + p.offset - s0);
        // Validity bits per 32-key chunk, then one branch-free masking pass.
        uint32_t vm[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int a0 = max(lo - c * 32, 0), b0 = min(hi - c * 32, 31);
          vm[c] = a0 > b0 ? 0u : ((0xFFFFFFFFu >> (31 - b0)) & (0xFFFFFFFFu << a0));
        }
        if (nr < 0) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t bits = 0;
            for (int i = 0; i < 32; ++i) bits |= (qid_row != 0 && kt[c * 32 + i] == qid_row) ? 1u << i : 0u;
            vm[c] &= bits;
          }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const int k = c * 32 + i;
            x[k] = (vm[c] >> i) & 1u ? x[k] : NEG;
            x[k + 1] = (vm[c] >> (i + 1)) & 1u ? x[k + 1] : NEG;
            x[k + 2] = (vm[c] >> (i + 2)) & 1u ? x[k + 2] : NEG;
            x[k + 3] = (vm[c] >> (i + 3)) & 1u ? x[k + 3] : NEG;
            mx0 = fmaxf(mx0, __uint_as_float(x[k]));
            mx1 = fmaxf(mx1, __uint_as_float(x[k + 1]));
            mx2 = fmaxf(mx2, __uint_as_float(x[k + 2]));
            mx3 = fmaxf(mx3, __uint_as_float(x[k + 3]));
          }
        }
      }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
      // Lazy rescale: a row whose max rose by more than 2^8 moves its
      // reference max and rescales its O accumulator (column 64 holds the row
      // sum); the previous products have landed (s_full follows them).
      // tcgen05.ld/st are warp-collective, so the warp rescales together when
      // any of its rows moves; the other rows scale by exactly 1.
      const bool up = mx > M + 8.f;
      if (it > 0 && __any_sync(0xffffffffu, up && M != -INFINITY)) {
        const float sc = (up && M != -INFINITY) ? ex2(M - mx) : 1.f;
#pragma unroll
        for (int c = 0; c < TF_ON / 16; ++c) {
          uint32_t v[16];
          tc::tmem_ld_32x32b_x16(o_t + c * 16, v);
          tc::tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * sc);
          tc::tmem_st_32x32b_x16(o_t + c * 16, v);
        }
      }
      if (up) M = mx;
      const float nmu = M == -INFINITY ? 0.f : -M;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float e0 = ex2(fmaf(__uint_as_float(x[c * 32 + i]), sl2, nmu));
          const float e1 = ex2(fmaf(__uint_as_float(x[c * 32 + i + 1]), sl2, nmu));
          pk[i >> 1] = pack_bf16(e0, e1);
        }
        tc::tmem_st_32x32b_x16(s_t + c * 16, pk);
      }
      tc::tmem_st_wait();
      tc::tc_fence_before();
      tc::mbar_arrive(p_full(g));
    }
    uint32_t ou[64];
    float l = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) ou[i] = 0u;
    const bool o_ready = ok && it > 0 && tc::mbar_wait(o_full(g), 0, status, 20);
    if (__all_sync(0xffffffffu, o_ready)) {
      tc::tc_fence_after();
      uint32_t lv[16];
      tc::tmem_ld_32x32b_x32(o_t, ou);
      tc::tmem_ld_32x32b_x32(o_t + 32, ou + 32);
      tc::tmem_ld_32x32b_x16(o_t + 64, lv);
      tc::tmem_ld_wait();
      l = __uint_as_float(lv[0]);
    }
    // Epilogue: normalise; rows without a valid key follow the empty policy.
    const bool empty = !(l > 0.f);
    const float inv = empty ? 0.f : 1.f / l;
    const bool need_uniform = p.policy == MFB_EMPTY_UNIFORM && __any_sync(0xffffffffu, empty && t < p.T);
    float vm0 = 0.f, vm1 = 0.f;
    if (need_uniform) {
      const __nv_bfloat16* vbase = p.v + ((long long)b * p.S * p.Hk + hk) * HD;
      for (int s = 0; s < p.S; ++s) {
        const __nv_bfloat162 v2 = *reinterpret_cast<const __nv_bfloat162*>(vbase + (long long)s * p.Hk * HD + 2 * lane);
        vm0 += __bfloat162float(v2.x);
        vm1 += __bfloat162float(v2.y);
      }
      vm0 /= (float)p.S;
      vm1 /= (float)p.S;
    }
    // Normalised bf16 pairs, packed in place into ou[0, 32).
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      float a0 = __uint_as_float(ou[2 * e]) * inv, a1 = __uint_as_float(ou[2 * e + 1]) * inv;
      if (need_uniform) {
        const float u0 = __shfl_sync(0xffffffffu, vm0, e), u1 = __shfl_sync(0xffffffffu, vm1, e);
        if (empty) a0 = u0, a1 = u1;
      }
      ou[e] = pack_bf16(a0, a1);
    }
    if (t < p.T) p.lse[((long long)b * p.H + h) * p.T + t] = empty ? -INFINITY : M + __log2f(l);
    if (q0 + TQ <= p.T) {
      // Whole tile: rows into the head's Q buffer (every product that read it
      // has completed: o_full follows them) in the TMA tile layout, then one
      // TMA store per head. All eight softmax warps reach the barrier. A tile
      // without live key tiles issues no products, so nothing else has waited
      // for the Q load that could still land on the staged rows: wait for it.
      tc::mbar_wait(q_full, 0, status, 22);
      uint8_t* stage = smem + TF_Q_OFF + g * 16384;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        *reinterpret_cast<uint4*>(stage + r * 128 + ((c8 ^ (r & 7)) << 4)) =
            make_uint4(ou[4 * c8], ou[4 * c8 + 1], ou[4 * c8 + 2], ou[4 * c8 + 3]);
      tc::fence_proxy_async_smem();
      asm volatile("bar.sync 1, 256;\n" ::: "memory");
      if (warp == 2 && lane == 0) {
        tc::tma_store_2d(&to, sb + TF_Q_OFF, h0 * 64, b * p.T + q0);
        tc::tma_store_2d(&to, sb + TF_Q_OFF + 16384, (h0 + 1) * 64, b * p.T + q0);
        tc::bulk_commit_group();
        tc::bulk_wait_group_read0();  // the staging must outlive the reads; the writes complete with the grid
      }
    } else if (t < p.T) {
      __nv_bfloat16* orow = p.o + (((long long)b * p.T + t) * p.H + h) * HD;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        *reinterpret_cast<uint4*>(orow + c8 * 8) = make_uint4(ou[4 * c8], ou[4 * c8 + 1], ou[4 * c8 + 2], ou[4 * c8 + 3]);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Backward on tcgen05.
//
// CTA = (128 keys, one KV head, batch row); it loops over the group's query
// heads x live 128-row query tiles ("items"), each split into two 64-query
// sub-items so the tensor core works on one sub-item while the
// softmax-gradient warps work on the other. Warp roles (704 threads):
//   warp 0      producer: K and V once (thread 0, right after the barrier
//               set-up, so the load overlaps the prologue); per item the Q and
//               dO tiles (TMA, three stages; item 0's as soon as the warp has
//               built the item list) and the per-query lse, dsum and query id
//               (loaded one item ahead).
//   warp 1      TMEM owner and MMA issuer (whole warp, one elected lane).
//   warps 2-17  softmax-gradient, two groups of eight taking alternate
//               sub-items (half 0 / half 1 of every item): one key row (TMEM
//               lane) per thread, 32 of the sub-item's 64 query columns per
//               warp, two warps of a group per TMEM lane quarter. Prologue: K
//               and V rows into TMEM; epilogue: dK/dV rows into the first Q/dO
//               stage, out as two TMA stores (partial tiles store rows).
//   warps 18-21 dQ flush: add each item's dQ tile into the FP32 accumulator
//               while the next item is computed: TMEM -> swizzled shared
//               staging -> TMA tensor reduce-add (the reductions run in the
//               TMA unit and L2, off the SM's load/store path that the
//               mbarrier polls and the shared-memory traffic share).
// Products (M = 128 keys unless noted), issued in the order
//   S/dP(j), [dQ tile free] dQ(item pending), [P ready j-1] dV/dK(j-1), S/dP(j+1)...
//   S^T_j  = K Q_j^T        TS (K from TMEM), N = 64 -> TMEM buffer j%2 [0,64)
//   dP^T_j = V dO_j^T       TS (V from TMEM), N = 64 -> TMEM buffer j%2 [64,128)
//   P^T_j (bf16) goes back into its warp's own consumed S^T columns; dS^T_j
//   (bf16) into shared memory (128-byte swizzle, item parity buffer, 64-query
//   atom per sub-item).
//   dV += P^T_j dO_j        TS (A from TMEM) -> TMEM [256,320)
//   dK += dS^T_j Q_j        SS               -> TMEM [320,384)
//   dQ  = dS K              SS, A = the item's dS^T read MN-major (M = 128
//                           queries), after both sub-items -> TMEM [384,448)
// ---------------------------------------------------------------------------
constexpr int TB_ST = 3;
// Softmax-gradient warps per TMEM lane quarter (TB_SMW), in two groups that
// take alternate sub-items (group g the sub-items of half g of every item, so
// one group computes while the other waits for its scores); each warp handles
// TB_PW query columns of its sub-items. TB_CW = the head dims (and K/V
// columns) each of a quarter's warps covers in the prologue and epilogue.
// Warp roles: producer, MMA issuer, 4 * TB_SMW softmax-gradient warps, 4 dQ
// flush warps.
constexpr int TB_SMW = 4;
constexpr int TB_PW = 128 / TB_SMW;
constexpr int TB_CW = 64 / TB_SMW;
constexpr int TB_SM_WARPS = 4 * TB_SMW;
constexpr int TB_THREADS = (2 + TB_SM_WARPS + 4) * 32;
constexpr int TB_K_OFF = 0;
constexpr int TB_V_OFF = 16384;
constexpr int TB_QD_OFF = 32768;  // stage st: Q at +st*32768, dO at +st*32768+16384
constexpr int TB_DS_OFF = TB_QD_OFF + TB_ST * 32768;  // two 32 KB dS^T buffers (item parity)
constexpr int TB_COL_OFF = TB_DS_OFF + 2 * 32768;
// Per stage: lse[128], dsum[128], qid[128], then per 16-query chunk its id
// (valid when the chunk's bit in the mask word that follows is set: all 16
// queries share it).
constexpr int TB_COL_STRIDE = 3 * 128 + 8 + 8;
constexpr int TB_LIST_OFF = TB_COL_OFF + TB_ST * TB_COL_STRIDE * 4;
constexpr int TB_BAR_OFF = TB_LIST_OFF + (TF_MAX_TILES + 4) * 4;
// TMEM columns of the backward: S^T/dP^T double buffer [0,256), dV [256,320),
// dK [320,384), dQ [384,448), K [448,480) and V [480,512) (bf16 pairs).
constexpr int TB_KT_COL = 448, TB_VT_COL = 480;
// dQ staging: one 4 KB box (32 query rows x 32 FP32 columns, 128-byte
// swizzle) per dQ flush warp, 1024-byte aligned for the TMA reduction.
constexpr int TB_DQS_OFF = (TB_BAR_OFF + 256 + 1023) / 1024 * 1024;
constexpr int TB_SMEM = 1024 + TB_DQS_OFF + 4 * 4096;
static_assert(TB_SMEM <= 227 * 1024, "backward shared memory");

// P and dS for one key row and N query columns: p = 2^(s*scale*log2e - lse)
// (zero where the query's id differs from the key row's, or before the
// causal first column), ds = p * (dp - dsum); both packed to bf16 pairs. DENSE skips
// the mask (the whole tile is valid). A key row with id 0 needs no test of its
// own: only inactive queries carry id 0, and their lse is +inf (p = 0).
template <bool DENSE, int N>
__device__ __forceinline__ void ds_chunk(const uint32_t (&sx)[N], const uint32_t (&dx)[N], const float* lse_s,
                                         const float* dsum_s, const int* qid_s, int kid_row, int cfirst, float sl2,
                                         uint32_t (&pk)[N / 2], uint32_t (&dk4)[N / 2]) {
#pragma unroll
  for (int i = 0; i < N; i += 4) {
    const float4 l4 = *reinterpret_cast<const float4*>(lse_s + i);
    const float4 d4 = *reinterpret_cast<const float4*>(dsum_s + i);
    const float ls[4] = {l4.x, l4.y, l4.z, l4.w}, dsm[4] = {d4.x, d4.y, d4.z, d4.w};
    int qd[4] = {0, 0, 0, 0};
    if (!DENSE) {
      const int4 q4 = *reinterpret_cast<const int4*>(qid_s + i);
      qd[0] = q4.x, qd[1] = q4.y, qd[2] = q4.z, qd[3] = q4.w;
    }
    float pv[4], dv4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float pe = ex2(fmaf(__uint_as_float(sx[i + e]), sl2, -ls[e]));
      pv[e] = DENSE ? pe : ((qd[e] == kid_row && i + e >= cfirst) ? pe : 0.f);
      dv4[e] = pv[e] * (__uint_as_float(dx[i + e]) - dsm[e]);
    }
    pk[i >> 1] = pack_bf16(pv[0], pv[1]);
    pk[(i >> 1) + 1] = pack_bf16(pv[2], pv[3]);
    dk4[i >> 1] = pack_bf16(dv4[0], dv4[1]);
    dk4[(i >> 1) + 1] = pack_bf16(dv4[2], dv4[3]);
  }
}

__global__ void __launch_bounds__(TB_THREADS, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                       const __grid_constant__ CUtensorMap tdq, const __grid_constant__ CUtensorMap tdk,
                       const __grid_constant__ CUtensorMap tdv, Params p) {
  extern __shared__ uint8_t smem_raw[];
  // Offset from the __shared__ array itself so accesses keep the shared state space.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(smem);
  const uint32_t bars = sb + TB_BAR_OFF;
  const uint32_t kv_full = bars;
  auto qd_full = [&](int s) { return bars + 8u * (1 + s); };
  auto qd_empty = [&](int s) { return bars + 8u * (1 + TB_ST + s); };
  auto s_full = [&](int u) { return bars + 8u * (1 + 2 * TB_ST + u); };
  auto p_full = [&](int u) { return bars + 8u * (3 + 2 * TB_ST + u); };
  const uint32_t dq_full = bars + 8u * (5 + 2 * TB_ST);
  const uint32_t dq_free = bars + 8u * (6 + 2 * TB_ST);
  const uint32_t done_bar = bars + 8u * (7 + 2 * TB_ST);
  const uint32_t kv_tm = bars + 8u * (8 + 2 * TB_ST);  // K and V copied into TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TB_BAR_OFF + 8 * (9 + 2 * TB_ST));
  int* cols = reinterpret_cast<int*>(smem + TB_COL_OFF);
  int* list = reinterpret_cast<int*>(smem + TB_LIST_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work item (key tile, batch row) from the longest-first order; the KV heads
  // of one item are adjacent launches.
  const int item = p.order[blockIdx.x / p.Hk];
  const int kt = item % cdiv(p.S, TK), b = item / cdiv(p.S, TK), hk = blockIdx.x % p.Hk;
  const int s0 = kt * TK;
  const int ntq = cdiv(p.T, TQ);
  const Range krange = range128(p.kr + (long long)b * p.nkb, p.nkb, kt);
  const Range* qrs = p.qr + (long long)b * p.nqb;
  int* status = &g_tc_status;

  if (threadIdx.x == 0) {
    tc::mbar_init(kv_full, 1);
    for (int s = 0; s < TB_ST; ++s) {
      tc::mbar_init(qd_full(s), 1 + 32);
      tc::mbar_init(qd_empty(s), 1);
    }
    for (int u = 0; u < 2; ++u) {
      tc::mbar_init(s_full(u), 1);
      tc::mbar_init(p_full(u), 32 * TB_SM_WARPS / 2);
    }
    tc::mbar_init(dq_full, 1);
    tc::mbar_init(dq_free, 128);
    tc::mbar_init(done_bar, 1);
    tc::mbar_init(kv_tm, 32 * TB_SM_WARPS);
    tc::mbar_fence_init();
    // K and V do not depend on the item list: their load overlaps the prologue.
    tc::mbar_expect_tx(kv_full, 2 * 16384);
    tc::tma_load_2d(sb + TB_K_OFF, &tk, hk * 64, b * p.S + s0, kv_full);
    tc::tma_load_2d(sb + TB_V_OFF, &tv, hk * 64, b * p.S + s0, kv_full);
  }
  if (warp == 0) {
    int count = 0;
    for (int base = 0; base < ntq; base += 32) {
      const int i = base + lane;
      bool live = false, full = false;
      if (i < ntq) {
        const Range qr = range128(qrs, p.nqb, i);
        live = tile_live128(p, qr, krange, i * TQ, s0);
        full = live && tile_full128(p, qr, krange, i * TQ, s0);
      }
      const unsigned bal = __ballot_sync(0xffffffffu, live);
      if (live) list[1 + count + __popc(bal & ((1u << lane) - 1))] = i | (full ? 1 << 30 : 0);
      count += __popc(bal);
    }
    if (lane == 0) list[0] = count;
    __syncwarp();
    if (lane == 0 && count > 0) {  // item 0's Q and dO: the load overlaps the rest of the prologue
      const int q0 = (list[1] & 0xFFFF) * TQ;
      tc::mbar_expect_tx(qd_full(0), 2 * 16384);
      tc::tma_load_2d(sb + TB_QD_OFF, &tq, (hk * p.G) * 64, b * p.T + q0, qd_full(0));
      tc::tma_load_2d(sb + TB_QD_OFF + 16384, &tdo, (hk * p.G) * 64, b * p.T + q0, qd_full(0));
    }
  } else if (warp == 1) {
    tc::tmem_alloc(smem_u32(tmem_slot), 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nlive = list[0];
  const int nitems = p.G * nlive;

  if (warp == 0) {
    if (lane == 0) {
      tc::tma_prefetch_desc(&tq);
      tc::tma_prefetch_desc(&tk);
      tc::tma_prefetch_desc(&tv);
      tc::tma_prefetch_desc(&tdo);
    }
    // Column data (lse, dsum, query id) of an item, loaded one item ahead so
    // that the global-load latency overlaps the wait for a free stage.
    float cl[4], cd[4];
    int cq[4];
    auto load_cols = [&](int it) {
      const int h = hk * p.G + it / nlive;
      const int q0 = (list[1 + it % nlive] & 0xFFFF) * TQ;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = q0 + 4 * lane + e;
        const long long li = ((long long)b * p.H + h) * p.T + t;
        cl[e] = INFINITY, cd[e] = 0.f, cq[e] = 0;
        if (t < p.T) {
          cl[e] = p.lse[li];
          cd[e] = p.dsum[li];
          cq[e] = p.qid[(long long)b * p.T + t];
        }
      }
    };
    if (nitems > 0) load_cols(0);
    for (int it = 0; it < nitems; ++it) {
      const int st = it % TB_ST;
      const uint32_t ph = (it / TB_ST) & 1;
      const int h = hk * p.G + it / nlive;
      const int entry = list[1 + it % nlive];
      const int q0 = (entry & 0xFFFF) * TQ;
      if (!tc::mbar_wait(qd_empty(st), ph ^ 1, status, 31)) break;
      if (lane == 0 && it > 0) {  // item 0's tiles were requested before the prologue barrier
        const uint32_t qb_ = sb + TB_QD_OFF + st * 32768;
        tc::mbar_expect_tx(qd_full(st), 2 * 16384);
        tc::tma_load_2d(qb_, &tq, h * 64, b * p.T + q0, qd_full(st));
        tc::tma_load_2d(qb_ + 16384, &tdo, h * 64, b * p.T + q0, qd_full(st));
      }
      int* cs = cols + st * TB_COL_STRIDE;
      float* lse_s = reinterpret_cast<float*>(cs);
      float* dsum_s = reinterpret_cast<float*>(cs + 128);
      int* qid_s = cs + 256;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = 4 * lane + e;
        lse_s[c] = cl[e] == -INFINITY ? INFINITY : cl[e];  // a row without valid keys contributes no P
        dsum_s[c] = cd[e];
        qid_s[c] = cq[e];
      }
      {  // 16-query chunks whose queries all carry one id (lanes 4c..4c+3 hold chunk c)
        const int first = __shfl_sync(0xffffffffu, cq[0], lane & ~3);
        const bool same = cq[0] == first && cq[1] == first && cq[2] == first && cq[3] == first;
        const unsigned bal = __ballot_sync(0xffffffffu, same);
        if ((lane & 3) == 0) qid_s[128 + (lane >> 2)] = first;
        if (lane == 0) {
          unsigned m = 0;
          for (int c = 0; c < 8; ++c) m |= ((bal >> (4 * c)) & 0xFu) == 0xFu ? 1u << c : 0u;
          qid_s[136] = (int)m;
        }
      }
      __syncwarp();
      tc::mbar_arrive(qd_full(st));
      if (it + 1 < nitems) load_cols(it + 1);
    }
  } else if (warp == 1) {
    // The whole warp runs the issue loop (converged); one elected lane issues.
    {
      const uint32_t idesc_s = tc::idesc_bf16_f32(128, 64, 0, 0);
      const uint32_t idesc_kn = tc::idesc_bf16_f32(128, 64, 0, 1);  // K-major A, MN-major B
      const uint32_t idesc_nn = tc::idesc_bf16_f32(128, 64, 1, 1);  // MN-major A and B
      const uint32_t dv_t = tmem + 256, dk_t = tmem + 320, dq_t = tmem + 384;
      const uint32_t k_tm = tmem + TB_KT_COL, v_tm = tmem + TB_VT_COL;
      // The MN-major K descriptor (dQ's B operand) does not change; the
      // per-step advance is added to the start-address field (bits 0-13, in
      // 16-byte units).
      const uint64_t kdesc_mn = tc::smem_desc_sw128(sb + TB_K_OFF, 8192, 1024);
      bool ok = tc::mbar_wait_w(kv_tm, 0, status, 32);
      tc::tc_fence_after();
      const int nsub = 2 * nitems;
      // dV/dK of sub-item j (its P^T is ready); after the second half of an
      // item, frees the item's Q/dO stage.
      auto finish = [&](int j) -> bool {
        const int it = j >> 1, hf = j & 1, u = j & 1, st = it % TB_ST;
        if (!tc::mbar_wait_w(p_full(u), (j >> 1) & 1, status, 34)) return false;
        tc::tc_fence_after();
        const uint32_t qb_ = sb + TB_QD_OFF + st * 32768 + hf * 8192, dob_ = qb_ + 16384;
        const uint32_t ds_ = sb + TB_DS_OFF + (it & 1) * 32768;
        const uint32_t s_t = tmem + u * 128;
        const uint64_t qd_mn = tc::smem_desc_sw128(qb_, 8192, 1024), dod_mn = tc::smem_desc_sw128(dob_, 8192, 1024);
        const uint64_t dsd = tc::smem_desc_sw128(ds_ + hf * 16384, 16, 1024);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::mma_bf16_ts_w(dv_t, s_t + (16 * k / TB_PW) * TB_PW + (16 * k % TB_PW) / 2,
                            dod_mn + (uint64_t)(k * 2048 >> 4), idesc_kn, (j | k) != 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::mma_bf16_w(dk_t, dsd + (uint64_t)(k * 32 >> 4), qd_mn + (uint64_t)(k * 2048 >> 4), idesc_kn,
                         (j | k) != 0 ? 1u : 0u);
        if (hf == 1) tc::mma_commit_w(qd_empty(st));
        return true;
      };
      // dQ of item `it` from its dS^T (both halves written) once the flush
      // warps have emptied the dQ columns.
      auto issue_dq = [&](int it) -> bool {
        if (it > 0 && !tc::mbar_wait_w(dq_free, (it - 1) & 1, status, 39)) return false;
        tc::tc_fence_after();
        const uint64_t dsn = tc::smem_desc_sw128(sb + TB_DS_OFF + (it & 1) * 32768, 16384, 1024);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          tc::mma_bf16_w(dq_t, dsn + (uint64_t)(k * 2048 >> 4), kdesc_mn + (uint64_t)(k * 2048 >> 4), idesc_nn,
                         k > 0 ? 1u : 0u);
        tc::mma_commit_w(dq_full);
        return true;
      };
      // Order: S/dP(j), then the dQ an item left pending, then dV/dK(j-1).
      // The next scores (which the softmax-gradient warps wait for) follow
      // dV/dK directly; an item's dQ goes after the next sub-item's scores.
      // dS^T buffer reuse stays safe: dQ(it) precedes S/dP of item it+2,
      // whose completion the writers of dS^T(it+2) wait for.
      int pend = -1;
      for (int j = 0; ok && j < nsub; ++j) {
        const int it = j >> 1, hf = j & 1, u = j & 1, st = it % TB_ST;
        if (hf == 0) {
          if (!(ok = tc::mbar_wait_w(qd_full(st), (it / TB_ST) & 1, status, 33))) break;
          tc::tc_fence_after();
        }
        const uint32_t qb_ = sb + TB_QD_OFF + st * 32768 + hf * 8192, dob_ = qb_ + 16384;
        const uint32_t s_t = tmem + u * 128, dp_t = s_t + 64;
        const uint64_t qd = tc::smem_desc_sw128(qb_, 16, 1024), dod = tc::smem_desc_sw128(dob_, 16, 1024);
        // A = K / V from TMEM (16 head dims = 8 columns per step), B = Q / dO.
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::mma_bf16_ts_w(s_t, k_tm + k * 8, qd + (uint64_t)(k * 32 >> 4), idesc_s, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::mma_bf16_ts_w(dp_t, v_tm + k * 8, dod + (uint64_t)(k * 32 >> 4), idesc_s, k > 0 ? 1u : 0u);
        tc::mma_commit_w(s_full(u));
        if (pend >= 0) {
          if (!(ok = issue_dq(pend))) break;
          pend = -1;
        }
        if (j > 0) {
          if (!(ok = finish(j - 1))) break;
          if ((j - 1) & 1) pend = (j - 1) >> 1;
        }
      }
      if (ok && nsub > 0) {
        ok = finish(nsub - 1);
        if (ok) ok = issue_dq(nitems - 1);
      }
      tc::mma_commit_w(done_bar);
      tc::mbar_wait_w(done_bar, 0, status, 35);
    }
  } else if (warp < 2 + TB_SM_WARPS) {
    const int quarter = warp & 3, wq = (warp - 2) >> 2;  // wq: which TB_CW of the sub-item's 64 columns
    const int r = quarter * 32 + lane;
    const int s = s0 + r;
    const int kid_row = s < p.S ? p.kid[(long long)b * p.S + s] : 0;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    bool ok;
    const int nsub = 2 * nitems;
    {
      // Key row r of K and V into TMEM as the A operand of the score
      // products (K in columns [0,32), V in [32,64) of the K/V block; two
      // bf16 per column): this warp copies TB_CW of those 64 columns,
      // un-swizzling the 128-byte shared rows.
      ok = __all_sync(0xffffffffu, tc::mbar_wait(kv_full, 0, status, 41));
      if (ok) {
        const int c0 = wq * TB_CW;  // first column of the K/V block
        const uint8_t* row = smem + (c0 >= 32 ? TB_V_OFF : TB_K_OFF) + r * 128;
        uint32_t w[TB_CW];
#pragma unroll
        for (int c = 0; c < TB_CW / 4; ++c) {
          const int chunk = (c0 % 32) / 4 + c;
          const uint4 x = *reinterpret_cast<const uint4*>(row + ((chunk ^ (r & 7)) << 4));
          w[4 * c] = x.x, w[4 * c + 1] = x.y, w[4 * c + 2] = x.z, w[4 * c + 3] = x.w;
        }
        const uint32_t dst = tmem + lane_off + TB_KT_COL + c0;
#pragma unroll
        for (int c = 0; c < TB_CW; c += 16) tc::tmem_st_32x32b_x16(dst + c, w + c);
        tc::tmem_st_wait();
      }
      tc::tc_fence_before();
      tc::mbar_arrive(kv_tm);
    }
    const int g = wq >> 1, wh = wq & 1;  // group (= sub-item half), which TB_PW of its 64 columns
    for (int j = g; ok && j < nsub; j += 2) {
      const int it = j >> 1, u = g, st = it % TB_ST;
      const int* cs = cols + st * TB_COL_STRIDE;
      // Warp-uniform wait outcomes: the TMEM accesses below are warp-collective.
      // The item's column data, whether its whole tile is valid, and this key
      // row's first causally valid column (key s sees queries t >= s - offset).
      ok = tc::mbar_wait(qd_full(st), (it / TB_ST) & 1, status, 37);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      const int entry = list[1 + it % nlive];
      const bool full = (entry >> 30) & 1;
      const int cfirst = p.causal ? s - p.offset - (entry & 0xFFFF) * TQ : -TQ;
      ok = tc::mbar_wait(s_full(u), it & 1, status, 36);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc::tc_fence_after();
      const uint32_t s_t = tmem + lane_off + u * 128 + wh * TB_PW, dp_t = s_t + 64;
      uint8_t* ds_row = smem + TB_DS_OFF + (it & 1) * 32768 + g * 16384 + r * 128;
      // 16 columns at a time: P^T (bf16 pairs) into the first TB_PW / 2 of this
      // warp's own consumed S^T columns; dS^T into the item's shared buffer
      // (128-byte swizzle, 64-query atom rows).
#pragma unroll
      for (int c = 0; c < TB_PW; c += 16) {
        const int cbase = g * 64 + wh * TB_PW + c;  // query columns within the item
        // Chunk class for the warp's 32 key rows: dense (every pair valid),
        // zero (none valid: P = dS = 0 without touching the scores) or mixed.
        bool dense = full, zero = false;
        if (!full) {
          const bool uni = (cs[256 + 136] >> (cbase >> 4)) & 1;
          const int uid = cs[256 + 128 + (cbase >> 4)];
          dense = __all_sync(0xffffffffu, uni && uid == kid_row && cfirst <= cbase);
          zero = !dense && __all_sync(0xffffffffu, (uni && uid != kid_row) || cfirst > cbase + 15);
        }
        uint32_t pk[8], dk4[8];
        if (zero) {
#pragma unroll
          for (int e = 0; e < 8; ++e) pk[e] = 0u, dk4[e] = 0u;
        } else {
          uint32_t sx[16], dx[16];
          tc::tmem_ld_32x32b_x16(s_t + c, sx);
          tc::tmem_ld_32x32b_x16(dp_t + c, dx);
          tc::tmem_ld_wait();
          const float* lse_s = reinterpret_cast<const float*>(cs) + cbase;
          const float* dsum_s = reinterpret_cast<const float*>(cs + 128) + cbase;
          if (dense)
            ds_chunk<true, 16>(sx, dx, lse_s, dsum_s, nullptr, kid_row, 0, sl2, pk, dk4);
          else
            ds_chunk<false, 16>(sx, dx, lse_s, dsum_s, cs + 256 + cbase, kid_row, cfirst - cbase, sl2, pk, dk4);
        }
        tc::tmem_st_32x32b_x8(s_t + c / 2, pk);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int c16 = (wh * TB_PW + c) / 8 + jj;  // 16-byte chunk of the atom row
          *reinterpret_cast<uint4*>(ds_row + ((c16 ^ (r & 7)) << 4)) =
              make_uint4(dk4[4 * jj], dk4[4 * jj + 1], dk4[4 * jj + 2], dk4[4 * jj + 3]);
        }
      }
      tc::tmem_st_wait();
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(p_full(u));
    }
    // Epilogue: after the last products, dK (times the logit scale) and dV
    // (plus the uniform-row term) for this key row, this warp's TB_CW dims.
    // A whole 128-key tile goes through the first Q/dO stage (free once every
    // product has completed) in the TMA tile layout and leaves as two TMA
    // stores; a partial tile stores its rows. Every softmax-gradient warp
    // reaches the staging barrier, whatever its waits returned.
    const bool done_ok = ok && tc::mbar_wait(done_bar, 0, status, 38);
    const bool go = __all_sync(0xffffffffu, done_ok);
    const bool whole = s0 + TK <= p.S;
    uint4 ka[TB_CW / 8], va[TB_CW / 8];
    if (go) {
      tc::tc_fence_after();
      uint32_t kv[TB_CW], vv[TB_CW];
#pragma unroll
      for (int c = 0; c < TB_CW; c += 16) {
        tc::tmem_ld_32x32b_x16(tmem + lane_off + 320 + wq * TB_CW + c, kv + c);
        tc::tmem_ld_32x32b_x16(tmem + lane_off + 256 + wq * TB_CW + c, vv + c);
      }
      tc::tmem_ld_wait();
      const float* uv = p.uvec + ((long long)b * p.Hk + hk) * HD + wq * TB_CW;
      const bool uni = p.policy == MFB_EMPTY_UNIFORM;
#pragma unroll
      for (int c8 = 0; c8 < TB_CW / 8; ++c8) {
        uint32_t* aw = reinterpret_cast<uint32_t*>(&ka[c8]);
        uint32_t* cw = reinterpret_cast<uint32_t*>(&va[c8]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = c8 * 8 + 2 * e;
          const float k0 = nitems > 0 ? __uint_as_float(kv[d]) * p.scale : 0.f;
          const float k1 = nitems > 0 ? __uint_as_float(kv[d + 1]) * p.scale : 0.f;
          float v0 = nitems > 0 ? __uint_as_float(vv[d]) : 0.f;
          float v1 = nitems > 0 ? __uint_as_float(vv[d + 1]) : 0.f;
          if (uni) v0 += uv[d], v1 += uv[d + 1];
          aw[e] = pack_bf16(k0, k1);
          cw[e] = pack_bf16(v0, v1);
        }
      }
    }
    if (whole) {
      if (go) {
#pragma unroll
        for (int c8 = 0; c8 < TB_CW / 8; ++c8) {
          const uint32_t off = r * 128 + ((((wq * TB_CW) / 8 + c8) ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(smem + TB_QD_OFF + off) = ka[c8];
          *reinterpret_cast<uint4*>(smem + TB_QD_OFF + 16384 + off) = va[c8];
        }
      }
      tc::fence_proxy_async_smem();
      asm volatile("bar.sync 1, %0;\n" ::"r"(32 * TB_SM_WARPS) : "memory");
      if (warp == 2 && lane == 0) {
        tc::tma_store_2d(&tdk, sb + TB_QD_OFF, hk * 64, b * p.S + s0);
        tc::tma_store_2d(&tdv, sb + TB_QD_OFF + 16384, hk * 64, b * p.S + s0);
        tc::bulk_commit_group();
        tc::bulk_wait_group_read0();  // the staging must outlive the reads; the writes complete with the grid
      }
    } else if (go && s < p.S) {
      const long long off = (((long long)b * p.S + s) * p.Hk + hk) * HD + wq * TB_CW;
#pragma unroll
      for (int c8 = 0; c8 < TB_CW / 8; ++c8) {
        *reinterpret_cast<uint4*>(p.dk + off + c8 * 8) = ka[c8];
        *reinterpret_cast<uint4*>(p.dv + off + c8 * 8) = va[c8];
      }
    }
  } else {
    // dQ flush warps: query row = TMEM lane (this warp's 32 rows), all 64
    // columns, reduced into the accumulator as two 32-column boxes.
    const int quarter = warp & 3;
    const uint32_t dq_t = tmem + ((uint32_t)(quarter * 32) << 16) + 384;
    uint8_t* stage = smem + TB_DQS_OFF + quarter * 4096;
    const uint32_t stage_u = sb + TB_DQS_OFF + quarter * 4096;
    for (int it = 0; it < nitems; ++it) {
      if (!__all_sync(0xffffffffu, tc::mbar_wait(dq_full, it & 1, status, 40))) break;
      tc::tc_fence_after();
      const int h = hk * p.G + it / nlive;
      const int t0 = (list[1 + it % nlive] & 0xFFFF) * TQ + quarter * 32;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t v[32];
        tc::tmem_ld_32x32b_x32(dq_t + 32 * half, v);
        tc::tmem_ld_wait();
        if (half == 1) {  // the dQ columns are free for the next item's product
          tc::tc_fence_before();
          tc::mbar_arrive(dq_free);
        }
        if (t0 < p.T) {  // rows past T inside the box are clipped by the tensor map
          // The staging box is free once the previous reduction has read it.
          if (lane == 0) tc::bulk_wait_group_read0();
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tc::tma_reduce_add_4d(&tdq, stage_u, 32 * half, h, t0, b);
            tc::bulk_commit_group();
          }
        }
      }
    }
    // The accumulator is read by the next kernel: every reduction complete.
    if (lane == 0) tc::bulk_wait_group0();
    __syncwarp();
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
struct Workspace {
  Range* qr;
  Range* kr;
  int* order;
  float* dsum;
  float* uvec;
  float* dq_acc;
  size_t bytes;
};

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

Workspace carve(void* base, int B, int T, int S, int H, int Hk) {
  Workspace w;
  const int nqb = cdiv(T, BQ), nkb = cdiv(S, BK);
  size_t off = 0;
  char* p = static_cast<char*>(base);
  w.qr = reinterpret_cast<Range*>(p + off);
  off += align256(sizeof(Range) * (size_t)B * nqb);
  w.kr = reinterpret_cast<Range*>(p + off);
  off += align256(sizeof(Range) * (size_t)B * nkb);
  w.order = reinterpret_cast<int*>(p + off);
  off += align256(sizeof(int) * (size_t)B * (size_t)max(cdiv(T, TQ), cdiv(S, TK)));
  w.dsum = reinterpret_cast<float*>(p + off);
  off += align256(sizeof(float) * (size_t)B * H * T);
  w.uvec = reinterpret_cast<float*>(p + off);
  off += align256(sizeof(float) * (size_t)B * Hk * HD);
  w.dq_acc = reinterpret_cast<float*>(p + off);
  off += align256(sizeof(float) * (size_t)B * T * H * HD);
  w.bytes = off;
  return w;
}

int check_dims(int B, int T, int S, int H, int Hk, int D) {
  MFB_CHECK_ARG(B > 0 && T > 0 && S > 0, "Attention needs nonempty batch/query/key dims (B=%d T=%d S=%d)", B, T, S);
  MFB_CHECK_ARG(H > 0 && Hk > 0 && H % Hk == 0, "Query heads must be divisible by KV heads (H=%d Hk=%d)", H, Hk);
  MFB_CHECK_ARG(D == HD, "head_dim %d unsupported: this build implements D = 64", D);
  MFB_CHECK_ARG((H / Hk) % TF_HPB == 0, "GQA group size %d must be a multiple of %d", H / Hk, TF_HPB);
  return MFB_OK;
}

int set_smem(const void* fn, int bytes) {
  int dev = 0;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  MFB_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  (void)dev;
  return MFB_OK;
}

Params make_params(const Workspace& w, int B, int T, int S, int H, int Hk, int causal, int offset, int policy,
                   float scale) {
  Params p{};
  p.qr = w.qr;
  p.kr = w.kr;
  p.order = w.order;
  p.dsum = w.dsum;
  p.uvec = w.uvec;
  p.dq_acc = w.dq_acc;
  p.B = B;
  p.T = T;
  p.S = S;
  p.H = H;
  p.Hk = Hk;
  p.G = H / Hk;
  p.causal = causal ? 1 : 0;
  p.offset = offset;
  p.policy = policy;
  p.nqb = cdiv(T, BQ);
  p.nkb = cdiv(S, BK);
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  return p;
}

// Longest-first order of the tensor-core kernels' work items (uneven segment
// lengths make some tiles several times longer than others; launching them
// first keeps the last wave short). Forward items are (query tile, batch row)
// weighted by their live key tiles, backward items (key tile, batch row) by
// their live query tiles -- the same tile test the kernels use. One CTA,
// counting sort over the tile counts. The range records are staged in shared
// memory with coalesced loads and each weight is computed once, when they fit
// (SCHED_RANGES records, SCHED_ITEMS items); otherwise they are read from the
// workspace.
constexpr int SCHED_RANGES = 1536;
constexpr int SCHED_ITEMS = 4096;
__global__ void __launch_bounds__(1024) schedule_kernel(Params p, int backward, int* order) {
  __shared__ int hist[TF_MAX_TILES + 1], base[TF_MAX_TILES + 1];
  __shared__ Range sr[SCHED_RANGES];
  __shared__ int wt[SCHED_ITEMS];
  const int ntq = cdiv(p.T, TQ), nkt = cdiv(p.S, TK);
  const int per = backward ? nkt : ntq, other = backward ? ntq : nkt;
  const int n = p.B * per;
  const int nqr = p.B * p.nqb, nr = nqr + p.B * p.nkb;
  const bool staged = nr <= SCHED_RANGES, keep = n <= SCHED_ITEMS;
  if (staged)
    for (int i = threadIdx.x; i < nr; i += blockDim.x) sr[i] = i < nqr ? p.qr[i] : p.kr[i - nqr];
  for (int i = threadIdx.x; i <= other; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const Range* qbase = staged ? sr : p.qr;
  const Range* kbase = staged ? sr + nqr : p.kr;
  auto weight = [&](int it) {
    const int t = it % per, b = it / per;
    const Range* qrs = qbase + (long long)b * p.nqb;
    const Range* krs = kbase + (long long)b * p.nkb;
    int c = 0;
    if (backward) {
      const Range kr = range128(krs, p.nkb, t);
      for (int j = 0; j < other; ++j) c += tile_live128(p, range128(qrs, p.nqb, j), kr, j * TQ, t * TK) ? 1 : 0;
    } else {
      const Range qr = range128(qrs, p.nqb, t);
      for (int j = 0; j < other; ++j) c += tile_live128(p, qr, range128(krs, p.nkb, j), t * TQ, j * TK) ? 1 : 0;
    }
    return c;
  };
  for (int it = threadIdx.x; it < n; it += blockDim.x) {
    const int w = weight(it);
    if (keep) wt[it] = w;
    atomicAdd(&hist[w], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // weights are tile counts, at most `other`
    int acc = 0;
    for (int c = other; c >= 0; --c) {
      base[c] = acc;
      acc += hist[c];
    }
  }
  __syncthreads();
  for (int it = threadIdx.x; it < n; it += blockDim.x) order[atomicAdd(&base[keep ? wt[it] : weight(it)], 1)] = it;
}

int launch_ranges(const Params& p, const int* qid, const int* kid, cudaStream_t s) {
  dim3 grid(max(p.nqb, p.nkb), p.B, 2);
  ranges_kernel<<<grid, 64, 0, s>>>(qid, kid, const_cast<Range*>(p.qr), const_cast<Range*>(p.kr), p.B, p.T, p.S,
                                    p.nqb, p.nkb);
  MFB_LAUNCH_CHECK("attention ranges");
  return MFB_OK;
}


}  // namespace attn
}  // namespace mfb

using namespace mfb;
using namespace mfb::attn;

extern "C" int mfb_attn_ids(int mode, const int32_t* mask, const int32_t* segment_ids, const int32_t* aux,
                            int32_t* qid, int32_t* kid, int B, int T, int S, int P, int* causal, int* causal_offset,
                            int* empty_policy, void* stream) {
  MFB_CHECK_ARG(mode >= MFB_MASK_CAUSAL && mode <= MFB_MASK_CACHED, "Unknown mask mode %d", mode);
  MFB_CHECK_ARG(B > 0 && T > 0 && S > 0, "empty attention dims");
  MFB_CHECK_ARG(qid && kid, "qid/kid are NULL");
  int c = 0, off = 0, pol = MFB_EMPTY_UNIFORM;
  switch (mode) {
    case MFB_MASK_CAUSAL:
      MFB_CHECK_ARG(mask && S == T, "causal mask needs mask [B,T] and S == T");
      c = 1;
      break;
    case MFB_MASK_PREFIX:
      MFB_CHECK_ARG(mask && aux && P >= 0 && S == P + T, "prefix mask needs prefix [B,P], suffix [B,T], S = P+T");
      c = 1;
      off = P;
      break;
    case MFB_MASK_PACKED:
      MFB_CHECK_ARG(mask && segment_ids && S == T, "Packed attention query/KV shapes are incompatible");
      c = 1;
      pol = MFB_EMPTY_ZERO;
      break;
    case MFB_MASK_BIDIR:
      MFB_CHECK_ARG(mask && S == T, "bidirectional attention needs mask [B,T] and S == T");
      pol = MFB_EMPTY_ZERO;
      break;
    default:
      MFB_CHECK_ARG(aux && T == 1, "cached attention needs valid_length [B] and one query per row");
      break;
  }
  const long long n = (long long)B * (long long)max(T, S);
  ids_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(mode, mask, segment_ids, aux, qid, kid, B,
                                                                             T, S, P);
  MFB_LAUNCH_CHECK("mfb_attn_ids");
  if (causal) *causal = c;
  if (causal_offset) *causal_offset = off;
  if (empty_policy) *empty_policy = pol;
  return MFB_OK;
}

// Reads (and clears) the attention tensor-core kernels' device status word of
// the current device: 0 = ok, otherwise the id of a bounded wait that gave up.
extern "C" int mfb_attn_status(int* code) {
  MFB_CHECK_ARG(code != nullptr, "code is NULL");
  *code = 0;
  MFB_CUDA_TRY(cudaMemcpyFromSymbol(code, g_tc_status, sizeof(int)));
  if (*code) {
    const int zero = 0;
    MFB_CUDA_TRY(cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int)));
  }
  return MFB_OK;
}

extern "C" size_t mfb_attn_workspace_size(int B, int T, int S, int H, int Hk, int D) {
  (void)D;
  if (B <= 0 || T <= 0 || S <= 0 || H <= 0 || Hk <= 0) return 0;
  return carve(nullptr, B, T, S, H, Hk).bytes;
}

extern "C" int mfb_attn_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, float* lse,
                            const int32_t* qid, const int32_t* kid, int B, int T, int S, int H, int Hk, int D,
                            int causal, int causal_offset, int empty_policy, float scale, void* workspace,
                            size_t workspace_bytes, void* stream) {
  int st = check_dims(B, T, S, H, Hk, D);
  if (st) return st;
  MFB_CHECK_ARG(q && k && v && o && lse && qid && kid, "NULL tensor argument");
  MFB_CHECK_ARG(empty_policy == MFB_EMPTY_UNIFORM || empty_policy == MFB_EMPTY_ZERO, "bad empty policy");
  const Workspace w = carve(workspace, B, T, S, H, Hk);
  const size_t need = reinterpret_cast<char*>(w.dsum) - static_cast<char*>(workspace);
  if (!workspace || workspace_bytes < need)
    return set_error(MFB_ERR_WORKSPACE, "attention forward workspace needs %zu bytes", need);
  Params p = make_params(w, B, T, S, H, Hk, causal, causal_offset, empty_policy, scale);
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.k = reinterpret_cast<const __nv_bfloat16*>(k);
  p.v = reinterpret_cast<const __nv_bfloat16*>(v);
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.lse = lse;
  p.qid = qid;
  p.kid = kid;
  cudaStream_t s = (cudaStream_t)stream;
  if ((st = launch_ranges(p, qid, kid, s))) return st;
  MFB_CHECK_ARG(((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0 &&
                    ((uintptr_t)o & 15) == 0,
                "q/k/v/o must be 16-byte aligned");
  CUtensorMap tq, tk, tv, to;
  if ((st = tc::make_tmap_bf16(&tq, q, (uint64_t)H * HD, (uint64_t)B * T, (uint64_t)H * HD, TQ))) return st;
  if ((st = tc::make_tmap_bf16(&tk, k, (uint64_t)Hk * HD, (uint64_t)B * S, (uint64_t)Hk * HD, TK))) return st;
  if ((st = tc::make_tmap_bf16(&tv, v, (uint64_t)Hk * HD, (uint64_t)B * S, (uint64_t)Hk * HD, TK))) return st;
  if ((st = tc::make_tmap_bf16(&to, o, (uint64_t)H * HD, (uint64_t)B * T, (uint64_t)H * HD, TQ))) return st;
  MFB_CHECK_ARG(S <= TF_MAX_TILES * TK, "key length %d above the supported %d", S, TF_MAX_TILES * TK);
  if ((st = set_smem((const void*)attn_fwd_tc_kernel, TF_SMEM))) return st;
  schedule_kernel<<<1, 1024, 0, s>>>(p, 0, w.order);
  MFB_LAUNCH_CHECK("attention forward schedule");
  const long long fwd_ctas = (long long)B * cdiv(T, TQ) * (H / TF_HPB);
  attn_fwd_tc_kernel<<<(unsigned)fwd_ctas, TF_THREADS, TF_SMEM, s>>>(tq, tk, tv, to, p);
  MFB_LAUNCH_CHECK("mfb_attn_fwd");
  return MFB_OK;
}

extern "C" int mfb_attn_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                            const float* lse, const uint16_t* d_o, uint16_t* dq, uint16_t* dk, uint16_t* dv,
                            const int32_t* qid, const int32_t* kid, int B, int T, int S, int H, int Hk, int D,
                            int causal, int causal_offset, int empty_policy, float scale, void* workspace,
                            size_t workspace_bytes, void* stream) {
  int st = check_dims(B, T, S, H, Hk, D);
  if (st) return st;
  MFB_CHECK_ARG(q && k && v && o && lse && d_o && dq && dk && dv && qid && kid, "NULL tensor argument");
  MFB_CHECK_ARG(empty_policy == MFB_EMPTY_UNIFORM || empty_policy == MFB_EMPTY_ZERO, "bad empty policy");
  const Workspace w = carve(workspace, B, T, S, H, Hk);
  if (!workspace || workspace_bytes < w.bytes)
    return set_error(MFB_ERR_WORKSPACE, "attention backward workspace needs %zu bytes", w.bytes);
  Params p = make_params(w, B, T, S, H, Hk, causal, causal_offset, empty_policy, scale);
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.k = reinterpret_cast<const __nv_bfloat16*>(k);
  p.v = reinterpret_cast<const __nv_bfloat16*>(v);
  p.o = reinterpret_cast<__nv_bfloat16*>(const_cast<uint16_t*>(o));
  p.lse = const_cast<float*>(lse);
  p.d_o = reinterpret_cast<const __nv_bfloat16*>(d_o);
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  p.qid = qid;
  p.kid = kid;
  cudaStream_t s = (cudaStream_t)stream;
  // The uniform-row accumulator is read and written only under the uniform
  // empty-row policy.
  if (empty_policy == MFB_EMPTY_UNIFORM) MFB_CUDA_TRY(cudaMemsetAsync(w.uvec, 0, sizeof(float) * (size_t)B * Hk * HD, s));
  const long long rows = (long long)B * T * H;
  const long long npre = (rows + 31) / 32, nranges = (long long)B * (p.nqb + p.nkb);
  attn_bwd_pre_kernel<<<(unsigned)(npre + (nranges + 3) / 4), 256, 0, s>>>(p, qid, kid, (int)npre);
  MFB_LAUNCH_CHECK("attention backward preprocess");
  MFB_CHECK_ARG(T <= TF_MAX_TILES * TQ, "query length %d above the supported %d", T, TF_MAX_TILES * TQ);
  MFB_CHECK_ARG(((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0 &&
                    ((uintptr_t)d_o & 15) == 0 && ((uintptr_t)dk & 15) == 0 && ((uintptr_t)dv & 15) == 0,
                "q/k/v/d_o/dk/dv must be 16-byte aligned");
  CUtensorMap tq, tk, tv, tdo, tdq, tdk, tdv;
  if ((st = tc::make_tmap_bf16(&tq, q, (uint64_t)H * HD, (uint64_t)B * T, (uint64_t)H * HD, TQ))) return st;
  if ((st = tc::make_tmap_bf16(&tdo, d_o, (uint64_t)H * HD, (uint64_t)B * T, (uint64_t)H * HD, TQ))) return st;
  if ((st = tc::make_tmap_f32_rows_heads(&tdq, w.dq_acc, H, (uint64_t)T, (uint64_t)B, 32))) return st;
  if ((st = tc::make_tmap_bf16(&tk, k, (uint64_t)Hk * HD, (uint64_t)B * S, (uint64_t)Hk * HD, TK))) return st;
  if ((st = tc::make_tmap_bf16(&tv, v, (uint64_t)Hk * HD, (uint64_t)B * S, (uint64_t)Hk * HD, TK))) return st;
  if ((st = tc::make_tmap_bf16(&tdk, dk, (uint64_t)Hk * HD, (uint64_t)B * S, (uint64_t)Hk * HD, TK))) return st;
  if ((st = tc::make_tmap_bf16(&tdv, dv, (uint64_t)Hk * HD, (uint64_t)B * S, (uint64_t)Hk * HD, TK))) return st;
  if ((st = set_smem((const void*)attn_bwd_tc_kernel, TB_SMEM))) return st;
  schedule_kernel<<<1, 1024, 0, s>>>(p, 1, w.order);
  MFB_LAUNCH_CHECK("attention backward schedule");
  const long long bwd_ctas = (long long)B * cdiv(S, TK) * Hk;
  attn_bwd_tc_kernel<<<(unsigned)bwd_ctas, TB_THREADS, TB_SMEM, s>>>(tq, tk, tv, tdo, tdq, tdk, tdv, p);
  MFB_LAUNCH_CHECK("attention backward");
  const long long n4 = (long long)B * T * H * HD / 4;
  dq_convert_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, s>>>(w.dq_acc, reinterpret_cast<__nv_bfloat16*>(dq), n4,
                                                                 scale);
  MFB_LAUNCH_CHECK("attention dq convert");
  return MFB_OK;
}
