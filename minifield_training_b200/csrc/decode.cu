// KV-cached single-query GQA decode with fused cache append, D = 64.
//
// Replaces, for one decode step, the dynamic_update_slice cache write of
// attention_block_step (src/minifield_training/layers/attention.py:309-314)
// followed by dense_cached_attention (src/minifield_training/kernels/
// attention.py:264-282): the query of row b attends to cache slots
// < valid_length[b] (non-causal); valid_length <= 0 leaves every slot masked,
// which the reference's finfo.min fill turns into a uniform average over all
// capacity slots.
//
// HBM layout: caches [B, cap, Hk, 64] bf16 (decode.py:96-117), so the cache
// positions of all KV heads are contiguous (Hk x 128 bytes each).
//
// Work split ("stream-K" over positions): the valid positions of all rows,
// sum_b len_b, are divided into equal contiguous shares, one per resident CTA;
// a share is cut at row boundaries into segments. A producer thread streams
// each segment's K and V through a 3-stage shared-memory ring, one 3-D TMA box
// {64 dims, 16 positions, Hk heads} per operand and stage (128-byte swizzle,
// no multicast), and brings the segment's query row -- and, at the stage that
// holds the append slot, the new key/value row -- into a side slot of the same
// stage with bulk copies, so the compute warps issue no global loads. Eight
// compute warps (one KV head each) run the scores and P.V on the warp-level
// tensor-core MMA with the GQA group's query heads as rows -- the kernel is
// bandwidth-bound, the MMA only removes per-element conversions and shuffles --
// and an FP32 online softmax. A row that lies inside one share is written
// directly. Only the first and last row of a share can be cut; their (m, l, o)
// partials go to the workspace, and once the CTA has finished all its stages
// it takes one ticket per cut row; the last CTA of a row (atomic ticket, no
// waiting) combines its partials.
#include <math.h>

#include <algorithm>
#include <mutex>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "tc.cuh"

namespace mfb {
namespace dec {

constexpr int HD = 64;
constexpr int WARPS = 8;                   // compute warps
constexpr int THREADS = 32 * (WARPS + 1);  // + one producer warp
constexpr int MAXG = 4;
constexpr int NST = 3;                     // ring stages
constexpr int SP = 16;                     // positions per stage
constexpr int HEAD_TILE = SP * 128;        // one KV head's 16 positions x 64 dims
constexpr int STAGE_K = 8 * HEAD_TILE;     // K (and V) bytes per stage for up to 8 KV heads
constexpr int MAX_GRID = 1024;             // CTAs per launch (partial slots reserved per call)
constexpr int MAX_B = 8192;
constexpr int MAX_H = 8 * MAXG;

// Dynamic shared memory, offsets from the 1024-byte-aligned base:
//   ring   NST x {K [Hk][16][64], V [Hk][16][64]}, 128-byte swizzled
//   side   NST x {q row [H][64], new k [Hk][64], new v [Hk][64]}
//   bars   NST full + NST empty mbarriers
//   pref   [B + 1] int: exclusive prefix of the rows' valid lengths
//   wslot  [B] int: each row's append slot (-1: no append)
//   uflag  [B] uint8: 1 when valid_length <= 0 (uniform row)
struct Layout {
  uint32_t side, side_bytes, bars, pref, wslot, uflag, total;
};

__host__ __device__ inline Layout layout(int B, int H, int Hk) {
  Layout L;
  L.side = NST * 2 * STAGE_K;
  L.side_bytes = (uint32_t)(H + 2 * Hk) * 128u;
  L.bars = L.side + NST * L.side_bytes;
  L.pref = L.bars + 2 * NST * 8;
  L.wslot = L.pref + 4u * (uint32_t)(B + 1);
  L.uflag = L.wslot + 4u * (uint32_t)B;
  L.total = L.uflag + (uint32_t)B;
  return L;
}

// Bounded-wait status word of the decode kernel on each device.
__device__ int g_dec_status;

struct Params {
  const __nv_bfloat16* q;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  const __nv_bfloat16* nk;
  const __nv_bfloat16* nv;
  const int* positions;
  const int* valid_length;
  __nv_bfloat16* o;
  float* part_o;    // [MAX_GRID + B][H][64]: slot (cta + row)
  float2* part_ml;  // [MAX_GRID + B][H]
  int* tickets;     // [B]
  int B, cap, H, Hk;
  float scale_log2;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];\n" : "=r"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

__device__ __forceinline__ void sts128(uint32_t a, const uint4& v) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
}

// The CTA whose share [floor(i*T/g), floor((i+1)*T/g)) holds position x.
__device__ __forceinline__ int cta_of(int x, int total, int g) {
  return (int)(((long long)(x + 1) * g + total - 1) / total) - 1;
}

__device__ __forceinline__ void compute_bar() { asm volatile("bar.sync 1, 256;\n" ::: "memory"); }

// Merges the partials of row b written by CTAs c0..c1 (one pass, online max;
// four partials' loads in flight at a time) and writes the bf16 output row.
__device__ __forceinline__ void combine_row(const Params& p, int b, int c0, int c1, int tid) {
  for (int item = tid; item < p.H * (HD / 4); item += 32 * WARPS) {
    const int h = item / (HD / 4), d4 = (item % (HD / 4)) * 4;
    float m = -INFINITY, den = 0.f, n0 = 0.f, n1 = 0.f, n2 = 0.f, n3 = 0.f;
    for (int c = c0; c <= c1; c += 4) {
      float2 ml[4];
      float4 ov[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        ml[u] = make_float2(-INFINITY, 0.f);
        ov[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c + u <= c1) {
          const long long pi = ((long long)c + u + b) * p.H + h;
          ml[u] = __ldcg(p.part_ml + pi);
          ov[u] = __ldcg(reinterpret_cast<const float4*>(p.part_o + pi * HD + d4));
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (c + u <= c1) {
          const float mn = fmaxf(m, ml[u].x);
          const float a = ex2(m - mn), w = ex2(ml[u].x - mn);
          den = den * a + ml[u].y * w;
          n0 = n0 * a + ov[u].x * w;
          n1 = n1 * a + ov[u].y * w;
          n2 = n2 * a + ov[u].z * w;
          n3 = n3 * a + ov[u].w * w;
          m = mn;
        }
      }
    }
    const float inv = 1.f / den;
    uint2 out;
    out.x = pack_bf16(n0 * inv, n1 * inv);
    out.y = pack_bf16(n2 * inv, n3 * inv);
    *reinterpret_cast<uint2*>(p.o + ((long long)b * p.H + h) * HD + d4) = out;
  }
}

template <int G>
__global__ void __launch_bounds__(THREADS, 2)
    decode_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, Params p) {
  allow_dependents();
  extern __shared__ uint8_t smem_raw[];
  // Offset from the __shared__ array itself so accesses keep the shared state space.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const Layout lay = layout(p.B, p.H, p.Hk);
  int* pref = reinterpret_cast<int*>(smem + lay.pref);
  int* wslot = reinterpret_cast<int*>(smem + lay.wslot);
  uint8_t* uflag = smem + lay.uflag;
  __shared__ int s_wsum[WARPS + 1], s_comb[2];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t sb = smem_u32(smem);
  const uint32_t bars = sb + lay.bars;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (NST + s); };
  int* status = &g_dec_status;
  const int row_elems = p.Hk * HD;
  const bool append = p.nk != nullptr;

  // Prologue: the rows' valid lengths (prefix), append slots and uniform flags.
  {
    const int per = cdiv(p.B, THREADS);
    const int r0 = min(p.B, tid * per), r1 = min(p.B, r0 + per);
    int local = 0;
    for (int r = r0; r < r1; ++r) {
      const int L = p.valid_length[r];
      const int len = L <= 0 ? p.cap : min(L, p.cap);
      pref[r] = len;
      uflag[r] = L <= 0;
      wslot[r] = append ? min(max(p.positions[r], 0), p.cap - 1) : -1;
      local += len;
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_wsum[warp] = incl;
    if (tid == 0) {
      for (int s = 0; s < NST; ++s) {
        tc::mbar_init(full_bar(s), 1);
        tc::mbar_init(empty_bar(s), WARPS);
      }
      tc::mbar_fence_init();
    }
    __syncthreads();
    int off = incl - local;
    for (int w = 0; w < warp; ++w) off += s_wsum[w];
    for (int r = r0; r < r1; ++r) {
      const int len = pref[r];
      pref[r] = off;
      off += len;
    }
    if (tid == THREADS - 1) pref[p.B] = off;
    __syncthreads();
  }
  const int total = pref[p.B];
  const int g = min((int)gridDim.x, total);  // every share is nonempty
  const int i = blockIdx.x;
  if (i >= g) return;
  const int x0 = (int)((long long)i * total / g), x1 = (int)((long long)(i + 1) * total / g);
  int b0 = 0;
  {
    int lo = 0, hi = p.B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pref[mid] <= x0) lo = mid;
      else hi = mid - 1;
    }
    b0 = lo;
  }

  if (warp == WARPS) {
    // Producer: per stage one K box and one V box (all KV heads), plus the
    // query row on a segment's first stage and the new key/value rows on the
    // stage that holds the append slot, all counted on the stage's barrier.
    if (lane == 0) {
      tc::tma_prefetch_desc(&tk);
      tc::tma_prefetch_desc(&tv);
      const uint32_t kv_bytes = 2u * p.Hk * HEAD_TILE, q_bytes = p.H * 128u, n_bytes = p.Hk * 128u;
      int it = 0;
      bool ok = true;
      for (int b = b0; ok && b < p.B && pref[b] < x1; ++b) {
        const int lo = max(x0, pref[b]) - pref[b], hi = min(x1, pref[b + 1]) - pref[b];
        const int ws = wslot[b];
        for (int p0 = lo; p0 < hi; p0 += SP, ++it) {
          const int st = it % NST;
          if (!(ok = tc::mbar_wait(empty_bar(st), ((it / NST) & 1) ^ 1, status, 1))) break;
          const int np = min(SP, hi - p0);
          const bool first = p0 == lo, patch = ws >= p0 && ws < p0 + np;
          const uint32_t side = sb + lay.side + st * lay.side_bytes;
          tc::mbar_expect_tx(full_bar(st), kv_bytes + (first ? q_bytes : 0u) + (patch ? 2u * n_bytes : 0u));
          tc::tma_load_3d(sb + st * 2 * STAGE_K, &tk, 0, b * p.cap + p0, 0, full_bar(st));
          tc::tma_load_3d(sb + st * 2 * STAGE_K + STAGE_K, &tv, 0, b * p.cap + p0, 0, full_bar(st));
          if (first) tc::bulk_load(side, p.q + (long long)b * p.H * HD, q_bytes, full_bar(st));
          if (patch) {
            tc::bulk_load(side + q_bytes, p.nk + (long long)b * row_elems, n_bytes, full_bar(st));
            tc::bulk_load(side + q_bytes + n_bytes, p.nv + (long long)b * row_elems, n_bytes, full_bar(st));
          }
        }
      }
    }
    return;
  }

  // Compute warps: warp w owns KV head w (heads >= Hk only keep the ring
  // moving). Per 16-position stage, on the warp-level tensor-core MMA
  // (m16n8k16, rows = the GQA group's query heads, unused rows zero):
  //   S = Q K^T   (4 k-steps x 2 position tiles), K from shared memory by ldmatrix
  //   online softmax on the S fragments (quad shuffles per row)
  //   O += P V    (P from the S fragments as the A operand, V by ldmatrix.trans)
  const int hk = warp;
  const bool active = hk < p.Hk;
  const int g4 = lane >> 2, c4 = lane & 3;  // fragment row (query head in the group) and column pair
  const float sl2 = p.scale_log2;
  int it = 0, b_last = b0;
  bool ok = true;
  for (int b = b0; b < p.B && pref[b] < x1; ++b) {
    b_last = b;
    const int lo = max(x0, pref[b]) - pref[b], hi = min(x1, pref[b + 1]) - pref[b];
    const bool uniform = uflag[b] != 0;
    const int ws = wslot[b];
    uint32_t qa[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) qa[kk][0] = qa[kk][1] = qa[kk][2] = qa[kk][3] = 0u;
    float o[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int p0 = lo; p0 < hi; p0 += SP, ++it) {
      const int st = it % NST;
      // After a timed-out wait the warp skips the remaining waits but keeps
      // the named-barrier schedule of the other compute warps.
      if (ok) ok = tc::mbar_wait(full_bar(st), (it / NST) & 1, status, 2);
      if (ok && active) {
        const int np = min(SP, hi - p0);
        const uint32_t kt = sb + st * 2 * STAGE_K + hk * HEAD_TILE, vt = kt + STAGE_K;
        const uint32_t side = sb + lay.side + st * lay.side_bytes;
        if (p0 == lo && g4 < G) {
          // Q fragments (unscaled bf16) of query head hk*G + g4 from the side slot.
          const uint32_t qrow = side + (hk * G + g4) * 128u + 4u * c4;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            qa[kk][0] = lds32(qrow + kk * 32);
            qa[kk][2] = lds32(qrow + kk * 32 + 16);
          }
        }
        if (ws >= p0 && ws < p0 + np) {
          // The new token: patch its key / value row into this head's tiles
          // (the stage holds the old row) and append it to the caches in HBM.
          const int r = ws - p0;
          if (lane < 8) {
            const uint32_t nrow = side + p.H * 128u + hk * 128u + lane * 16u;
            const uint4 nk4 = lds128(nrow), nv4 = lds128(nrow + p.Hk * 128u);
            sts128(kt + swz64(r, lane * 8), nk4);
            sts128(vt + swz64(r, lane * 8), nv4);
            const long long at = ((long long)b * p.cap + ws) * row_elems + hk * HD + lane * 8;
            *reinterpret_cast<uint4*>(p.kc + at) = nk4;
            *reinterpret_cast<uint4*>(p.vc + at) = nv4;
            tc::fence_proxy_async_smem();  // the ring's next TMA write to this stage must follow
          }
          __syncwarp();
        }
        float sc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          uint32_t b0r, b1r, b2r, b3r;
          ldmatrix_x4(kt + swz64((lane & 7) + ((lane >> 4) << 3), kk * 16 + ((lane >> 3) & 1) * 8), b0r, b1r, b2r, b3r);
          const uint32_t x0f[2] = {b0r, b1r}, x1f[2] = {b2r, b3r};
          mma_bf16_16816(sc[0], qa[kk], x0f);
          mma_bf16_16816(sc[1], qa[kk], x1f);
        }
        // Scale, mask positions past the segment, online softmax of row g4.
        float v[4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int k = nt * 8 + 2 * c4 + e;
            v[nt * 2 + e] = k < np ? (uniform ? 0.f : sc[nt][e] * sl2) : -INFINITY;
          }
        float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m, mx);
        const float mu = mn == -INFINITY ? 0.f : mn;
        const float alpha = ex2(m - mu);
        m = mn;
        float pr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pr[e] = ex2(v[e] - mu);
        l = l * alpha + (pr[0] + pr[1]) + (pr[2] + pr[3]);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) o[nt][0] *= alpha, o[nt][1] *= alpha;
        uint32_t pa[4];
        pa[0] = pack_bf16(pr[0], pr[1]);
        pa[1] = 0u;
        pa[2] = pack_bf16(pr[2], pr[3]);
        pa[3] = 0u;
#pragma unroll
        for (int nd2 = 0; nd2 < 4; ++nd2) {
          uint32_t b0r, b1r, b2r, b3r;
          ldmatrix_x4_trans(vt + swz64((lane & 7) + ((lane >> 3) & 1) * 8, nd2 * 16 + (lane >> 4) * 8), b0r, b1r, b2r,
                            b3r);
          const uint32_t x0f[2] = {b0r, b1r}, x1f[2] = {b2r, b3r};
          mma_bf16_16816(o[2 * nd2], pa, x0f);
          mma_bf16_16816(o[2 * nd2 + 1], pa, x1f);
        }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(empty_bar(st));
    }
    // Segment end, rows g4 < G (the quad's four lanes hold 16 dims each): a
    // row inside this share is finished here; a cut row leaves its partial.
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (active && g4 < G) {
      const int c0 = cta_of(pref[b], total, g), c1 = cta_of(pref[b + 1] - 1, total, g);
      const int h = hk * G + g4;
      if (c0 == c1) {
        const float inv = 1.f / l;
        __nv_bfloat16* orow = p.o + ((long long)b * p.H + h) * HD + 2 * c4;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
          *reinterpret_cast<uint32_t*>(orow + nt * 8) = pack_bf16(o[nt][0] * inv, o[nt][1] * inv);
      } else {
        const long long pi = ((long long)i + b) * p.H + h;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
          *reinterpret_cast<float2*>(p.part_o + pi * HD + nt * 8 + 2 * c4) = make_float2(o[nt][0], o[nt][1]);
        if (c4 == 0) p.part_ml[pi] = make_float2(m, l);
      }
    }
  }

  // All stages done: one ticket per cut row (at most the share's first and
  // last row); the last CTA of a row to arrive combines the row's partials.
  __threadfence();
  compute_bar();
  if (tid < 2) {
    int row = -1;
    const int b = tid == 0 ? b0 : b_last;
    if (tid == 0 || b_last != b0) {
      const int c0 = cta_of(pref[b], total, g), c1 = cta_of(pref[b + 1] - 1, total, g);
      if (c0 != c1 && atomicAdd(p.tickets + b, 1) == c1 - c0) row = b;
    }
    s_comb[tid] = row;
  }
  compute_bar();
#pragma unroll 1
  for (int k = 0; k < 2; ++k) {
    const int b = s_comb[k];
    if (b < 0) continue;
    __threadfence();
    combine_row(p, b, cta_of(pref[b], total, g), cta_of(pref[b + 1] - 1, total, g), tid);
    if (tid == 0) p.tickets[b] = 0;
  }
  // Appends whose slot is not a valid position of its row (at or beyond
  // valid_length): nothing reads that slot this step; row b goes to CTA b % g.
  if (append) {
    for (int b = i; b < p.B; b += g) {
      const int ws = wslot[b];
      if (ws >= pref[b + 1] - pref[b]) {
        for (int e = tid; e < row_elems / 8; e += 32 * WARPS) {
          const long long at = ((long long)b * p.cap + ws) * row_elems + e * 8;
          *reinterpret_cast<uint4*>(p.kc + at) = *reinterpret_cast<const uint4*>(p.nk + (long long)b * row_elems + e * 8);
          *reinterpret_cast<uint4*>(p.vc + at) = *reinterpret_cast<const uint4*>(p.nv + (long long)b * row_elems + e * 8);
        }
      }
    }
  }
}

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct Workspace {
  float* part_o;
  float2* part_ml;
  int* tickets;
  size_t bytes;
};

Workspace carve(void* base, int B, int H) {
  const size_t slots = (size_t)MAX_GRID + B;
  char* p = static_cast<char*>(base);
  Workspace w;
  size_t off = 0;
  w.part_o = reinterpret_cast<float*>(p + off);
  off += align256(sizeof(float) * slots * H * HD);
  w.part_ml = reinterpret_cast<float2*>(p + off);
  off += align256(sizeof(float2) * slots * H);
  w.tickets = reinterpret_cast<int*>(p + off);
  off += align256(sizeof(int) * (size_t)B);
  w.bytes = off;
  return w;
}

int check(const void* q, const void* kc, const void* vc, const void* nk, const void* nv, const void* positions,
          const void* vl, const void* o, int B, int capacity, int H, int Hk, int D) {
  MFB_CHECK_ARG(B > 0 && capacity > 0, "Cached attention needs a nonempty batch and cache (B=%d cap=%d)", B, capacity);
  MFB_CHECK_ARG(B <= MAX_B, "decode batch %d above the supported %d rows", B, MAX_B);
  MFB_CHECK_ARG(D == HD, "Cached attention query/KV shapes are incompatible (head_dim %d; this build needs 64)", D);
  MFB_CHECK_ARG(H > 0 && Hk > 0 && H % Hk == 0, "Query heads must be divisible by KV heads (H=%d Hk=%d)", H, Hk);
  MFB_CHECK_ARG(H / Hk <= MAXG && (H / Hk == 1 || H / Hk == 2 || H / Hk == 4), "GQA group size %d unsupported (1, 2 or 4)",
                H / Hk);
  MFB_CHECK_ARG(Hk == 1 || Hk == 2 || Hk == 4 || Hk == 8, "decode supports 1, 2, 4 or 8 KV heads (Hk=%d)", Hk);
  MFB_CHECK_ARG(q && kc && vc && vl && o, "NULL tensor argument");
  MFB_CHECK_ARG((nk == nullptr) == (nv == nullptr), "new_k and new_v must both be given or both be NULL");
  MFB_CHECK_ARG(nk == nullptr || positions != nullptr, "positions are required with new_k/new_v");
  MFB_CHECK_ARG((long long)B * capacity < (1LL << 31), "decode needs B x capacity < 2^31 cache positions (%lld)",
                (long long)B * capacity);
  MFB_CHECK_ARG(((uintptr_t)kc & 15) == 0 && ((uintptr_t)vc & 15) == 0, "caches must be 16-byte aligned");
  MFB_CHECK_ARG(((uintptr_t)q & 15) == 0 && ((uintptr_t)o & 15) == 0 && ((uintptr_t)nk & 15) == 0 &&
                    ((uintptr_t)nv & 15) == 0,
                "q, o, new_k and new_v must be 16-byte aligned");
  return MFB_OK;
}

// Sets the kernel's dynamic shared-memory limit (on every call: the setting
// belongs to the CUDA context, which a device reset replaces) and returns how
// many CTAs of `smem` bytes fit on one SM.
template <int G>
int resident_ctas(int dev, size_t smem, int* occ) {
  (void)dev;
  const int smem_max = 1024 + (int)layout(MAX_B, MAX_H, 8).total;
  MFB_CUDA_TRY(cudaFuncSetAttribute(decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max));
  MFB_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, decode_kernel<G>, THREADS, smem));
  return MFB_OK;
}

template <int G>
int launch(const CUtensorMap& tk, const CUtensorMap& tv, const Params& p, int dev, int sms, size_t smem,
           cudaStream_t s) {
  int occ = 0, st;
  if ((st = resident_ctas<G>(dev, smem, &occ))) return st;
  const int grid = std::min(std::max(occ, 1) * sms, MAX_GRID);
  decode_kernel<G><<<grid, THREADS, smem, s>>>(tk, tv, p);
  MFB_LAUNCH_CHECK("decode kernel");
  return MFB_OK;
}

// Zeroes the row tickets and launches on stream s over the given workspace.
int run(const uint16_t* q, uint16_t* k_cache, uint16_t* v_cache, const uint16_t* new_k, const uint16_t* new_v,
        const int32_t* positions, const int32_t* valid_length, uint16_t* o, int B, int capacity, int H, int Hk,
        float scale, const Workspace& w, cudaStream_t s) {
  Params p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.kc = reinterpret_cast<__nv_bfloat16*>(k_cache);
  p.vc = reinterpret_cast<__nv_bfloat16*>(v_cache);
  p.nk = reinterpret_cast<const __nv_bfloat16*>(new_k);
  p.nv = reinterpret_cast<const __nv_bfloat16*>(new_v);
  p.positions = positions;
  p.valid_length = valid_length;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.part_o = w.part_o;
  p.part_ml = w.part_ml;
  p.tickets = w.tickets;
  p.B = B;
  p.cap = capacity;
  p.H = H;
  p.Hk = Hk;
  p.scale_log2 = scale * kLog2e;
  int dev = 0, sms = 148;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  MFB_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const size_t smem = 1024 + layout(B, H, Hk).total;
  CUtensorMap tk, tv;
  int st;
  const uint64_t rows = (uint64_t)B * capacity;
  if ((st = tc::make_tmap_bf16_heads(&tk, k_cache, rows, Hk, SP))) return st;
  if ((st = tc::make_tmap_bf16_heads(&tv, v_cache, rows, Hk, SP))) return st;
  MFB_CUDA_TRY(cudaMemsetAsync(w.tickets, 0, sizeof(int) * (size_t)B, s));
  switch (H / Hk) {
    case 1: return launch<1>(tk, tv, p, dev, sms, smem, s);
    case 2: return launch<2>(tk, tv, p, dev, sms, smem, s);
    default: return launch<4>(tk, tv, p, dev, sms, smem, s);
  }
}

}  // namespace dec
}  // namespace mfb

using namespace mfb;

extern "C" size_t mfb_decode_workspace_size(int B, int capacity, int H, int D) {
  (void)D;
  if (B <= 0 || capacity <= 0 || H <= 0) return 0;
  return dec::carve(nullptr, B, H).bytes;
}

extern "C" int mfb_decode_attn(const uint16_t* q, uint16_t* k_cache, uint16_t* v_cache, const uint16_t* new_k,
                               const uint16_t* new_v, const int32_t* positions, const int32_t* valid_length,
                               uint16_t* o, int B, int capacity, int H, int Hk, int D, float scale, void* workspace,
                               size_t workspace_bytes, void* stream) {
  int st = dec::check(q, k_cache, v_cache, new_k, new_v, positions, valid_length, o, B, capacity, H, Hk, D);
  if (st) return st;
  const dec::Workspace w = dec::carve(workspace, B, H);
  if (!workspace || workspace_bytes < w.bytes)
    return set_error(MFB_ERR_WORKSPACE, "decode workspace needs %zu bytes", w.bytes);
  return dec::run(q, k_cache, v_cache, new_k, new_v, positions, valid_length, o, B, capacity, H, Hk, scale, w,
                  (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot call cudaMalloc: code running inside a CUDA-graph
// capture region or a framework's custom-call handler (an XLA FFI handler may
// only use the buffers the runtime hands it), or a serving loop that forbids
// allocation after start-up. mfb_decode_attn_noalloc gives them the decode
// step with its split-K partials in a fixed scratch array compiled into this
// library instead of a caller workspace.
// ---------------------------------------------------------------------------
namespace mfb {
namespace dec {

// Scratch for the partials and tickets: MFB_DECODE_NOALLOC_SCRATCH_BYTES per
// device that loads the library, held until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[MFB_DECODE_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch per device ordinal, with the unique ID
// of the CUDA context it was resolved in (the host-side symbol is only a
// stand-in). A context that is destroyed and re-created -- cudaDeviceReset,
// or the primary context released and retained again -- loads the library's
// module again at another address, so the cached address is only used while
// the calling thread's current context has the same ID; otherwise it is
// looked up again. Slots are read and written under g_noalloc_mutex.
constexpr int kMaxDevices = 64;
struct NoallocSlot {
  unsigned long long context_id;
  void* ptr;
};
static NoallocSlot g_noalloc_slot[kMaxDevices] = {};
static std::mutex g_noalloc_mutex;

// Unique ID of the calling thread's current context (cuCtxGetId never reuses
// an ID within a process), or 0 when there is none or the driver cannot say.
static unsigned long long current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag resolved;
  std::call_once(resolved, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// The scratch array's device address in the current context of device dev.
static int noalloc_scratch(int dev, void** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoallocSlot& slot = g_noalloc_slot[dev];
  unsigned long long id = current_context_id();
  if (slot.ptr == nullptr || id == 0 || slot.context_id != id) {
    void* ptr = nullptr;
    MFB_CUDA_TRY(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
    // The lookup makes the device's primary context current if none was, so
    // read the ID again for the record.
    slot.context_id = id ? id : current_context_id();
    slot.ptr = ptr;
  }
  *out = slot.ptr;
  return MFB_OK;
}

}  // namespace dec
}  // namespace mfb

extern "C" int mfb_decode_attn_noalloc(const uint16_t* q, uint16_t* k_cache, uint16_t* v_cache,
                                       const uint16_t* new_k, const uint16_t* new_v, const int32_t* positions,
                                       const int32_t* valid_length, uint16_t* o, int B, int capacity, int H, int Hk,
                                       int D, float scale, void* stream) {
  int st = dec::check(q, k_cache, v_cache, new_k, new_v, positions, valid_length, o, B, capacity, H, Hk, D);
  if (st) return st;
  const size_t need = dec::carve(nullptr, B, H).bytes;
  MFB_CHECK_ARG(need <= (size_t)MFB_DECODE_NOALLOC_SCRATCH_BYTES,
                "mfb_decode_attn_noalloc: B=%d, H=%d need %zu scratch bytes, above the fixed %d-byte "
                "maximum; use mfb_decode_attn with a caller workspace",
                B, H, need, (int)MFB_DECODE_NOALLOC_SCRATCH_BYTES);
  int dev = 0;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  MFB_CHECK_ARG(dev >= 0 && dev < dec::kMaxDevices, "device ordinal %d out of range", dev);
  void* scratch = nullptr;
  if ((st = dec::noalloc_scratch(dev, &scratch))) return st;
  // The array keeps the previous call's contents; the run clears the per-row
  // tickets, which must start at zero, before the launch.
  const dec::Workspace w = dec::carve(scratch, B, H);
  return dec::run(q, k_cache, v_cache, new_k, new_v, positions, valid_length, o, B, capacity, H, Hk, scale, w,
                  (cudaStream_t)stream);
}
