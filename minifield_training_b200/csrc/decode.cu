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
// sum_b len_b, are divided into equal contiguous shares, one per CTA (two CTAs
// per SM); a share is cut at row boundaries into segments. A producer warp
// streams each segment's K and V through a 3-stage shared-memory ring with
// per-head 2-D TMA boxes (16 positions x 64 dims, 128-byte swizzle, no
// multicast), without draining between segments. Eight compute warps (one KV
// head each) run the scores and P.V on the warp-level tensor-core MMA with the
// GQA group's query heads as rows -- the kernel is bandwidth-bound, the MMA
// only removes the per-element conversions and shuffles -- and an FP32 online
// softmax. Each (CTA, row) segment writes one (m, l, o) partial; the last
// segment of a row to finish (atomic ticket, no waiting) combines them.
#include <math.h>

#include "common.cuh"
#include "tc.cuh"

namespace mfb {
namespace dec {

constexpr int HD = 64;
constexpr int WARPS = 8;                  // compute warps
constexpr int THREADS = 32 * (WARPS + 1);  // + one producer warp
constexpr int MAXG = 4;
constexpr int NST = 3;                    // ring stages
constexpr int SP = 16;                    // positions per stage
constexpr int STAGE_K = SP * 8 * 128;     // bytes of K (and of V) per stage: 16 positions x up to 8 heads
constexpr int MAX_GRID = 1024;            // CTAs per launch (partial slots reserved per call)
constexpr int MAX_B = 8192;
constexpr int SMEM_BASE = 1024 + NST * 2 * STAGE_K + 64;

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
  int B, cap, H, Hk, G;
  float scale_log2;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

__device__ __forceinline__ int row_len(const Params& p, int b) {
  const int L = p.valid_length[b];
  return L <= 0 ? p.cap : min(L, p.cap);
}

__device__ __forceinline__ int row_slot(const Params& p, int b) {
  return (p.nk != nullptr && p.positions != nullptr) ? min(max(p.positions[b], 0), p.cap - 1) : -1;
}

// The CTA whose share [floor(i*T/g), floor((i+1)*T/g)) holds position x.
__device__ __forceinline__ int cta_of(long long x, long long total, int g) {
  return (int)(((x + 1) * g + total - 1) / total) - 1;
}

__device__ __forceinline__ void compute_bar() { asm volatile("bar.sync 1, 256;\n" ::: "memory"); }

template <int G>
__global__ void __launch_bounds__(THREADS, 2)
    decode_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, Params p) {
  extern __shared__ uint8_t smem_raw[];
  // Offset from the __shared__ array itself so accesses keep the shared state space.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  int* pref = reinterpret_cast<int*>(smem + NST * 2 * STAGE_K + 64);  // [B + 1] exclusive prefix of lengths
  __shared__ int s_wsum[WARPS + 1], s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t sb = smem_u32(smem);
  const uint32_t bars = sb + NST * 2 * STAGE_K;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (NST + s); };
  int* status = &g_dec_status;
  const long long row_elems = (long long)p.Hk * HD;

  // Exclusive prefix of the rows' valid lengths.
  {
    const int per = cdiv(p.B, THREADS);
    const int r0 = min(p.B, tid * per), r1 = min(p.B, r0 + per);
    int local = 0;
    for (int r = r0; r < r1; ++r) local += row_len(p, r);
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
      pref[r] = off;
      off += row_len(p, r);
    }
    if (tid == THREADS - 1) pref[p.B] = off;
    __syncthreads();
  }
  const long long total = pref[p.B];
  // Appends whose slot is not a valid position of the row (at or beyond
  // valid_length): one CTA per row, nothing reads that slot this step.
  for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
    const int wpos = row_slot(p, b);
    if (wpos >= 0 && wpos >= row_len(p, b) && tid < (int)(row_elems / 8)) {
      for (int i = tid; i < (int)(row_elems / 8); i += THREADS) {
        *reinterpret_cast<uint4*>(p.kc + ((long long)b * p.cap + wpos) * row_elems + i * 8) =
            *reinterpret_cast<const uint4*>(p.nk + (long long)b * row_elems + i * 8);
        *reinterpret_cast<uint4*>(p.vc + ((long long)b * p.cap + wpos) * row_elems + i * 8) =
            *reinterpret_cast<const uint4*>(p.nv + (long long)b * row_elems + i * 8);
      }
    }
  }
  const int g = (int)min((long long)gridDim.x, total);  // every share is nonempty
  const int i = blockIdx.x;
  if (i >= g) return;
  const long long x0 = i * total / g, x1 = (i + 1) * total / g;
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
    // Producer: per stage and KV head, one 16-position x 64-dim TMA box of K
    // and one of V (128-byte swizzle), so each head's tile is conflict-free
    // for ldmatrix.
    if (lane == 0) {
      tc::tma_prefetch_desc(&tk);
      tc::tma_prefetch_desc(&tv);
      int it = 0;
      bool ok = true;
      for (int b = b0; ok && b < p.B && pref[b] < x1; ++b) {
        const int lo = (int)(max(x0, (long long)pref[b]) - pref[b]);
        const int hi = (int)(min(x1, (long long)pref[b + 1]) - pref[b]);
        for (int p0 = lo; p0 < hi; p0 += SP, ++it) {
          const int st = it % NST;
          if (!(ok = tc::mbar_wait(empty_bar(st), ((it / NST) & 1) ^ 1, status, 1))) break;
          tc::mbar_expect_tx(full_bar(st), 2 * p.Hk * SP * 128);
          for (int h = 0; h < p.Hk; ++h) {
            tc::tma_load_2d(sb + st * 2 * STAGE_K + h * 2048, &tk, h * HD, b * p.cap + p0, full_bar(st));
            tc::tma_load_2d(sb + st * 2 * STAGE_K + STAGE_K + h * 2048, &tv, h * HD, b * p.cap + p0, full_bar(st));
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
  int it = 0;
  bool ok = true;
  for (int b = b0; b < p.B && pref[b] < x1; ++b) {
    const int lo = (int)(max(x0, (long long)pref[b]) - pref[b]);
    const int hi = (int)(min(x1, (long long)pref[b + 1]) - pref[b]);
    const int L = p.valid_length[b];
    const bool uniform = L <= 0;
    const int wpos = row_slot(p, b);
    const bool own_slot = wpos >= lo && wpos < hi;
    if (own_slot) {
      // The cache append of this row; stage tiles may hold the old row at
      // wpos, which each warp overwrites in shared memory below.
      for (int e = tid; e < (int)(row_elems / 8); e += 32 * WARPS) {
        *reinterpret_cast<uint4*>(p.kc + ((long long)b * p.cap + wpos) * row_elems + e * 8) =
            *reinterpret_cast<const uint4*>(p.nk + (long long)b * row_elems + e * 8);
        *reinterpret_cast<uint4*>(p.vc + ((long long)b * p.cap + wpos) * row_elems + e * 8) =
            *reinterpret_cast<const uint4*>(p.nv + (long long)b * row_elems + e * 8);
      }
    }
    // Q fragments (unscaled bf16; rows >= G are zero).
    uint32_t qa[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      qa[kk][0] = qa[kk][1] = qa[kk][2] = qa[kk][3] = 0u;
      if (active && g4 < G) {
        const __nv_bfloat16* qr = p.q + ((long long)b * p.H + hk * G + g4) * HD + kk * 16 + 2 * c4;
        qa[kk][0] = *reinterpret_cast<const uint32_t*>(qr);
        qa[kk][2] = *reinterpret_cast<const uint32_t*>(qr + 8);
      }
    }
    float o[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float m = -INFINITY, l = 0.f;
    const float sl2 = p.scale_log2;
    for (int p0 = lo; p0 < hi; p0 += SP, ++it) {
      const int st = it % NST;
      // After a timed-out wait the warp skips the remaining waits but keeps
      // the named-barrier schedule of the other compute warps.
      if (ok) ok = tc::mbar_wait(full_bar(st), (it / NST) & 1, status, 2);
      if (ok && active) {
        const int np = min(SP, hi - p0);
        const uint32_t kt = sb + st * 2 * STAGE_K + hk * 2048, vt = kt + STAGE_K;
        if (own_slot && wpos >= p0 && wpos < p0 + np) {
          // Patch the new token's key / value row into this head's tiles.
          const int r = wpos - p0;
          if (lane < 8) {
            const uint4 nk4 = *reinterpret_cast<const uint4*>(p.nk + ((long long)b * p.Hk + hk) * HD + lane * 8);
            const uint4 nv4 = *reinterpret_cast<const uint4*>(p.nv + ((long long)b * p.Hk + hk) * HD + lane * 8);
            asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(kt + swz64(r, lane * 8)), "r"(nk4.x), "r"(nk4.y),
                         "r"(nk4.z), "r"(nk4.w));
            asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(vt + swz64(r, lane * 8)), "r"(nv4.x), "r"(nv4.y),
                         "r"(nv4.z), "r"(nv4.w));
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
    // Segment partial of rows g4 < G: the quad's four lanes hold 16 dims each.
    const long long slot = (long long)i + b;
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (active && g4 < G) {
      const long long pi = slot * p.H + hk * G + g4;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
        *reinterpret_cast<float2*>(p.part_o + pi * HD + nt * 8 + 2 * c4) = make_float2(o[nt][0], o[nt][1]);
      if (c4 == 0) p.part_ml[pi] = make_float2(m, l);
    }
    // The last segment of row b to finish combines the row's partials.
    const int c0 = cta_of(pref[b], total, g), c1 = cta_of((long long)pref[b + 1] - 1, total, g);
    __threadfence();
    compute_bar();
    if (tid == 0) s_last = atomicAdd(p.tickets + b, 1) == c1 - c0;
    compute_bar();
    if (s_last) {
      __threadfence();
      for (int idx = tid; idx < p.H * HD; idx += 32 * WARPS) {
        const int h = idx / HD, d = idx % HD;
        float mx = -INFINITY;
        for (int c = c0; c <= c1; ++c) mx = fmaxf(mx, __ldcg(p.part_ml + ((long long)c + b) * p.H + h).x);
        float num = 0.f, den = 0.f;
        for (int c = c0; c <= c1; ++c) {
          const long long pi = ((long long)c + b) * p.H + h;
          const float2 ml = __ldcg(p.part_ml + pi);
          const float w = ex2(ml.x - mx);
          den += ml.y * w;
          num += __ldcg(p.part_o + pi * HD + d) * w;
        }
        p.o[((long long)b * p.H + h) * HD + d] = __float2bfloat16_rn(num / den);
      }
      if (tid == 0) p.tickets[b] = 0;
    }
    compute_bar();
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
  MFB_CHECK_ARG(((uintptr_t)kc & 15) == 0 && ((uintptr_t)vc & 15) == 0, "caches must be 16-byte aligned");
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
  p.G = H / Hk;
  p.scale_log2 = scale * kLog2e;
  int dev = 0, sms = 148;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  MFB_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = 2 * sms < MAX_GRID ? 2 * sms : MAX_GRID;
  const size_t smem = SMEM_BASE + sizeof(int) * (size_t)(B + 1);
  const int smem_max = SMEM_BASE + (int)sizeof(int) * (MAX_B + 1);
  CUtensorMap tk, tv;
  int st;
  const uint64_t rows = (uint64_t)B * capacity, cols = (uint64_t)Hk * HD;
  if ((st = tc::make_tmap_bf16(&tk, k_cache, cols, rows, cols, SP))) return st;
  if ((st = tc::make_tmap_bf16(&tv, v_cache, cols, rows, cols, SP))) return st;
  MFB_CUDA_TRY(cudaMemsetAsync(w.tickets, 0, sizeof(int) * (size_t)B, s));
  switch (p.G) {
    case 1:
      MFB_CUDA_TRY(cudaFuncSetAttribute(decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max));
      decode_kernel<1><<<grid, THREADS, smem, s>>>(tk, tv, p);
      break;
    case 2:
      MFB_CUDA_TRY(cudaFuncSetAttribute(decode_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max));
      decode_kernel<2><<<grid, THREADS, smem, s>>>(tk, tv, p);
      break;
    default:
      MFB_CUDA_TRY(cudaFuncSetAttribute(decode_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max));
      decode_kernel<4><<<grid, THREADS, smem, s>>>(tk, tv, p);
      break;
  }
  MFB_LAUNCH_CHECK("decode kernel");
  return MFB_OK;
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

// Device address of g_noalloc_scratch per device ordinal, resolved once per
// device with that device current (the host-side symbol is only a stand-in).
constexpr int kMaxDevices = 64;
static void* g_noalloc_ptr[kMaxDevices] = {nullptr};

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
  if (dec::g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    MFB_CUDA_TRY(cudaGetSymbolAddress(&ptr, dec::g_noalloc_scratch));
    dec::g_noalloc_ptr[dev] = ptr;
  }
  // The array keeps the previous call's contents; the run clears the per-row
  // tickets, which must start at zero, before the launch.
  const dec::Workspace w = dec::carve(dec::g_noalloc_ptr[dev], B, H);
  return dec::run(q, k_cache, v_cache, new_k, new_v, positions, valid_length, o, B, capacity, H, Hk, scale, w,
                  (cudaStream_t)stream);
}
