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
// HBM layout: caches [B, cap, Hk, 64] bf16 (decode.py:96-117), so one cache
// position of all KV heads is 1 KB contiguous. A CTA owns (row b, a chunk of
// CHUNK positions) and all KV heads: warp w streams KV head w's 128-byte rows
// with 16-byte non-allocating loads, 8 positions in flight per lane (unrolled),
// computes the GQA group's scores with 8-lane shuffles, keeps them in shared
// memory, and reduces P.V in FP32. Work is split over the cache length
// (split-K); each chunk writes (m, l, o) partials to the caller's workspace and
// the last chunk of a row to finish (atomic ticket, no waiting) combines them.
#include <math.h>

#include "common.cuh"

namespace mfb {
namespace dec {

constexpr int HD = 64;
constexpr int CHUNK = 256;
constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;
constexpr int MAXG = 4;
constexpr int UNROLL = 8;

struct Params {
  const __nv_bfloat16* q;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  const __nv_bfloat16* nk;
  const __nv_bfloat16* nv;
  const int* positions;
  const int* valid_length;
  __nv_bfloat16* o;
  float* part_o;   // [B][nch_max][H][64]
  float2* part_ml; // [B][nch_max][H]
  int* tickets;    // [B]
  int B, cap, H, Hk, G, nch_max;
  float scale_log2;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
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

template <int G>
__global__ void __launch_bounds__(THREADS) decode_kernel(Params p) {
  __shared__ float sS[WARPS][G][CHUNK];
  __shared__ int s_last;
  const int c = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int L = p.valid_length[b];
  const bool uniform = L <= 0;
  const int leff = uniform ? p.cap : min(L, p.cap);
  const int nch = cdiv(leff, CHUNK);
  const long long row_elems = (long long)p.Hk * HD;
  __nv_bfloat16* kb = p.kc + (long long)b * p.cap * row_elems;
  __nv_bfloat16* vb = p.vc + (long long)b * p.cap * row_elems;

  // Cache append (dynamic_update_slice clamps the slot into range).
  int wpos = -1;
  if (p.nk != nullptr && p.positions != nullptr) wpos = min(max(p.positions[b], 0), p.cap - 1);
  if (wpos >= 0 && wpos / CHUNK == c) {
    for (int i = tid; i < p.Hk * HD / 8; i += THREADS) {
      const uint4 nk = *reinterpret_cast<const uint4*>(p.nk + (long long)b * row_elems + i * 8);
      const uint4 nv = *reinterpret_cast<const uint4*>(p.nv + (long long)b * row_elems + i * 8);
      *reinterpret_cast<uint4*>(kb + (long long)wpos * row_elems + i * 8) = nk;
      *reinterpret_cast<uint4*>(vb + (long long)wpos * row_elems + i * 8) = nv;
    }
  }
  if (c >= nch) return;
  const int start = c * CHUNK;
  const int n = min(CHUNK, leff - start);
  const int p4 = lane >> 3, dc = (lane & 7) * 8;

  for (int hk = warp; hk < p.Hk; hk += WARPS) {
    float qv[G][8];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      {
        const uint4 u = *reinterpret_cast<const uint4*>(p.q + ((long long)b * p.H + hk * G + gi) * HD + dc);
        unpack8(u, qv[gi]);
#pragma unroll
        for (int i = 0; i < 8; ++i) qv[gi][i] *= p.scale_log2;
      }
    }
    const __nv_bfloat16* krow = kb + (long long)hk * HD + dc;
    const __nv_bfloat16* vrow = vb + (long long)hk * HD + dc;
    const __nv_bfloat16* nkrow = p.nk ? p.nk + ((long long)b * p.Hk + hk) * HD + dc : nullptr;
    const __nv_bfloat16* nvrow = p.nv ? p.nv + ((long long)b * p.Hk + hk) * HD + dc : nullptr;

    // Pass 1: scores (log2 domain) into shared memory.
    for (int base = 0; base < n; base += 4 * UNROLL) {
      uint4 kr[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int i = base + u * 4 + p4;
        const int pos = start + i;
        kr[u] = make_uint4(0, 0, 0, 0);
        if (i < n && !uniform) kr[u] = pos == wpos ? *reinterpret_cast<const uint4*>(nkrow) : ld_stream(krow + pos * row_elems);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int i = base + u * 4 + p4;
        float kf[8];
        unpack8(kr[u], kf);
#pragma unroll
        for (int gi = 0; gi < G; ++gi) {
          {
            float s = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) s = fmaf(qv[gi][e], kf[e], s);
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            s += __shfl_xor_sync(0xffffffffu, s, 4);
            if ((lane & 7) == 0 && i < n) sS[warp][gi][i] = uniform ? 0.f : s;
          }
        }
      }
    }
    __syncwarp();
    float m[G], l[G];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      m[gi] = -INFINITY;
      l[gi] = 0.f;
      {
        for (int i = lane; i < n; i += 32) m[gi] = fmaxf(m[gi], sS[warp][gi][i]);
        m[gi] = warp_max(m[gi]);
        for (int i = lane; i < n; i += 32) {
          const float e = ex2(sS[warp][gi][i] - m[gi]);
          sS[warp][gi][i] = e;
          l[gi] += e;
        }
        l[gi] = warp_sum(l[gi]);
      }
    }
    __syncwarp();

    // Pass 2: o = P V over this chunk.
    float acc[G][8];
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[gi][e] = 0.f;
    for (int base = 0; base < n; base += 4 * UNROLL) {
      uint4 vr[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int i = base + u * 4 + p4;
        const int pos = start + i;
        vr[u] = make_uint4(0, 0, 0, 0);
        if (i < n) vr[u] = pos == wpos ? *reinterpret_cast<const uint4*>(nvrow) : ld_stream(vrow + pos * row_elems);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int i = base + u * 4 + p4;
        if (i < n) {
          float vf[8];
          unpack8(vr[u], vf);
#pragma unroll
          for (int gi = 0; gi < G; ++gi) {
            {
              const float pw = sS[warp][gi][i];
#pragma unroll
              for (int e = 0; e < 8; ++e) acc[gi][e] = fmaf(pw, vf[e], acc[gi][e]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          acc[gi][e] += __shfl_xor_sync(0xffffffffu, acc[gi][e], 8);
          acc[gi][e] += __shfl_xor_sync(0xffffffffu, acc[gi][e], 16);
        }
        const int h = hk * G + gi;
        const long long pi = ((long long)b * p.nch_max + c) * p.H + h;
        if (lane < 8) {
          float4* dst = reinterpret_cast<float4*>(p.part_o + pi * HD + dc);
          dst[0] = make_float4(acc[gi][0], acc[gi][1], acc[gi][2], acc[gi][3]);
          dst[1] = make_float4(acc[gi][4], acc[gi][5], acc[gi][6], acc[gi][7]);
        }
        if (lane == 0) p.part_ml[pi] = make_float2(m[gi], l[gi]);
      }
    }
    __syncwarp();
  }

  // Last chunk of row b to finish combines the partials.
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(p.tickets + b, 1);
    s_last = (prev == nch - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = tid; idx < p.H * HD; idx += THREADS) {
    const int h = idx / HD, d = idx % HD;
    float mx = -INFINITY;
    for (int cc = 0; cc < nch; ++cc) {
      const float2 ml = __ldcg(p.part_ml + ((long long)b * p.nch_max + cc) * p.H + h);
      mx = fmaxf(mx, ml.x);
    }
    float num = 0.f, den = 0.f;
    for (int cc = 0; cc < nch; ++cc) {
      const long long pi = ((long long)b * p.nch_max + cc) * p.H + h;
      const float2 ml = __ldcg(p.part_ml + pi);
      const float w = ex2(ml.x - mx);
      den += ml.y * w;
      num += __ldcg(p.part_o + pi * HD + d) * w;
    }
    p.o[((long long)b * p.H + h) * HD + d] = __float2bfloat16_rn(num / den);
  }
  if (tid == 0) p.tickets[b] = 0;
}

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct Workspace {
  float* part_o;
  float2* part_ml;
  int* tickets;
  size_t bytes;
};

Workspace carve(void* base, int B, int cap, int H) {
  const int nch = cdiv(cap, CHUNK);
  char* p = static_cast<char*>(base);
  Workspace w;
  size_t off = 0;
  w.part_o = reinterpret_cast<float*>(p + off);
  off += align256(sizeof(float) * (size_t)B * nch * H * HD);
  w.part_ml = reinterpret_cast<float2*>(p + off);
  off += align256(sizeof(float2) * (size_t)B * nch * H);
  w.tickets = reinterpret_cast<int*>(p + off);
  off += align256(sizeof(int) * (size_t)B);
  w.bytes = off;
  return w;
}

}  // namespace dec
}  // namespace mfb

using namespace mfb;

extern "C" size_t mfb_decode_workspace_size(int B, int capacity, int H, int D) {
  (void)D;
  if (B <= 0 || capacity <= 0 || H <= 0) return 0;
  return dec::carve(nullptr, B, capacity, H).bytes;
}

extern "C" int mfb_decode_attn(const uint16_t* q, uint16_t* k_cache, uint16_t* v_cache, const uint16_t* new_k,
                               const uint16_t* new_v, const int32_t* positions, const int32_t* valid_length,
                               uint16_t* o, int B, int capacity, int H, int Hk, int D, float scale, void* workspace,
                               size_t workspace_bytes, void* stream) {
  MFB_CHECK_ARG(B > 0 && capacity > 0, "Cached attention needs a nonempty batch and cache (B=%d cap=%d)", B, capacity);
  MFB_CHECK_ARG(D == dec::HD, "Cached attention query/KV shapes are incompatible (head_dim %d; this build needs 64)", D);
  MFB_CHECK_ARG(H > 0 && Hk > 0 && H % Hk == 0, "Query heads must be divisible by KV heads (H=%d Hk=%d)", H, Hk);
  MFB_CHECK_ARG(H / Hk <= dec::MAXG, "GQA group size %d exceeds %d", H / Hk, dec::MAXG);
  MFB_CHECK_ARG(q && k_cache && v_cache && valid_length && o, "NULL tensor argument");
  MFB_CHECK_ARG((new_k == nullptr) == (new_v == nullptr), "new_k and new_v must both be given or both be NULL");
  MFB_CHECK_ARG(new_k == nullptr || positions != nullptr, "positions are required with new_k/new_v");
  const dec::Workspace w = dec::carve(workspace, B, capacity, H);
  if (!workspace || workspace_bytes < w.bytes)
    return set_error(MFB_ERR_WORKSPACE, "decode workspace needs %zu bytes", w.bytes);
  dec::Params p{};
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
  p.nch_max = cdiv(capacity, dec::CHUNK);
  p.scale_log2 = scale * kLog2e;
  cudaStream_t s = (cudaStream_t)stream;
  MFB_CUDA_TRY(cudaMemsetAsync(w.tickets, 0, sizeof(int) * (size_t)B, s));
  dim3 grid(p.nch_max, B);
  switch (p.G) {
    case 1:
      dec::decode_kernel<1><<<grid, dec::THREADS, 0, s>>>(p);
      break;
    case 2:
      dec::decode_kernel<2><<<grid, dec::THREADS, 0, s>>>(p);
      break;
    case 4:
      dec::decode_kernel<4><<<grid, dec::THREADS, 0, s>>>(p);
      break;
    default:
      return set_error(MFB_ERR_UNSUPPORTED, "GQA group size %d unsupported (1, 2 or 4)", p.G);
  }
  MFB_LAUNCH_CHECK("mfb_decode_attn");
  return MFB_OK;
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
  MFB_CHECK_ARG(B > 0 && capacity > 0, "Cached attention needs a nonempty batch and cache (B=%d cap=%d)", B, capacity);
  MFB_CHECK_ARG(D == dec::HD, "Cached attention query/KV shapes are incompatible (head_dim %d; this build needs 64)", D);
  MFB_CHECK_ARG(H > 0 && Hk > 0 && H % Hk == 0, "Query heads must be divisible by KV heads (H=%d Hk=%d)", H, Hk);
  MFB_CHECK_ARG(q && k_cache && v_cache && valid_length && o, "NULL tensor argument");
  MFB_CHECK_ARG((new_k == nullptr) == (new_v == nullptr), "new_k and new_v must both be given or both be NULL");
  MFB_CHECK_ARG(new_k == nullptr || positions != nullptr, "positions are required with new_k/new_v");
  const size_t need = dec::carve(nullptr, B, capacity, H).bytes;
  MFB_CHECK_ARG(need <= (size_t)MFB_DECODE_NOALLOC_SCRATCH_BYTES,
                "mfb_decode_attn_noalloc: B=%d, capacity=%d, H=%d need %zu scratch bytes, above the fixed %d-byte "
                "maximum; use mfb_decode_attn with a caller workspace",
                B, capacity, H, need, (int)MFB_DECODE_NOALLOC_SCRATCH_BYTES);
  int dev = 0;
  MFB_CUDA_TRY(cudaGetDevice(&dev));
  MFB_CHECK_ARG(dev >= 0 && dev < dec::kMaxDevices, "device ordinal %d out of range", dev);
  if (dec::g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    MFB_CUDA_TRY(cudaGetSymbolAddress(&ptr, dec::g_noalloc_scratch));
    dec::g_noalloc_ptr[dev] = ptr;
  }
  const dec::Workspace w = dec::carve(dec::g_noalloc_ptr[dev], B, capacity, H);
  dec::Params p{};
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
  p.nch_max = cdiv(capacity, dec::CHUNK);
  p.scale_log2 = scale * kLog2e;
  cudaStream_t s = (cudaStream_t)stream;
  // The array keeps the previous call's contents: the per-row tickets must start at zero.
  MFB_CUDA_TRY(cudaMemsetAsync(w.tickets, 0, sizeof(int) * (size_t)B, s));
  dim3 grid(p.nch_max, B);
  switch (p.G) {
    case 1:
      dec::decode_kernel<1><<<grid, dec::THREADS, 0, s>>>(p);
      break;
    case 2:
      dec::decode_kernel<2><<<grid, dec::THREADS, 0, s>>>(p);
      break;
    case 4:
      dec::decode_kernel<4><<<grid, dec::THREADS, 0, s>>>(p);
      break;
    default:
      return set_error(MFB_ERR_UNSUPPORTED, "GQA group size %d unsupported (1, 2 or 4)", p.G);
  }
  MFB_LAUNCH_CHECK("mfb_decode_attn_noalloc");
  return MFB_OK;
}
