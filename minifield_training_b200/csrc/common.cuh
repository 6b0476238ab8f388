// Shared helpers for the sm_100a kernels of libmfb200: status codes, the
// thread-local last-error string, argument checks and small PTX wrappers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mfb200.h"

namespace mfb {

// Records a message for mfb_last_error() and returns the status.
int set_error(int status, const char* fmt, ...);
// Maps a CUDA runtime error to MFB_ERR_CUDA with context.
int cuda_error(cudaError_t err, const char* where);

}  // namespace mfb

#define MFB_CHECK_ARG(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) return mfb::set_error(MFB_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define MFB_CUDA_TRY(expr)                                     \
  do {                                                         \
    cudaError_t _e = (expr);                                   \
    if (_e != cudaSuccess) return mfb::cuda_error(_e, #expr);  \
  } while (0)

#define MFB_LAUNCH_CHECK(where)                                 \
  do {                                                          \
    cudaError_t _e = cudaGetLastError();                        \
    if (_e != cudaSuccess) return mfb::cuda_error(_e, where);   \
  } while (0)

namespace mfb {

__host__ __device__ inline int cdiv(int a, int b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// Device helpers (legacy-path PTX used by the warp-level kernels).
// ---------------------------------------------------------------------------

// Programmatic dependent launch. allow_dependents lets the next kernel on the
// stream start now if it was launched as a programmatic dependent (a decode
// GEMM streaming its weights); that kernel still runs wait_prerequisites, which
// returns once this grid has completed and its writes are visible, before it
// reads anything this grid produces. Both are no-ops without such a launch.
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void wait_prerequisites() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;  // zero-fill when the source row is out of range
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D (fp32)
__device__ __forceinline__ void mma_bf16_16816(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // .x = lo (low half), .y = hi
  return *reinterpret_cast<uint32_t*>(&v);
}


// 64-column bf16 tile rows are 128 bytes = 8 chunks of 16 bytes; chunk index is
// XOR-swizzled with (row % 8) so ldmatrix row reads hit distinct banks.
__device__ __forceinline__ uint32_t swz64(int row, int col) {
  return static_cast<uint32_t>(row * 128 + ((((col >> 3) ^ (row & 7)) << 4)) + ((col & 7) << 1));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr float kLog2e = 1.4426950408889634f;

}  // namespace mfb
