// Runtime helpers of the C ABI: error reporting, device memory, streams and
// events. They let a host without its own device allocator (ctypes + NumPy,
// or a JAX FFI shim in tests) drive the kernels.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace mfb {

static thread_local char g_last_error[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_error(cudaError_t err, const char* where) {
  return set_error(MFB_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorString(err), cudaGetErrorName(err));
}

}  // namespace mfb

extern "C" {

const char* mfb_last_error(void) { return mfb::g_last_error; }

int mfb_version(void) { return 1; }

int mfb_device_count(int* count) {
  MFB_CHECK_ARG(count != nullptr, "count is NULL");
  MFB_CUDA_TRY(cudaGetDeviceCount(count));
  return MFB_OK;
}

int mfb_set_device(int device) {
  MFB_CUDA_TRY(cudaSetDevice(device));
  return MFB_OK;
}

int mfb_device_sm_version(int device, int* major, int* minor) {
  MFB_CHECK_ARG(major && minor, "NULL out-param");
  MFB_CUDA_TRY(cudaDeviceGetAttribute(major, cudaDevAttrComputeCapabilityMajor, device));
  MFB_CUDA_TRY(cudaDeviceGetAttribute(minor, cudaDevAttrComputeCapabilityMinor, device));
  return MFB_OK;
}

int mfb_malloc(void** ptr, size_t bytes) {
  MFB_CHECK_ARG(ptr != nullptr, "ptr is NULL");
  *ptr = nullptr;
  if (bytes == 0) return MFB_OK;
  MFB_CUDA_TRY(cudaMalloc(ptr, bytes));
  return MFB_OK;
}

int mfb_free(void* ptr) {
  if (ptr) MFB_CUDA_TRY(cudaFree(ptr));
  return MFB_OK;
}

int mfb_host_alloc(void** ptr, size_t bytes) {
  MFB_CHECK_ARG(ptr != nullptr, "ptr is NULL");
  *ptr = nullptr;
  if (bytes == 0) return MFB_OK;
  MFB_CUDA_TRY(cudaMallocHost(ptr, bytes));
  return MFB_OK;
}

int mfb_host_free(void* ptr) {
  if (ptr) MFB_CUDA_TRY(cudaFreeHost(ptr));
  return MFB_OK;
}

int mfb_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return MFB_OK;
  MFB_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
  return MFB_OK;
}

int mfb_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return MFB_OK;
  MFB_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  return MFB_OK;
}

int mfb_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return MFB_OK;
  MFB_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
  return MFB_OK;
}

int mfb_memcpy2d_d2d(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width, size_t height,
                     void* stream) {
  if (width == 0 || height == 0) return MFB_OK;
  MFB_CHECK_ARG(dst && src && width <= dst_pitch && width <= src_pitch, "bad strided copy (width %zu)", width);
  MFB_CUDA_TRY(cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width, height, cudaMemcpyDeviceToDevice,
                                 (cudaStream_t)stream));
  return MFB_OK;
}

int mfb_memset(void* dst, int value, size_t bytes, void* stream) {
  if (bytes == 0) return MFB_OK;
  MFB_CUDA_TRY(cudaMemsetAsync(dst, value, bytes, (cudaStream_t)stream));
  return MFB_OK;
}

int mfb_stream_create(void** stream) {
  MFB_CHECK_ARG(stream != nullptr, "stream is NULL");
  cudaStream_t s;
  MFB_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = s;
  return MFB_OK;
}

int mfb_stream_destroy(void* stream) {
  if (stream) MFB_CUDA_TRY(cudaStreamDestroy((cudaStream_t)stream));
  return MFB_OK;
}

int mfb_stream_sync(void* stream) {
  MFB_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
  return MFB_OK;
}

int mfb_device_sync(void) {
  MFB_CUDA_TRY(cudaDeviceSynchronize());
  return MFB_OK;
}

int mfb_device_reset(void) {
  MFB_CUDA_TRY(cudaDeviceReset());
  return MFB_OK;
}

int mfb_event_create(void** event) {
  MFB_CHECK_ARG(event != nullptr, "event is NULL");
  cudaEvent_t e;
  MFB_CUDA_TRY(cudaEventCreate(&e));
  *event = e;
  return MFB_OK;
}

int mfb_event_destroy(void* event) {
  if (event) MFB_CUDA_TRY(cudaEventDestroy((cudaEvent_t)event));
  return MFB_OK;
}

int mfb_event_record(void* event, void* stream) {
  MFB_CUDA_TRY(cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream));
  return MFB_OK;
}

// Later work on `stream` waits for `event`'s most recent record (no-op if never recorded).
int mfb_stream_wait_event(void* stream, void* event) {
  MFB_CHECK_ARG(event != nullptr, "event is NULL");
  MFB_CUDA_TRY(cudaStreamWaitEvent((cudaStream_t)stream, (cudaEvent_t)event, 0));
  return MFB_OK;
}

int mfb_event_elapsed_ms(void* start, void* end, float* ms) {
  MFB_CHECK_ARG(ms != nullptr, "ms is NULL");
  MFB_CUDA_TRY(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end));
  return MFB_OK;
}

// Work recorded on a stream between mfb_graph_begin and mfb_graph_end becomes
// one executable CUDA graph (relaxed capture: the library's host-side queries
// during capture, such as tensor-map encoding, are allowed); mfb_graph_launch
// replays it on a stream. Kernel arguments, buffers and sizes are fixed at
// capture; the buffers' contents may change between replays.
int mfb_graph_begin(void* stream) {
  MFB_CHECK_ARG(stream != nullptr, "graph capture needs a created stream (not the legacy default stream)");
  MFB_CUDA_TRY(cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeRelaxed));
  return MFB_OK;
}

int mfb_graph_end(void* stream, void** graph_exec) {
  MFB_CHECK_ARG(stream != nullptr && graph_exec != nullptr, "NULL graph argument");
  cudaGraph_t g = nullptr;
  MFB_CUDA_TRY(cudaStreamEndCapture((cudaStream_t)stream, &g));
  cudaGraphExec_t e = nullptr;
  const cudaError_t err = cudaGraphInstantiate(&e, g, 0);
  cudaGraphDestroy(g);
  if (err != cudaSuccess) return mfb::set_error(MFB_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(err));
  *graph_exec = e;
  return MFB_OK;
}

int mfb_graph_launch(void* graph_exec, void* stream) {
  MFB_CHECK_ARG(graph_exec != nullptr, "NULL graph");
  MFB_CUDA_TRY(cudaGraphLaunch((cudaGraphExec_t)graph_exec, (cudaStream_t)stream));
  return MFB_OK;
}

int mfb_graph_destroy(void* graph_exec) {
  if (graph_exec) MFB_CUDA_TRY(cudaGraphExecDestroy((cudaGraphExec_t)graph_exec));
  return MFB_OK;
}

}  // extern "C"
