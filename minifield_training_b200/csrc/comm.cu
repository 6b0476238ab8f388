// NCCL communicator for the data-parallel gradient exchange of the encoder
// training step: the psum of (loss, count, gradient tree) over the "data" mesh
// axis (src/minifield_training/engine/step.py:36-78, psum at :62), and the
// scalar reductions and master all-gather of the sharded AdamW transaction.
//
// NCCL is loaded at run time (dlopen) from the path the host passes, so the
// library builds without NCCL and a process that already holds an NCCL (for
// instance through another framework) keeps one copy: dlopen of the same
// soname returns the loaded one.
//
// Failure handling (no wait without a limit): the communicator is created
// non-blocking, so initialisation and every collective call return at once and
// are polled with ncclCommGetAsyncError against a deadline. mfb_comm_wait
// polls a stream together with the communicator's asynchronous error; when a
// peer fails or stops, the deadline passes, the communicator is aborted
// (ncclCommAbort makes NCCL's kernels on this GPU return) and the call reports
// MFB_ERR_COMM. An aborted communicator rejects further collectives.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <time.h>
#include <unistd.h>

#include <mutex>

#include "common.cuh"

namespace mfb {
namespace comm {

struct Api {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommFinalize)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*ReduceScatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                cudaStream_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*Reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  ncclResult_t (*GetVersion)(int*);
  const char* (*GetErrorString)(ncclResult_t);
};

static Api g_api;
static void* g_handle = nullptr;
static std::mutex g_load_mutex;

struct Comm {
  ncclComm_t nc;
  int rank, world;
  double timeout_s;
  int aborted;
};

static double now_s() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

static const char* nccl_text(ncclResult_t r) { return g_api.GetErrorString ? g_api.GetErrorString(r) : "?"; }

static int require_loaded() {
  if (!g_handle) return set_error(MFB_ERR_UNSUPPORTED, "NCCL is not loaded (call mfb_comm_load first)");
  return MFB_OK;
}

// Polls the communicator until its pending operation settles: MFB_OK when it
// succeeded; on an NCCL error or when the deadline passes the communicator is
// aborted and MFB_ERR_COMM returned.
static int settle(Comm* c, ncclResult_t issued, const char* what) {
  if (issued != ncclSuccess && issued != ncclInProgress) {
    g_api.CommAbort(c->nc);
    c->aborted = 1;
    return set_error(MFB_ERR_COMM, "%s failed: %s (communicator aborted)", what, nccl_text(issued));
  }
  const double deadline = now_s() + c->timeout_s;
  for (;;) {
    ncclResult_t state = ncclSuccess;
    ncclResult_t q = g_api.CommGetAsyncError(c->nc, &state);
    if (q != ncclSuccess) state = q;
    if (state == ncclSuccess) return MFB_OK;
    if (state != ncclInProgress) {
      g_api.CommAbort(c->nc);
      c->aborted = 1;
      return set_error(MFB_ERR_COMM, "%s: NCCL reported %s (communicator aborted)", what, nccl_text(state));
    }
    if (now_s() > deadline) {
      g_api.CommAbort(c->nc);
      c->aborted = 1;
      return set_error(MFB_ERR_COMM, "%s did not complete within %.1f s (communicator aborted)", what,
                       c->timeout_s);
    }
    usleep(100);
  }
}

static int check_comm(void* comm, Comm** out) {
  int st = require_loaded();
  if (st) return st;
  MFB_CHECK_ARG(comm != nullptr, "communicator is NULL");
  Comm* c = static_cast<Comm*>(comm);
  if (c->aborted) return set_error(MFB_ERR_COMM, "the communicator was aborted after an earlier failure");
  *out = c;
  return MFB_OK;
}

static int map_dtype(int dtype, ncclDataType_t* t, size_t* bytes) {
  switch (dtype) {
    case MFB_COMM_F32: *t = ncclFloat32; *bytes = 4; return MFB_OK;
    case MFB_COMM_F64: *t = ncclFloat64; *bytes = 8; return MFB_OK;
    case MFB_COMM_BF16: *t = ncclBfloat16; *bytes = 2; return MFB_OK;
    case MFB_COMM_U8: *t = ncclUint8; *bytes = 1; return MFB_OK;
    case MFB_COMM_I32: *t = ncclInt32; *bytes = 4; return MFB_OK;
  }
  return set_error(MFB_ERR_INVALID, "unknown collective element type %d", dtype);
}

static int map_op(int op, ncclRedOp_t* r) {
  switch (op) {
    case MFB_COMM_SUM: *r = ncclSum; return MFB_OK;
    case MFB_COMM_MAX: *r = ncclMax; return MFB_OK;
    case MFB_COMM_MIN: *r = ncclMin; return MFB_OK;
  }
  return set_error(MFB_ERR_INVALID, "unknown reduction %d", op);
}

}  // namespace comm
}  // namespace mfb

using namespace mfb;
using namespace mfb::comm;

extern "C" int mfb_comm_load(const char* path, int* version) {
  std::lock_guard<std::mutex> lock(g_load_mutex);
  if (!g_handle) {
    const char* name = (path && *path) ? path : "libnccl.so.2";
    void* h = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
    if (!h) return set_error(MFB_ERR_UNSUPPORTED, "cannot load NCCL from %s: %s", name, dlerror());
    Api a{};
#define MFB_SYM(field, sym)                                                                      \
  a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, sym));                                  \
  if (!a.field) {                                                                                \
    dlclose(h);                                                                                  \
    return set_error(MFB_ERR_UNSUPPORTED, "NCCL at %s lacks %s", name, sym);                     \
  }
    MFB_SYM(GetUniqueId, "ncclGetUniqueId");
    MFB_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    MFB_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    MFB_SYM(CommAbort, "ncclCommAbort");
    MFB_SYM(CommFinalize, "ncclCommFinalize");
    MFB_SYM(CommDestroy, "ncclCommDestroy");
    MFB_SYM(AllReduce, "ncclAllReduce");
    MFB_SYM(ReduceScatter, "ncclReduceScatter");
    MFB_SYM(AllGather, "ncclAllGather");
    MFB_SYM(Reduce, "ncclReduce");
    MFB_SYM(Broadcast, "ncclBroadcast");
    MFB_SYM(GroupStart, "ncclGroupStart");
    MFB_SYM(GroupEnd, "ncclGroupEnd");
    MFB_SYM(GetVersion, "ncclGetVersion");
    MFB_SYM(GetErrorString, "ncclGetErrorString");
#undef MFB_SYM
    g_api = a;
    g_handle = h;
  }
  if (version) g_api.GetVersion(version);
  return MFB_OK;
}

extern "C" int mfb_comm_unique_id(void* id, size_t bytes) {
  int st = require_loaded();
  if (st) return st;
  MFB_CHECK_ARG(id && bytes >= sizeof(ncclUniqueId), "unique id buffer needs %zu bytes", sizeof(ncclUniqueId));
  ncclUniqueId u;
  ncclResult_t r = g_api.GetUniqueId(&u);
  if (r != ncclSuccess) return set_error(MFB_ERR_COMM, "ncclGetUniqueId failed: %s", nccl_text(r));
  memcpy(id, &u, sizeof(u));
  return MFB_OK;
}

extern "C" size_t mfb_comm_unique_id_bytes(void) { return sizeof(ncclUniqueId); }

extern "C" int mfb_comm_init(const void* id, size_t id_bytes, int world, int rank, double timeout_s, void** comm) {
  int st = require_loaded();
  if (st) return st;
  MFB_CHECK_ARG(id && id_bytes == sizeof(ncclUniqueId), "unique id must be %zu bytes", sizeof(ncclUniqueId));
  MFB_CHECK_ARG(world >= 1 && rank >= 0 && rank < world, "rank %d out of range for %d ranks", rank, world);
  MFB_CHECK_ARG(timeout_s > 0, "timeout must be positive");
  MFB_CHECK_ARG(comm != nullptr, "comm output is NULL");
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  Comm* c = new Comm{nullptr, rank, world, timeout_s, 0};
  ncclResult_t r = g_api.CommInitRankConfig(&c->nc, world, u, rank, &config);
  if (c->nc == nullptr) {
    delete c;
    return set_error(MFB_ERR_COMM, "ncclCommInitRankConfig failed: %s", nccl_text(r));
  }
  if ((st = settle(c, r, "communicator initialisation"))) {
    delete c;  // settle aborted the communicator, which releases it
    return st;
  }
  *comm = c;
  return MFB_OK;
}

extern "C" int mfb_comm_allreduce(void* comm, const void* send, void* recv, size_t count, int dtype, int op,
                                  void* stream) {
  Comm* c = nullptr;
  int st = check_comm(comm, &c);
  if (st) return st;
  ncclDataType_t t;
  ncclRedOp_t r;
  size_t bytes;
  if ((st = map_dtype(dtype, &t, &bytes)) || (st = map_op(op, &r))) return st;
  MFB_CHECK_ARG(count == 0 || (send && recv), "NULL collective buffer");
  if (count == 0) return MFB_OK;
  return settle(c, g_api.AllReduce(send, recv, count, t, r, c->nc, (cudaStream_t)stream), "all-reduce");
}

extern "C" int mfb_comm_reduce_scatter(void* comm, const void* send, void* recv, size_t recv_count, int dtype, int op,
                                       void* stream) {
  Comm* c = nullptr;
  int st = check_comm(comm, &c);
  if (st) return st;
  ncclDataType_t t;
  ncclRedOp_t r;
  size_t bytes;
  if ((st = map_dtype(dtype, &t, &bytes)) || (st = map_op(op, &r))) return st;
  MFB_CHECK_ARG(recv_count == 0 || (send && recv), "NULL collective buffer");
  if (recv_count == 0) return MFB_OK;
  return settle(c, g_api.ReduceScatter(send, recv, recv_count, t, r, c->nc, (cudaStream_t)stream),
                "reduce-scatter");
}

extern "C" int mfb_comm_allgather(void* comm, const void* send, void* recv, size_t send_count, int dtype,
                                  void* stream) {
  Comm* c = nullptr;
  int st = check_comm(comm, &c);
  if (st) return st;
  ncclDataType_t t;
  size_t bytes;
  if ((st = map_dtype(dtype, &t, &bytes))) return st;
  MFB_CHECK_ARG(send_count == 0 || (send && recv), "NULL collective buffer");
  if (send_count == 0) return MFB_OK;
  return settle(c, g_api.AllGather(send, recv, send_count, t, c->nc, (cudaStream_t)stream), "all-gather");
}

extern "C" int mfb_comm_reduce(void* comm, const void* send, void* recv, size_t count, int dtype, int op, int root,
                               void* stream) {
  Comm* c = nullptr;
  int st = check_comm(comm, &c);
  if (st) return st;
  ncclDataType_t t;
  ncclRedOp_t r;
  size_t bytes;
  if ((st = map_dtype(dtype, &t, &bytes)) || (st = map_op(op, &r))) return st;
  MFB_CHECK_ARG(root >= 0 && root < c->world, "root %d out of range for %d ranks", root, c->world);
  MFB_CHECK_ARG(count == 0 || (send && (recv || c->rank != root)), "NULL collective buffer");
  if (count == 0) return MFB_OK;
  return settle(c, g_api.Reduce(send, recv, count, t, r, root, c->nc, (cudaStream_t)stream), "reduce");
}

extern "C" int mfb_comm_broadcast(void* comm, const void* send, void* recv, size_t count, int dtype, int root,
                                  void* stream) {
  Comm* c = nullptr;
  int st = check_comm(comm, &c);
  if (st) return st;
  ncclDataType_t t;
  size_t bytes;
  if ((st = map_dtype(dtype, &t, &bytes))) return st;
  MFB_CHECK_ARG(root >= 0 && root < c->world, "root %d out of range for %d ranks", root, c->world);
  MFB_CHECK_ARG(count == 0 || (recv && (send || c->rank != root)), "NULL collective buffer");
  if (count == 0) return MFB_OK;
  return settle(c, g_api.Broadcast(send, recv, count, t, root, c->nc, (cudaStream_t)stream), "broadcast");
}

extern "C" int mfb_comm_wait(void* comm, void* stream, double timeout_s) {
  Comm* c = nullptr;
  int st = check_comm(comm, &c);
  if (st) return st;
  MFB_CHECK_ARG(timeout_s > 0, "timeout must be positive");
  const double deadline = now_s() + timeout_s;
  for (;;) {
    cudaError_t q = cudaStreamQuery((cudaStream_t)stream);
    if (q == cudaSuccess) return MFB_OK;
    if (q != cudaErrorNotReady) return cuda_error(q, "mfb_comm_wait stream query");
    ncclResult_t state = ncclSuccess;
    if (g_api.CommGetAsyncError(c->nc, &state) != ncclSuccess || (state != ncclSuccess && state != ncclInProgress)) {
      g_api.CommAbort(c->nc);
      c->aborted = 1;
      return set_error(MFB_ERR_COMM, "a collective failed: %s (communicator aborted)", nccl_text(state));
    }
    if (now_s() > deadline) {
      g_api.CommAbort(c->nc);
      c->aborted = 1;
      return set_error(MFB_ERR_COMM, "stream work did not finish within %.1f s (communicator aborted)", timeout_s);
    }
    usleep(50);
  }
}

extern "C" int mfb_comm_abort(void* comm) {
  int st = require_loaded();
  if (st) return st;
  MFB_CHECK_ARG(comm != nullptr, "communicator is NULL");
  Comm* c = static_cast<Comm*>(comm);
  if (!c->aborted) g_api.CommAbort(c->nc);
  c->aborted = 1;
  return MFB_OK;
}

extern "C" int mfb_comm_destroy(void* comm) {
  int st = require_loaded();
  if (st) return st;
  if (!comm) return MFB_OK;
  Comm* c = static_cast<Comm*>(comm);
  if (!c->aborted) {
    // Finalize flushes outstanding operations (polled with the deadline),
    // then destroy frees the resources.
    ncclResult_t r = g_api.CommFinalize(c->nc);
    if ((st = settle(c, r, "communicator finalize"))) {
      delete c;
      return st;  // settle aborted it (abort also frees it)
    }
    g_api.CommDestroy(c->nc);
  }
  delete c;
  return MFB_OK;
}

extern "C" int mfb_comm_rank(void* comm, int* rank, int* world) {
  MFB_CHECK_ARG(comm && rank && world, "NULL argument");
  const Comm* c = static_cast<const Comm*>(comm);
  *rank = c->rank;
  *world = c->world;
  return MFB_OK;
}
