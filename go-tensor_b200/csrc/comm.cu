// Data-parallel gradient exchange over NCCL (NVLink 5 / NVSwitch on a B200
// node). The reference has no multi-device code; this is the one collective
// the data-parallel training step needs: an in-place average of the flat
// gradient buffer (or of one bucket of it) across ranks.
//
// NCCL is loaded with dlopen at first use so that a process that already
// holds a libnccl.so.2 (PyTorch's) shares it instead of loading a second
// copy. The communicator is created non-blocking and polled against a
// deadline: a missing rank makes gt_comm_init fail with an error rather than
// hang, and gt_comm_destroy(abort=1) tears down a communicator whose peers
// died.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <thread>

#include "gt_common.cuh"

namespace gt {

struct NcclApi {
  bool loaded = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

static NcclApi g_nccl;
static std::mutex g_nccl_mu;

static char* load_nccl() {
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  if (g_nccl.loaded) return nullptr;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return errorf("gt_comm: cannot load libnccl.so.2: %s", dlerror());
#define GT_SYM(field, name)                                                        \
  g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, name));         \
  if (!g_nccl.field) return errorf("gt_comm: libnccl.so.2 lacks %s", name);
  GT_SYM(GetUniqueId, "ncclGetUniqueId");
  GT_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
  GT_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
  GT_SYM(CommAbort, "ncclCommAbort");
  GT_SYM(CommDestroy, "ncclCommDestroy");
  GT_SYM(AllReduce, "ncclAllReduce");
  GT_SYM(GetErrorString, "ncclGetErrorString");
#undef GT_SYM
  g_nccl.loaded = true;
  return nullptr;
}

static char* nccl_error(ncclResult_t r, const char* what) {
  return errorf("%s: %s", what, g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "nccl error");
}

// A non-blocking communicator may return ncclInProgress from a call that is
// still being enqueued; it must not be used again until its state leaves
// ncclInProgress. Waits for that (bounded), reporting any error.
static char* nccl_settle(ncclComm_t comm, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return nullptr;
  if (r != ncclInProgress) return nccl_error(r, what);
  auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(60);
  ncclResult_t state = ncclInProgress;
  while (true) {
    ncclResult_t q = g_nccl.CommGetAsyncError(comm, &state);
    if (q != ncclSuccess) return nccl_error(q, "ncclCommGetAsyncError");
    if (state != ncclInProgress) break;
    if (std::chrono::steady_clock::now() > deadline) return errorf("%s: still in progress after 60 s", what);
    std::this_thread::yield();
  }
  return state == ncclSuccess ? nullptr : nccl_error(state, what);
}

}  // namespace gt

using namespace gt;

extern "C" {

char* gt_comm_unique_id(unsigned char id[128]) {
  GT_TRY(load_nccl());
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId uid;
  ncclResult_t r = g_nccl.GetUniqueId(&uid);
  if (r != ncclSuccess) return nccl_error(r, "ncclGetUniqueId");
  memcpy(id, &uid, 128);
  return nullptr;
}

char* gt_comm_init(gt_ctx* ctx, int rank, int world, const unsigned char id[128], int timeout_ms) {
  GT_ENTER(ctx);
  GT_TRY(load_nccl());
  if (ctx->nccl) return errorf("gt_comm_init: the context already has a communicator");
  if (world < 1 || rank < 0 || rank >= world) return errorf("gt_comm_init: rank %d of %d", rank, world);
  ncclUniqueId uid;
  memcpy(&uid, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = g_nccl.CommInitRankConfig(&comm, world, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_error(r, "ncclCommInitRankConfig");
  auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 1);
  ncclResult_t state = ncclInProgress;
  while (true) {
    r = g_nccl.CommGetAsyncError(comm, &state);
    if (r != ncclSuccess) {
      g_nccl.CommAbort(comm);
      return nccl_error(r, "ncclCommGetAsyncError");
    }
    if (state != ncclInProgress) break;
    if (std::chrono::steady_clock::now() > deadline) {
      g_nccl.CommAbort(comm);
      return errorf("gt_comm_init: rank %d of %d timed out after %d ms waiting for its peers", rank, world,
                    timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  if (state != ncclSuccess) {
    g_nccl.CommAbort(comm);
    return nccl_error(state, "ncclCommInitRankConfig");
  }
  ctx->nccl = comm;
  ctx->rank = rank;
  ctx->world = world;
  return nullptr;
}

char* gt_allreduce_avg(gt_ctx* ctx, int dtype, void* buf, int64_t n) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (!ctx->nccl) return errorf("gt_allreduce_avg: no communicator (call gt_comm_init)");
  if (n <= 0 || ctx->world == 1) return nullptr;
  ncclResult_t r = g_nccl.AllReduce(buf, buf, (size_t)n, dtype == GT_FLOAT64 ? ncclFloat64 : ncclFloat32, ncclAvg,
                                    (ncclComm_t)ctx->nccl, ctx->stream);
  return nccl_settle((ncclComm_t)ctx->nccl, r, "ncclAllReduce");
}

char* gt_allreduce_avg_async(gt_ctx* ctx, int dtype, void* buf, int64_t n) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (!ctx->nccl) return errorf("gt_allreduce_avg_async: no communicator (call gt_comm_init)");
  if (n <= 0 || ctx->world == 1) return nullptr;
  GT_CUDA(cudaEventRecord(ctx->fork, ctx->stream));
  GT_CUDA(cudaStreamWaitEvent(ctx->comm_stream, ctx->fork, 0));
  ncclResult_t r = g_nccl.AllReduce(buf, buf, (size_t)n, dtype == GT_FLOAT64 ? ncclFloat64 : ncclFloat32, ncclAvg,
                                    (ncclComm_t)ctx->nccl, ctx->comm_stream);
  return nccl_settle((ncclComm_t)ctx->nccl, r, "ncclAllReduce");
}

char* gt_comm_wait(gt_ctx* ctx) {
  GT_ENTER(ctx);
  GT_CUDA(cudaEventRecord(ctx->join, ctx->comm_stream));
  GT_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->join, 0));
  return nullptr;
}

char* gt_comm_destroy(gt_ctx* ctx, int abort) {
  if (!ctx) return nullptr;
  if (!ctx->nccl) return nullptr;
  GT_TRY(gt::enter(ctx));
  ncclComm_t comm = (ncclComm_t)ctx->nccl;
  ctx->nccl = nullptr;
  if (abort) {
    ncclResult_t r = g_nccl.CommAbort(comm);
    return r == ncclSuccess ? nullptr : nccl_error(r, "ncclCommAbort");
  }
  // Destroying waits for the communicator's queued work on the streams.
  cudaStreamSynchronize(ctx->comm_stream);
  cudaStreamSynchronize(ctx->stream);
  ncclResult_t r = g_nccl.CommDestroy(comm);
  if (r == ncclInProgress) {
    // A non-blocking destroy finishes in the background; the handle is freed
    // by NCCL and must not be queried after this call.
    return nullptr;
  }
  return r == ncclSuccess ? nullptr : nccl_error(r, "ncclCommDestroy");
}

}  // extern "C"
