// Context, errors and memory entry points of libgotensor_cuda.
//
// Memory comes from the device's stream-ordered pool (cudaMallocAsync with an
// unbounded release threshold), the CUDA counterpart of the Metal backend's
// size-class caching allocator (internal/mps/mps.go:29-164): a freed buffer
// goes back to the pool ordered after the work already queued on the stream,
// so it is reused without waiting for the GPU.
#include "gt_common.cuh"

#include <atomic>

namespace gt {

static std::atomic<int64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

char* errorf(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  size_t n = strlen(buf) + 1;
  char* out = (char*)malloc(n);
  if (out) memcpy(out, buf, n);
  return out;
}

char* enter(gt_ctx* ctx) {
  int cur = -1;
  GT_CUDA(cudaGetDevice(&cur));
  if (cur != ctx->device) GT_CUDA(cudaSetDevice(ctx->device));
  return nullptr;
}

char* scratch(gt_ctx* ctx, size_t bytes, void** out) {
  *out = nullptr;
  if (bytes == 0) return nullptr;
  GT_CUDA(cudaMallocFromPoolAsync(out, bytes, ctx->pool, ctx->stream));
  return nullptr;
}

void release(gt_ctx* ctx, void* p) {
  if (p) cudaFreeAsync(p, ctx->stream);
}

}  // namespace gt

extern "C" {

void gt_free_error(char* msg) { free(msg); }

int64_t gt_launch_count(void) { return gt::g_launches.load(std::memory_order_relaxed); }

char* gt_init(int device, gt_ctx** out) {
  if (!out) return gt::errorf("gt_init: null output");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return gt::cuda_error(e, "cudaGetDeviceCount", __FILE__, __LINE__);
  if (device < 0 || device >= count)
    return gt::errorf("gt_init: device %d does not exist (%d CUDA devices visible)", device, count);
  GT_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  GT_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10 || prop.minor != 0)
    return gt::errorf("gt_init: %s is compute capability %d.%d; this library is built for sm_100a (B200)",
                      prop.name, prop.major, prop.minor);
  gt_ctx* ctx = new gt_ctx();
  ctx->device = device;
  ctx->sm_count = prop.multiProcessorCount;
  snprintf(ctx->name, sizeof ctx->name, "%s", prop.name);
  GT_CUDA(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking));
  GT_CUDA(cudaStreamCreateWithFlags(&ctx->comm_stream, cudaStreamNonBlocking));
  GT_CUDA(cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking));
  GT_CUDA(cudaDeviceGetDefaultMemPool(&ctx->pool, device));
  uint64_t keep = UINT64_MAX;  // keep freed blocks cached, like a caching allocator
  GT_CUDA(cudaMemPoolSetAttribute(ctx->pool, cudaMemPoolAttrReleaseThreshold, &keep));
  GT_CUDA(cudaEventCreateWithFlags(&ctx->fork, cudaEventDisableTiming));
  GT_CUDA(cudaEventCreateWithFlags(&ctx->join, cudaEventDisableTiming));
  for (auto& e : ctx->marks) GT_CUDA(cudaEventCreate(&e));
  GT_CUDA(cudaMalloc((void**)&ctx->adam_done, sizeof(unsigned int)));
  GT_CUDA(cudaMemset(ctx->adam_done, 0, sizeof(unsigned int)));
  cudaDriverEntryPointQueryResult q;
  GT_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ctx->encode_tiled, cudaEnableDefault, &q));
  if (q != cudaDriverEntryPointSuccess) ctx->encode_tiled = nullptr;
  *out = ctx;
  return nullptr;
}

char* gt_destroy(gt_ctx* ctx) {
  if (!ctx) return nullptr;
  GT_TRY(gt::enter(ctx));
  if (ctx->nccl) GT_TRY(gt_comm_destroy(ctx, 0));
  GT_TRY(gt_gemm_timer_stop(ctx));
  cudaStreamSynchronize(ctx->stream);
  cudaStreamSynchronize(ctx->comm_stream);
  cudaStreamSynchronize(ctx->copy_stream);
  cudaEventDestroy(ctx->fork);
  cudaEventDestroy(ctx->join);
  for (auto& e : ctx->marks) cudaEventDestroy(e);
  if (ctx->adam_done) cudaFree(ctx->adam_done);
  cudaStreamDestroy(ctx->stream);
  cudaStreamDestroy(ctx->comm_stream);
  cudaStreamDestroy(ctx->copy_stream);
  delete ctx;
  return nullptr;
}

const char* gt_device_name(const gt_ctx* ctx) { return ctx ? ctx->name : ""; }
int gt_device_index(const gt_ctx* ctx) { return ctx ? ctx->device : -1; }
int gt_sm_count(const gt_ctx* ctx) { return ctx ? ctx->sm_count : 0; }
void* gt_stream(gt_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

char* gt_sync(gt_ctx* ctx) {
  GT_ENTER(ctx);
  GT_CUDA(cudaStreamSynchronize(ctx->stream));
  GT_CUDA(cudaGetLastError());
  return gt::tc_check_errors();
}

char* gt_alloc(gt_ctx* ctx, size_t bytes, void** out) {
  GT_ENTER(ctx);
  if (!out) return gt::errorf("gt_alloc: null output");
  // Never hand out a null pointer: zero-length storages are legal.
  GT_CUDA(cudaMallocFromPoolAsync(out, bytes ? bytes : 16, ctx->pool, ctx->stream));
  return nullptr;
}

char* gt_release(gt_ctx* ctx, void* ptr) {
  GT_ENTER(ctx);
  if (ptr) GT_CUDA(cudaFreeAsync(ptr, ctx->stream));
  return nullptr;
}

char* gt_pool_usage(gt_ctx* ctx, uint64_t* used_bytes, uint64_t* reserved_bytes) {
  GT_ENTER(ctx);
  uint64_t used = 0, reserved = 0;
  GT_CUDA(cudaMemPoolGetAttribute(ctx->pool, cudaMemPoolAttrUsedMemCurrent, &used));
  GT_CUDA(cudaMemPoolGetAttribute(ctx->pool, cudaMemPoolAttrReservedMemCurrent, &reserved));
  if (used_bytes) *used_bytes = used;
  if (reserved_bytes) *reserved_bytes = reserved;
  return nullptr;
}

char* gt_zero(gt_ctx* ctx, void* dst, size_t bytes) {
  GT_ENTER(ctx);
  if (bytes) GT_CUDA(cudaMemsetAsync(dst, 0, bytes, ctx->stream));
  return nullptr;
}

char* gt_upload(gt_ctx* ctx, void* dst, const void* src, size_t bytes) {
  GT_ENTER(ctx);
  // Pageable host memory: cudaMemcpyAsync stages the data before returning,
  // so the caller may reuse src at once.
  if (bytes) GT_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return nullptr;
}

char* gt_download(gt_ctx* ctx, void* dst, const void* src, size_t bytes) {
  GT_ENTER(ctx);
  if (bytes) GT_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  GT_CUDA(cudaStreamSynchronize(ctx->stream));
  return gt::tc_check_errors();
}

char* gt_upload_async(gt_ctx* ctx, void* dst, const void* src, size_t bytes) {
  GT_ENTER(ctx);
  if (bytes) GT_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return nullptr;
}

char* gt_download_async(gt_ctx* ctx, void* dst, const void* src, size_t bytes) {
  GT_ENTER(ctx);
  if (bytes) GT_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return nullptr;
}

char* gt_write(gt_ctx* ctx, void* dst, size_t dst_offset_bytes, const void* src, size_t bytes) {
  GT_ENTER(ctx);
  if (bytes)
    GT_CUDA(cudaMemcpyAsync((char*)dst + dst_offset_bytes, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
  return nullptr;
}

}  // extern "C"
