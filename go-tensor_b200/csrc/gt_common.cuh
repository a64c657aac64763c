// Shared definitions for the libgotensor_cuda kernels and C entry points.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "gt_cuda.h"

struct gt_ctx {
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;       // all compute work
  cudaStream_t comm_stream = nullptr;  // gradient all-reduce
  cudaStream_t copy_stream = nullptr;  // host -> device copies that overlap compute
  cudaMemPool_t pool = nullptr;
  char name[256] = {0};
  void* nccl = nullptr;  // ncclComm_t
  int rank = 0, world = 1;
  void* encode_tiled = nullptr;  // cuTensorMapEncodeTiled entry point
  cudaEvent_t fork = nullptr, join = nullptr;  // compute <-> comm ordering
  cudaEvent_t marks[8] = {};                   // gt_mark timing points
  struct gt_gemm_timer* gemm_timer = nullptr;  // gt_gemm_timer_start .. _stop
  int gemm_sm_reserve = 0;  // SMs the GEMM kernels leave free (gt_set_gemm_sm_reserve)
  unsigned int* adam_done = nullptr;  // 4 bytes of device memory: the Adam kernel's finished-block count
};

namespace gt {

// Returns a malloc'd message the caller frees with gt_free_error.
char* errorf(const char* fmt, ...);

inline char* cuda_error(cudaError_t e, const char* what, const char* file, int line) {
  return errorf("%s: %s (%s:%d)", what, cudaGetErrorString(e), file, line);
}

// Makes ctx's device current on this thread (callers may switch threads).
char* enter(gt_ctx* ctx);

// Reports a pipeline wait of a tcgen05 kernel that gave up (and clears it).
char* tc_check_errors();

// Allocates scratch from the context's pool on its stream; freed with release.
char* scratch(gt_ctx* ctx, size_t bytes, void** out);
void release(gt_ctx* ctx, void* p);

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline int grid_for(const gt_ctx* ctx, int64_t n, int threads, int per_thread = 1) {
  int64_t want = ceil_div(n, (int64_t)threads * per_thread);
  int64_t cap = (int64_t)ctx->sm_count * 32;
  if (want < 1) want = 1;
  return (int)(want < cap ? want : cap);
}

}  // namespace gt

#define GT_CUDA(call)                                                          \
  do {                                                                         \
    cudaError_t _e = (call);                                                   \
    if (_e != cudaSuccess) return gt::cuda_error(_e, #call, __FILE__, __LINE__); \
  } while (0)

namespace gt {
void count_launch(int n = 1);
}

// Follows every kernel launch: counts it and reports launch failures.
#define GT_LAUNCH_CHECK()                                                      \
  do {                                                                         \
    gt::count_launch();                                                        \
    cudaError_t _e = cudaGetLastError();                                       \
    if (_e != cudaSuccess) return gt::cuda_error(_e, "kernel launch", __FILE__, __LINE__); \
  } while (0)

#define GT_TRY(expr)                  \
  do {                                \
    char* _m = (expr);                \
    if (_m) return _m;                \
  } while (0)

#define GT_ENTER(ctx)                                        \
  do {                                                       \
    if (!(ctx)) return gt::errorf("gt: null context");       \
    GT_TRY(gt::enter(ctx));                                  \
  } while (0)

#define GT_CHECK_DTYPE(dt)                                                           \
  do {                                                                               \
    if ((dt) != GT_FLOAT32 && (dt) != GT_FLOAT64) return gt::errorf("gt: unknown dtype %d", (int)(dt)); \
  } while (0)

// Calls body with `using T = float` or `double` depending on dt.
#define GT_DISPATCH(dt, ...)          \
  do {                                \
    if ((dt) == GT_FLOAT64) {         \
      using T = double;               \
      __VA_ARGS__                     \
    } else {                          \
      using T = float;                \
      __VA_ARGS__                     \
    }                                 \
  } while (0)

namespace gt {

// Exactly rounded arithmetic in T, never contracted into FMA, so that every
// intermediate is rounded where go-tensor's CPU backend rounds it.
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double div_rn(double a, double b) { return __ddiv_rn(a, b); }
__device__ __forceinline__ float sqrt_rn(float a) { return __fsqrt_rn(a); }
__device__ __forceinline__ double sqrt_rn(double a) { return __dsqrt_rn(a); }

// Go's builtin max for floats: NaN propagates, max(-0, +0) = +0.
template <typename T>
__device__ __forceinline__ T go_max(T a, T b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}

// out[c] = sum over r of part[r * cols + c], for cols columns and rows partial
// rows, in a fixed order (deterministic): a block of 32 warps takes 32
// consecutive columns; warp w adds rows [w * rows / 32, (w + 1) * rows / 32)
// in order (each load a coalesced 128-byte row), and the 32 warp sums are
// then added in warp order. Launch with ceil(cols / 32) blocks of 1024
// threads.
template <typename T>
__global__ void __launch_bounds__(1024) column_sums_kernel(const T* __restrict__ part, int64_t rows, int64_t cols,
                                                           T* __restrict__ out) {
  __shared__ T ws[32][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  const int64_t r0 = w * rows / 32, r1 = (w + 1) * rows / 32;
  T acc = (T)0;
  if (c < cols) {
    if (r0 < r1) acc = part[r0 * cols + c];
#pragma unroll 8
    for (int64_t r = r0 + 1; r < r1; r++) acc = acc + part[r * cols + c];
  }
  ws[w][lane] = acc;
  __syncthreads();
  if (w == 0 && c < cols) {
    T s = (T)0;
    bool first = true;
    for (int k = 0; k < 32; k++)
      if (k * rows / 32 < (k + 1) * rows / 32) {
        s = first ? ws[k][lane] : s + ws[k][lane];
        first = false;
      }
    out[c] = s;
  }
}

// Forward activations, evaluated like go-tensor's CPU backend: ReLU is Go's
// max(x, 0); Tanh and Sigmoid are computed in float64 then rounded to T
// (internal/cpu/cpu.go:110-135).
template <typename T>
__device__ __forceinline__ T act_fwd(int act, T z) {
  switch (act) {
    case GT_ACT_RELU: return go_max(z, (T)0);
    case GT_ACT_TANH: return (T)tanh((double)z);
    case GT_ACT_SIGMOID: return (T)(1.0 / (1.0 + exp(-(double)z)));
    default: return z;
  }
}

// g * act'(.) given the activation's output y, with the reference's chain of
// rounded ops (tensor/ops.go:110, 116, 123):
//   ReLU:    g * Step(x)            (Step(x) == Step(y) for y = max(x, 0))
//   Tanh:    g * ((-(y*y)) + 1)
//   Sigmoid: g * (y * ((-y) + 1))
template <typename T>
__device__ __forceinline__ T act_bwd(int act, T g, T y) {
  switch (act) {
    case GT_ACT_RELU: return mul_rn(g, y > (T)0 ? (T)1 : (T)0);
    case GT_ACT_TANH: return mul_rn(g, add_rn(-mul_rn(y, y), (T)1));
    case GT_ACT_SIGMOID: return mul_rn(g, mul_rn(y, add_rn(-y, (T)1)));
    default: return g;
  }
}

}  // namespace gt
