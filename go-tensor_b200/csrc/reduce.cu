// Backend.Reduce (internal/backend/backend.go:145-147): Sum or Max over the
// middle axis of x viewed as (outer, n, inner); internal/cpu/cpu.go:270-296.
//
// Sums accumulate in the tensor's dtype, as the reference does, but in a tree
// instead of sequentially, so float32 results differ from the CPU by rounding
// only. Max follows Go's max() (NaN wins, max(-0, +0) = +0) and is exact.
//
// Two layouts:
//  * inner == 1: rows are contiguous; a warp reduces one row (or one chunk of
//    a row) with shuffles;
//  * inner > 1: a thread reduces one column, reading n values strided by inner,
//    which is coalesced across the threads of a warp.
// When outer*inner alone cannot fill the GPU, n is split into chunks whose
// partial results go to scratch memory and a second pass combines them in a
// fixed order, so results are deterministic.
#include "gt_common.cuh"

namespace gt {

template <typename T>
__device__ __forceinline__ T reduce_identity(int op) {
  return op == GT_MAX ? (T)(-INFINITY) : (T)0;
}

template <typename T>
__device__ __forceinline__ T reduce_op(int op, T a, T b) {
  return op == GT_MAX ? go_max(a, b) : add_rn(a, b);
}

// Warp per (row, split): out[row * nsplit + s] = reduce(x[row, s*chunk : ...]).
template <typename T>
__global__ void reduce_rows_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t rows, int64_t n,
                                   int op, int64_t chunk, int64_t nsplit) {
  const int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t t = warp; t < rows * nsplit; t += nwarps) {
    int64_t row = t / nsplit, s = t - row * nsplit;
    int64_t lo = s * chunk, hi = lo + chunk < n ? lo + chunk : n;
    const T* xr = x + row * n;
    // Start from the identity like the reference (a zero-filled sum, so that
    // -0 + -0 sums to +0); -inf never wins a Max over a real value.
    T acc = reduce_identity<T>(op);
    for (int64_t k = lo + lane; k < hi; k += 32) acc = reduce_op(op, acc, xr[k]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      T o = __shfl_down_sync(0xffffffffu, acc, off);
      acc = reduce_op(op, acc, o);
    }
    if (lane == 0) out[t] = acc;
  }
}

// Thread per (split, column): out[s * cols + c] with c = o*inner + i.
template <typename T>
__global__ void reduce_cols_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t outer, int64_t n,
                                   int64_t inner, int op, int64_t chunk, int64_t nsplit) {
  int64_t cols = outer * inner;
  int64_t total = cols * nsplit;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t s = t / cols, c = t - s * cols;
    int64_t o = c / inner, i = c - o * inner;
    int64_t lo = s * chunk, hi = lo + chunk < n ? lo + chunk : n;
    const T* xp = x + (o * n) * inner + i;
    // four interleaved accumulators, so that four loads are in flight, added
    // in a fixed order at the end
    T a0 = reduce_identity<T>(op), a1 = a0, a2 = a0, a3 = a0;
    int64_t k = lo;
    for (; k + 4 <= hi; k += 4) {
      const T v0 = xp[k * inner], v1 = xp[(k + 1) * inner], v2 = xp[(k + 2) * inner], v3 = xp[(k + 3) * inner];
      a0 = reduce_op(op, a0, v0), a1 = reduce_op(op, a1, v1), a2 = reduce_op(op, a2, v2), a3 = reduce_op(op, a3, v3);
    }
    for (; k < hi; k++) a0 = reduce_op(op, a0, xp[k * inner]);
    out[t] = reduce_op(op, reduce_op(op, a0, a1), reduce_op(op, a2, a3));
  }
}

// Chooses the split of n. Returns nsplit >= 1.
static int64_t pick_split(const gt_ctx* ctx, int64_t tasks, int64_t n, int64_t lanes_per_task, int64_t min_chunk) {
  int64_t target = (int64_t)ctx->sm_count * 2048;  // resident threads on the GPU
  int64_t have = tasks * lanes_per_task;
  if (have >= target || n <= min_chunk) return 1;
  int64_t ns = ceil_div(target, have);
  int64_t max_ns = ceil_div(n, min_chunk);
  return ns < max_ns ? ns : max_ns;
}

// Plans a reduction: how many partial values it needs in scratch (0: none).
static int64_t partials_needed(const gt_ctx* ctx, int64_t outer, int64_t n, int64_t inner, int64_t* nsplit_out) {
  int64_t ns;
  if (inner == 1)
    ns = pick_split(ctx, outer, n, 32, 1024);
  else
    ns = pick_split(ctx, outer * inner, n, 1, 64);
  *nsplit_out = ns;
  return ns > 1 ? outer * inner * ns : 0;
}

template <typename T>
static char* launch_reduce(gt_ctx* ctx, int op, const T* x, T* out, int64_t outer, int64_t n, int64_t inner,
                           T* partials, int64_t nsplit) {
  const int threads = 256;
  int64_t chunk = ceil_div(n, nsplit);
  if (inner == 1) {
    T* dst = nsplit > 1 ? partials : out;
    int64_t warps = outer * nsplit;
    reduce_rows_kernel<T><<<grid_for(ctx, warps * 32, threads), threads, 0, ctx->stream>>>(x, dst, outer, n, op, chunk,
                                                                                          nsplit);
    GT_LAUNCH_CHECK();
    if (nsplit > 1) {  // rows of nsplit partials, contiguous per row
      reduce_rows_kernel<T><<<grid_for(ctx, outer * 32, threads), threads, 0, ctx->stream>>>(partials, out, outer,
                                                                                             nsplit, op, nsplit, 1);
      GT_LAUNCH_CHECK();
    }
  } else {
    T* dst = nsplit > 1 ? partials : out;
    int64_t total = outer * inner * nsplit;
    reduce_cols_kernel<T><<<grid_for(ctx, total, threads), threads, 0, ctx->stream>>>(x, dst, outer, n, inner, op, chunk,
                                                                                      nsplit);
    GT_LAUNCH_CHECK();
    if (nsplit > 1) {  // partials are (nsplit, outer*inner): reduce the middle axis
      int64_t cols = outer * inner;
      if (op == GT_SUM)  // 32 warps per 32 columns, in a fixed order
        column_sums_kernel<T><<<(unsigned)ceil_div(cols, 32), 1024, 0, ctx->stream>>>(partials, nsplit, cols, out);
      else
        reduce_cols_kernel<T><<<grid_for(ctx, cols, threads), threads, 0, ctx->stream>>>(partials, out, 1, nsplit,
                                                                                          cols, op, nsplit, 1);
      GT_LAUNCH_CHECK();
    }
  }
  return nullptr;
}

static char* check_reduce(int op, int64_t outer, int64_t n, int64_t inner) {
  if (op != GT_SUM && op != GT_MAX) return errorf("gt_reduce: unknown op %d", op);
  if (outer < 0 || n < 0 || inner < 0) return errorf("gt_reduce: negative size");
  if (op == GT_MAX && n == 0 && outer * inner > 0) return errorf("gt_reduce: Max over an empty axis");
  return nullptr;
}

}  // namespace gt

using namespace gt;

extern "C" char* gt_reduce(gt_ctx* ctx, int dtype, int op, const void* x, void* out, int64_t outer, int64_t n,
                           int64_t inner) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_reduce(op, outer, n, inner));
  if (outer * inner == 0) return nullptr;
  size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  if (n == 0) {  // Sum over an empty axis is zero
    GT_CUDA(cudaMemsetAsync(out, 0, outer * inner * es, ctx->stream));
    return nullptr;
  }
  int64_t nsplit;
  int64_t np = partials_needed(ctx, outer, n, inner, &nsplit);
  void* partials = nullptr;
  GT_TRY(scratch(ctx, np * es, &partials));
  char* err;
  GT_DISPATCH(dtype, {
    err = launch_reduce<T>(ctx, op, (const T*)x, (T*)out, outer, n, inner, (T*)partials, nsplit);
  });
  release(ctx, partials);
  return err;
}
