// Evaluation on the device: Tensor.Argmax (tensor/ops.go:176-192) and the
// correct-prediction count of the reference's accuracy loop
// (examples/mnist/main.go:120-133), so that evaluating a batch returns B
// indices or one count instead of the B x C logits.
#include "gt_common.cuh"

namespace gt {

// Argmax of every row of x (rows x n), with the reference's rule: start at
// index 0 and move to j whenever x[j] > x[best] (compared in float64, which
// orders float32 values the same way). So the first maximum wins, a NaN at
// index 0 is never replaced (every comparison with it is false), and a NaN
// anywhere else is never taken.
//
// One warp per row. Lane l scans j = l, l + 32, ... in increasing order and
// keeps the first maximum of its non-NaN elements (index 0 included in any
// case); the lanes' candidates then combine by (larger value, then smaller
// index), which is the first maximum of the row. A NaN at index 0 overrides.
template <typename T>
__global__ void argmax_rows_kernel(const T* __restrict__ x, int64_t rows, int64_t n, int32_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    const T* xr = x + r * n;
    const bool nan0 = isnan(xr[0]);
    T bv = (T)0;
    int64_t bi = -1;
#pragma unroll 8
    for (int64_t j = lane; j < n; j += 32) {
      const T v = xr[j];
      if ((j == 0 || !isnan(v)) && (bi < 0 || v > bv)) {
        bv = v;
        bi = j;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const T ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) out[r] = nan0 ? 0 : (int32_t)bi;
  }
}

// *count = number of i with a[i] == b[i]; integer sums, so the result does
// not depend on the order in which blocks add.
__global__ void count_equal_kernel(const int32_t* __restrict__ a, const int32_t* __restrict__ b, int64_t n,
                                   unsigned long long* __restrict__ count) {
  unsigned long long c = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    c += a[i] == b[i];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
  __shared__ unsigned long long part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x < 32) {
    c = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
    if (threadIdx.x == 0 && c) atomicAdd(count, c);
  }
}

}  // namespace gt

using namespace gt;

extern "C" {

char* gt_argmax_rows(gt_ctx* ctx, int dtype, const void* x, int64_t rows, int64_t n, int32_t* out) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (rows < 0 || n < 1 || n > INT32_MAX) return errorf("gt_argmax_rows: %lld rows of %lld", (long long)rows,
                                                        (long long)n);
  if (rows == 0) return nullptr;
  GT_DISPATCH(dtype, {
    argmax_rows_kernel<T><<<grid_for(ctx, rows * 32, 256), 256, 0, ctx->stream>>>((const T*)x, rows, n, out);
  });
  GT_LAUNCH_CHECK();
  return nullptr;
}

char* gt_count_equal(gt_ctx* ctx, const int32_t* a, const int32_t* b, int64_t n, int64_t* count) {
  GT_ENTER(ctx);
  if (n < 0 || !count) return errorf("gt_count_equal: bad arguments");
  GT_CUDA(cudaMemsetAsync(count, 0, sizeof(int64_t), ctx->stream));
  if (n == 0) return nullptr;
  count_equal_kernel<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(a, b, n, (unsigned long long*)count);
  GT_LAUNCH_CHECK();
  return nullptr;
}

}  // extern "C"
