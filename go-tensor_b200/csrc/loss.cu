// Mean-squared-error and binary cross-entropy, forward and backward in one
// pass over the elements (nn/loss.go:6-9 and 17-22). Each intermediate is
// rounded where the reference's op chain rounds it, so the gradient equals the
// tape's element for element; only the order of the loss sum differs (a
// fixed-shape tree here, sequential there).
//
//   MSELoss = Mean(Pow(pred - target, 2))            (tensor/ops.go:31, 84, 154)
//     d = pred - target, term = d*d (Pow in float64 of a rounded d, rounded)
//     dpred = T(1/n) * (Pow(d, 1) * 2)                (Pow backward, ops.go:85)
//   BCELoss = -Mean(t*log(p) + (1-t)*log(1-p))
//     term = t*T(log p) + (T(1) - t)*T(log(T(1) - p))  (Log in float64, ops.go:94)
//     with s = T(-1) * T(1/n) from the Neg and MulScalar backward:
//     dpred = (s*t)/p + -((s*(1-t))/(1-p))             (Mul, Log, Neg backward)
#include "gt_common.cuh"

namespace gt {

constexpr int LOSS_THREADS = 256;

template <typename T, bool BCE>
__global__ void __launch_bounds__(LOSS_THREADS)
    loss_terms_kernel(const T* __restrict__ pred, const T* __restrict__ target, int64_t n, T c,
                      T* __restrict__ partial, T* __restrict__ dpred) {
  __shared__ T part[LOSS_THREADS];
  T acc = (T)0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const T p = pred[i], t = target[i];
    T e, g;
    if (!BCE) {
      const T d = sub_rn(p, t);
      e = mul_rn(d, d);
      g = mul_rn(c, mul_rn(d, (T)2));
    } else {
      const T nt = add_rn(-t, (T)1), np = add_rn(-p, (T)1);
      e = add_rn(mul_rn(t, (T)log((double)p)), mul_rn(nt, (T)log((double)np)));
      const T s = -c;
      g = add_rn(div_rn(mul_rn(s, t), p), -div_rn(mul_rn(s, nt), np));
    }
    acc = add_rn(acc, e);
    if (dpred) dpred[i] = g;
  }
  part[threadIdx.x] = acc;
  __syncthreads();
  for (int s = LOSS_THREADS / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) part[threadIdx.x] = add_rn(part[threadIdx.x], part[threadIdx.x + s]);
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = part[0];
}

// loss = Sum(partials) * c, negated for BCE; the partials are added in a
// fixed order, so the result does not depend on timing.
template <typename T, bool BCE>
__global__ void loss_sum_kernel(const T* __restrict__ partial, int64_t nb, T c, T* __restrict__ loss) {
  __shared__ T part[1024];
  T acc = (T)0;
  for (int64_t i = threadIdx.x; i < nb; i += blockDim.x) acc = add_rn(acc, partial[i]);
  part[threadIdx.x] = acc;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) part[threadIdx.x] = add_rn(part[threadIdx.x], part[threadIdx.x + s]);
    __syncthreads();
  }
  if (threadIdx.x == 0) *loss = BCE ? -mul_rn(part[0], c) : mul_rn(part[0], c);
}

template <bool BCE>
static char* loss_fwd_bwd(gt_ctx* ctx, int dtype, const void* pred, const void* target, int64_t n, void* loss,
                          void* dpred, const char* name) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (n < 0 || !loss || (n > 0 && (!pred || !target))) return errorf("%s: bad arguments", name);
  const size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  const int64_t nb = n > 0 ? grid_for(ctx, n, LOSS_THREADS) : 0;
  void* partial = nullptr;
  GT_TRY(scratch(ctx, (size_t)(nb > 0 ? nb : 1) * es, &partial));
  GT_DISPATCH(dtype, {
    // Mean multiplies by 1/float64(n) rounded to T; an empty input gives
    // 0 * (1/0) = NaN, as in the reference.
    const T c = (T)(1.0 / (double)n);
    if (nb > 0)
      loss_terms_kernel<T, BCE><<<(unsigned)nb, LOSS_THREADS, 0, ctx->stream>>>((const T*)pred, (const T*)target, n,
                                                                                c, (T*)partial, (T*)dpred);
    loss_sum_kernel<T, BCE><<<1, 1024, 0, ctx->stream>>>((const T*)partial, nb, c, (T*)loss);
  });
  count_launch(nb > 0 ? 2 : 1);
  cudaError_t e = cudaGetLastError();
  release(ctx, partial);
  if (e != cudaSuccess) return cuda_error(e, name, __FILE__, __LINE__);
  return nullptr;
}

}  // namespace gt

using namespace gt;

extern "C" {

char* gt_mse_fwd_bwd(gt_ctx* ctx, int dtype, const void* pred, const void* target, int64_t n, void* loss,
                     void* dpred) {
  return loss_fwd_bwd<false>(ctx, dtype, pred, target, n, loss, dpred, "gt_mse_fwd_bwd");
}

char* gt_bce_fwd_bwd(gt_ctx* ctx, int dtype, const void* pred, const void* target, int64_t n, void* loss,
                     void* dpred) {
  return loss_fwd_bwd<true>(ctx, dtype, pred, target, n, loss, dpred, "gt_bce_fwd_bwd");
}

}  // extern "C"
