// Fused softmax cross-entropy, forward and backward in one pass over the
// logits. Replaces CrossEntropyLoss = -mean(Pick(LogSoftmax(x), y))
// (nn/loss.go:12-14, tensor/ops.go:335-359) and the ~12 primitive passes of
// its backward, following the reference's rounding of each intermediate:
//
//   m_i   = max_j x_ij                     (Reduce Max)
//   s_ij  = x_ij - m_i                     (Sub)
//   e_ij  = T(exp(double(s_ij)))           (Exp)
//   S_i   = sum_j e_ij                     (SumDim; tree order here)
//   L_i   = T(log(double(S_i)))            (Log)
//   p_i   = s_iy - L_i                     (Sub, then Pick)
//   loss  = -(sum_i p_i * T(1/B))          (Sum, MulScalar, Neg)
//   dx_ij = (-c * onehot_ij) + (c / S_i) * e_ij,  c = T(1/B)
//
// (The backward expression is what the reference's tape evaluates: the Neg /
// MulScalar / Sum / SumDim closures seed -c at the label, the Sub closure for
// L sums it back to c, Log divides by S and Exp multiplies by e.)
//
// A warp owns a row; the row's loss term goes to scratch and a second,
// single-block kernel sums the B terms in a fixed order, so the loss is
// deterministic. HBM traffic: read B*C logits, write B*C gradients.
#include "gt_common.cuh"

namespace gt {

// One warp per row. R > 0: the row (C <= 32 * R) is read into registers
// once, element j = lane + 32 k in slot k, so every pass after the first read
// works from registers in the same per-lane order as the R == 0 form, which
// streams the row from memory in each pass (any C).
template <typename T, int R>
__global__ void xent_rows_kernel(const T* __restrict__ x, const int32_t* __restrict__ labels, int64_t B, int64_t C,
                                 T c, T* __restrict__ row_terms, T* __restrict__ dx, int32_t* bad_label) {
  const int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t i = warp; i < B; i += nwarps) {
    const T* xr = x + i * C;
    int32_t y = labels[i];
    bool bad = y < 0 || y >= C;
    if (bad && lane == 0 && bad_label) *bad_label = 1;
    T v[R > 0 ? R : 1];
    if (R > 0) {
#pragma unroll
      for (int k = 0; k < R; k++) {
        const int64_t j = lane + 32 * k;
        v[k] = j < C ? xr[j] : (T)0;
      }
    }
    T m = (T)(-INFINITY);
    if (R > 0) {
#pragma unroll
      for (int k = 0; k < R; k++)
        if (lane + 32 * k < C) m = go_max(m, v[k]);
    } else {
      for (int64_t j = lane; j < C; j += 32) m = go_max(m, xr[j]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = go_max(m, __shfl_xor_sync(0xffffffffu, m, off));
    T S = (T)0;
    if (R > 0) {
#pragma unroll
      for (int k = 0; k < R; k++)
        if (lane + 32 * k < C) S = add_rn(S, (T)exp((double)sub_rn(v[k], m)));
    } else {
      for (int64_t j = lane; j < C; j += 32) S = add_rn(S, (T)exp((double)sub_rn(xr[j], m)));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) S = add_rn(S, __shfl_xor_sync(0xffffffffu, S, off));
    T Lse = (T)log((double)S);
    // Pick multiplies every log-probability by the one-hot row and sums: a
    // non-finite log-probability off the label turns into NaN (inf * 0).
    bool nonfinite = false;
    T picked = (T)0;
    T q = div_rn(c, S);
    auto visit = [&](int64_t j, T xj) {
      T sj = sub_rn(xj, m);
      T lp = sub_rn(sj, Lse);
      if (j == y) {
        picked = lp;
      } else if (!isfinite(lp)) {
        nonfinite = true;
      }
      if (dx) {
        T e = (T)exp((double)sj);
        T g = mul_rn(q, e);
        dx[i * C + j] = j == y ? add_rn(-c, g) : g;
      }
    };
    if (R > 0) {
#pragma unroll
      for (int k = 0; k < R; k++)
        if (lane + 32 * k < C) visit(lane + 32 * k, v[k]);
    } else {
      for (int64_t j = lane; j < C; j += 32) visit(j, xr[j]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      picked = add_rn(picked, __shfl_xor_sync(0xffffffffu, picked, off));
      nonfinite |= __shfl_xor_sync(0xffffffffu, (int)nonfinite, off) != 0;
    }
    if (lane == 0) row_terms[i] = (nonfinite || bad) ? (T)NAN : picked;
  }
}

// Launches the row kernel with the smallest register row that holds C.
template <typename T>
static void launch_rows(gt_ctx* ctx, const T* x, const int32_t* labels, int64_t B, int64_t C, T c, T* terms, T* dx,
                        int32_t* bad) {
  const int grid = grid_for(ctx, B * 32, 256);
  const int max_r = sizeof(T) == 8 ? 16 : 32;
#define GT_XENT_ROWS(RR) \
  xent_rows_kernel<T, RR><<<grid, 256, 0, ctx->stream>>>(x, labels, B, C, c, terms, dx, bad)
  if (C <= 32 && max_r >= 1) {
    GT_XENT_ROWS(1);
  } else if (C <= 64) {
    GT_XENT_ROWS(2);
  } else if (C <= 128) {
    GT_XENT_ROWS(4);
  } else if (C <= 256) {
    GT_XENT_ROWS(8);
  } else if (C <= 512) {
    GT_XENT_ROWS(16);
  } else if (C <= 1024 && max_r >= 32) {
    if constexpr (sizeof(T) == 4) GT_XENT_ROWS(32);
  } else {
    GT_XENT_ROWS(0);
  }
#undef GT_XENT_ROWS
}

// loss = -(sum_i row_terms[i] * c), one block, fixed reduction order.
template <typename T>
__global__ void xent_sum_kernel(const T* __restrict__ row_terms, int64_t B, T c, T* __restrict__ loss) {
  __shared__ T part[1024];
  T acc = (T)0;
  for (int64_t i = threadIdx.x; i < B; i += blockDim.x) acc = add_rn(acc, row_terms[i]);
  part[threadIdx.x] = acc;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) part[threadIdx.x] = add_rn(part[threadIdx.x], part[threadIdx.x + s]);
    __syncthreads();
  }
  if (threadIdx.x == 0) *loss = -mul_rn(part[0], c);
}

}  // namespace gt

// Row terms of gt_xent_fwd_bwd_noalloc: a buffer compiled into the library
// (one per device), so that variant never asks the pool for memory. Each call
// writes every row term it later reads, so leftovers from an earlier call,
// larger or smaller, never leak into a result and nothing needs clearing.
static __device__ __align__(256) unsigned char g_xent_rows[GT_XENT_NOALLOC_MAX_ROWS * sizeof(double)];

namespace gt {

// Device address of g_xent_rows per device. Host code cannot pass the
// symbol itself to a kernel (on the host it names a host-side stand-in), so
// the address is looked up once per device, with that device current.
static void* g_xent_rows_addr[64];
static std::mutex g_xent_rows_mu;

static char* xent_rows_buffer(gt_ctx* ctx, void** out) {
  if (ctx->device < 0 || ctx->device >= 64) return errorf("gt_xent_fwd_bwd_noalloc: device %d out of range", ctx->device);
  std::lock_guard<std::mutex> lock(g_xent_rows_mu);
  if (!g_xent_rows_addr[ctx->device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_xent_rows);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_xent_rows)", __FILE__, __LINE__);
    g_xent_rows_addr[ctx->device] = p;
  }
  *out = g_xent_rows_addr[ctx->device];
  return nullptr;
}

}  // namespace gt

using namespace gt;

extern "C" char* gt_xent_fwd_bwd_noalloc(gt_ctx* ctx, int dtype, const void* logits, const int32_t* labels, int64_t B,
                                         int64_t C, void* loss, void* dlogits, int32_t* bad_label) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (B <= 0 || C <= 0) return errorf("gt_xent_fwd_bwd_noalloc: B and C must be positive");
  if (B > GT_XENT_NOALLOC_MAX_ROWS)
    return errorf("gt_xent_fwd_bwd_noalloc: batch of %lld rows exceeds the %d-row buffer; use gt_xent_fwd_bwd",
                  (long long)B, GT_XENT_NOALLOC_MAX_ROWS);
  void* terms = nullptr;
  GT_TRY(xent_rows_buffer(ctx, &terms));
  GT_DISPATCH(dtype, {
    T c = (T)(1.0 / (double)B);
    launch_rows<T>(ctx, (const T*)logits, labels, B, C, c, (T*)terms, (T*)dlogits, bad_label);
    xent_sum_kernel<T><<<1, 1024, 0, ctx->stream>>>((const T*)terms, B, c, (T*)loss);
  });
  count_launch(2);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "xent launch", __FILE__, __LINE__);
  return nullptr;
}

extern "C" char* gt_xent_fwd_bwd(gt_ctx* ctx, int dtype, const void* logits, const int32_t* labels, int64_t B,
                                 int64_t C, void* loss, void* dlogits, int32_t* bad_label) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (B <= 0 || C <= 0) return errorf("gt_xent_fwd_bwd: B and C must be positive");
  size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  void* terms = nullptr;
  GT_TRY(scratch(ctx, B * es, &terms));
  GT_DISPATCH(dtype, {
    T c = (T)(1.0 / (double)B);  // MulScalar(1/float64(N)) rounds the scalar to T
    launch_rows<T>(ctx, (const T*)logits, labels, B, C, c, (T*)terms, (T*)dlogits, bad_label);
    xent_sum_kernel<T><<<1, 1024, 0, ctx->stream>>>((const T*)terms, B, c, (T*)loss);
  });
  count_launch(2);
  cudaError_t e = cudaGetLastError();
  release(ctx, terms);
  if (e != cudaSuccess) return cuda_error(e, "xent launch", __FILE__, __LINE__);
  return nullptr;
}
