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
#include <algorithm>

#include "gt_common.cuh"

namespace gt {

template <typename T>
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
    T m = (T)(-INFINITY);
    for (int64_t j = lane; j < C; j += 32) m = go_max(m, xr[j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = go_max(m, __shfl_xor_sync(0xffffffffu, m, off));
    T S = (T)0;
    for (int64_t j = lane; j < C; j += 32) S = add_rn(S, (T)exp((double)sub_rn(xr[j], m)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) S = add_rn(S, __shfl_xor_sync(0xffffffffu, S, off));
    T Lse = (T)log((double)S);
    // Pick multiplies every log-probability by the one-hot row and sums: a
    // non-finite log-probability off the label turns into NaN (inf * 0).
    bool nonfinite = false;
    T picked = (T)0;
    T q = div_rn(c, S);
    for (int64_t j = lane; j < C; j += 32) {
      T s = sub_rn(xr[j], m);
      T lp = sub_rn(s, Lse);
      if (j == y) {
        picked = lp;
      } else if (!isfinite(lp)) {
        nonfinite = true;
      }
      if (dx) {
        T e = (T)exp((double)s);
        T g = mul_rn(q, e);
        dx[i * C + j] = j == y ? add_rn(-c, g) : g;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      picked = add_rn(picked, __shfl_xor_sync(0xffffffffu, picked, off));
      nonfinite |= __shfl_xor_sync(0xffffffffu, (int)nonfinite, off) != 0;
    }
    if (lane == 0) row_terms[i] = (nonfinite || bad) ? (T)NAN : picked;
  }
}

// The same for rows of at most 32 * NPL classes, with one float64 exp per
// element: lane l holds elements l, l + 32, ... of its row in registers (NPL
// values, a compile-time count so the array never leaves registers), loaded
// once. e = T(exp(double(x - m))) replaces x in place, is summed, and gives
// the gradient q * e from the same rounded value the streaming kernel
// recomputes, so both kernels produce identical bits. A log-probability
// x_j - m - L is non-finite exactly when x_j - m or L is (x - m <= 0 and
// 0 <= L <= log C), so the Pick's NaN rule needs no third pass either.
//
// With COLS (and dx), each lane also sums the gradient values it writes, per
// column, over the rows of its warp; the block's warps add theirs in warp
// order and write one partial row per block to col_part (gridDim.x x C), which
// xent_cols_kernel sums over the blocks: the column sums of dlogits, the bias
// gradient of the Linear that produced the logits, without a second pass
// over dlogits.
template <typename T, int NPL, bool COLS = false>
__global__ void xent_rows_reg_kernel(const T* __restrict__ x, const int32_t* __restrict__ labels, int64_t B, int C,
                                     T c, T* __restrict__ row_terms, T* __restrict__ dx, int32_t* bad_label,
                                     T* __restrict__ col_part = nullptr) {
  const int lane = threadIdx.x & 31;
  T cs[COLS ? NPL : 1];
#pragma unroll
  for (int t = 0; t < (COLS ? NPL : 1); t++) cs[t] = (T)0;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t i = warp; i < B; i += nwarps) {
    const T* xr = x + i * C;
    const int32_t y = labels[i];
    const bool bad = y < 0 || y >= C;
    if (bad && lane == 0 && bad_label) *bad_label = 1;
    T v[NPL];
#pragma unroll
    for (int t = 0; t < NPL; t++) {
      const int j = lane + 32 * t;
      v[t] = j < C ? __ldg(xr + j) : (T)(-INFINITY);
    }
    T m = (T)(-INFINITY);
#pragma unroll
    for (int t = 0; t < NPL; t++)
      if (lane + 32 * t < C) m = go_max(m, v[t]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = go_max(m, __shfl_xor_sync(0xffffffffu, m, off));
    T S = (T)0, s_y = (T)0;
    bool nonfinite = false;
#pragma unroll
    for (int t = 0; t < NPL; t++) {
      const int j = lane + 32 * t;
      if (j < C) {
        const T s = sub_rn(v[t], m);
        if (j == y) s_y = s;
        else if (!isfinite(s)) nonfinite = true;
        v[t] = (T)exp((double)s);
        S = add_rn(S, v[t]);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) S = add_rn(S, __shfl_xor_sync(0xffffffffu, S, off));
    const T Lse = (T)log((double)S);
    if (dx) {
      const T q = div_rn(c, S);
      T* dr = dx + i * C;
#pragma unroll
      for (int t = 0; t < NPL; t++) {
        const int j = lane + 32 * t;
        if (j < C) {
          const T g = mul_rn(q, v[t]);
          const T d = j == y ? add_rn(-c, g) : g;
          dr[j] = d;
          if constexpr (COLS) cs[t] = add_rn(cs[t], d);
        }
      }
    }
    // picked: the label's log-probability, summed over the warp like the
    // streaming kernel's picked terms (one lane non-zero)
    T picked = (lane == (y & 31) && !bad) ? sub_rn(s_y, Lse) : (T)0;
    if (!isfinite(Lse) && C > 1) nonfinite = true;  // every off-label log-probability is non-finite
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      picked = add_rn(picked, __shfl_xor_sync(0xffffffffu, picked, off));
      nonfinite |= __shfl_xor_sync(0xffffffffu, (int)nonfinite, off) != 0;
    }
    if (lane == 0) row_terms[i] = (nonfinite || bad) ? (T)NAN : picked;
  }
  if constexpr (COLS) {
    extern __shared__ unsigned char xent_smem[];
    T* part = reinterpret_cast<T*>(xent_smem);  // [warps][C]
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int t = 0; t < NPL; t++)
      if (lane + 32 * t < C) part[w * C + lane + 32 * t] = cs[t];
    __syncthreads();
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
      T acc = part[j];
      for (int k = 1; k < nw; k++) acc = add_rn(acc, part[k * C + j]);
      col_part[(int64_t)blockIdx.x * C + j] = acc;
    }
  }
}

// db[j] = sum over the blocks of col_part[b][j], in block order.
template <typename T>
__global__ void xent_cols_kernel(const T* __restrict__ col_part, int blocks, int C, T* __restrict__ db) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < C; j += gridDim.x * blockDim.x) {
    T acc = col_part[j];
    for (int b = 1; b < blocks; b++) acc = add_rn(acc, col_part[(int64_t)b * C + j]);
    db[j] = acc;
  }
}

// The row kernel with column sums for rows of at most 1024 classes (a block
// of 4 warps, at most 2 blocks per SM so that the partial rows stay few);
// returns false for wider rows.
template <typename T>
static bool xent_rows_cols_launch(gt_ctx* ctx, const T* x, const int32_t* labels, int64_t B, int64_t C, T c,
                                  T* terms, T* dx, int32_t* bad, T* col_part, int grid) {
  const size_t sm = 4 * (size_t)C * sizeof(T);
  if (C <= 32)
    xent_rows_reg_kernel<T, 1, true><<<grid, 128, sm, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad, col_part);
  else if (C <= 128)
    xent_rows_reg_kernel<T, 4, true><<<grid, 128, sm, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad, col_part);
  else if (C <= 512)
    xent_rows_reg_kernel<T, 16, true><<<grid, 128, sm, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad,
                                                                       col_part);
  else if (C <= 1024)
    xent_rows_reg_kernel<T, 32, true><<<grid, 128, sm, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad,
                                                                       col_part);
  else
    return false;
  return true;
}

// Launches the row kernel that fits C: register rows up to 1024 classes,
// else the streaming kernel.
template <typename T>
static void xent_rows_launch(gt_ctx* ctx, const T* x, const int32_t* labels, int64_t B, int64_t C, T c, T* terms,
                             T* dx, int32_t* bad) {
  const int grid = grid_for(ctx, B * 32, 256);
  if (C <= 32)
    xent_rows_reg_kernel<T, 1><<<grid, 256, 0, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad);
  else if (C <= 128)
    xent_rows_reg_kernel<T, 4><<<grid, 256, 0, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad);
  else if (C <= 512)
    xent_rows_reg_kernel<T, 16><<<grid, 256, 0, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad);
  else if (C <= 1024)
    xent_rows_reg_kernel<T, 32><<<grid, 256, 0, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad);
  else
    xent_rows_kernel<T><<<grid, 256, 0, ctx->stream>>>(x, labels, B, C, c, terms, dx, bad);
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
    xent_rows_launch<T>(ctx, (const T*)logits, labels, B, C, c, (T*)terms, (T*)dlogits, bad_label);
    xent_sum_kernel<T><<<1, 1024, 0, ctx->stream>>>((const T*)terms, B, c, (T*)loss);
  });
  count_launch(2);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "xent launch", __FILE__, __LINE__);
  return nullptr;
}

extern "C" char* gt_xent_fwd_bwd_db(gt_ctx* ctx, int dtype, const void* logits, const int32_t* labels, int64_t B,
                                    int64_t C, void* loss, void* dlogits, void* db, int32_t* bad_label) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (B <= 0 || C <= 0) return errorf("gt_xent_fwd_bwd_db: B and C must be positive");
  if (!dlogits || !db) return errorf("gt_xent_fwd_bwd_db: dlogits and db must not be NULL");
  if (C > 1024) {  // rows too wide for the register kernel: the gradient, then its column sums
    GT_TRY(gt_xent_fwd_bwd(ctx, dtype, logits, labels, B, C, loss, dlogits, bad_label));
    return gt_reduce(ctx, dtype, GT_SUM, dlogits, db, 1, B, C);
  }
  const size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  const int grid = (int)std::min<int64_t>(ceil_div(B, 4), 2 * (int64_t)ctx->sm_count);
  void *terms = nullptr, *part = nullptr;
  GT_TRY(scratch(ctx, B * es, &terms));
  char* err = scratch(ctx, (size_t)grid * C * es, &part);
  if (!err) {
    GT_DISPATCH(dtype, {
      T c = (T)(1.0 / (double)B);
      xent_rows_cols_launch<T>(ctx, (const T*)logits, labels, B, C, c, (T*)terms, (T*)dlogits, bad_label, (T*)part,
                               grid);
      xent_sum_kernel<T><<<1, 1024, 0, ctx->stream>>>((const T*)terms, B, c, (T*)loss);
      xent_cols_kernel<T><<<grid_for(ctx, C, 256), 256, 0, ctx->stream>>>((const T*)part, grid, (int)C, (T*)db);
    });
    count_launch(3);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) err = cuda_error(e, "xent launch", __FILE__, __LINE__);
  }
  release(ctx, terms);
  release(ctx, part);
  return err;
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
    xent_rows_launch<T>(ctx, (const T*)logits, labels, B, C, c, (T*)terms, (T*)dlogits, bad_label);
    xent_sum_kernel<T><<<1, 1024, 0, ctx->stream>>>((const T*)terms, B, c, (T*)loss);
  });
  count_launch(2);
  cudaError_t e = cudaGetLastError();
  release(ctx, terms);
  if (e != cudaSuccess) return cuda_error(e, "xent launch", __FILE__, __LINE__);
  return nullptr;
}
