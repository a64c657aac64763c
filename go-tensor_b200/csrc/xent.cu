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
// column_sums_kernel adds over the blocks: the column sums of dlogits, the bias
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

// Rows of 129 to 128 * VPT classes: a block of 128 threads per row (rows
// blockIdx.x, + gridDim.x, ...), thread t holding elements t, t + 128, ...:
// more rows in flight than a warp per row with 32 values in registers. One
// float64 exp per element as above; the sum adds each thread's values in
// order, then the warp butterfly, then the four warps in order. With COLS
// each thread also sums, per column, the gradient values of its block's rows
// and writes them as the block's partial row of col_part.
template <typename T, int VPT, bool COLS>
__global__ void __launch_bounds__(128) xent_rows_blk_kernel(const T* __restrict__ x, const int32_t* __restrict__ labels,
                                                            int64_t B, int C, T c, T* __restrict__ row_terms,
                                                            T* __restrict__ dx, int32_t* bad_label,
                                                            T* __restrict__ col_part) {
  __shared__ T red[4];
  __shared__ T pick;
  __shared__ int nonfin;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  T cs[COLS ? VPT : 1];
#pragma unroll
  for (int u = 0; u < (COLS ? VPT : 1); u++) cs[u] = (T)0;
  // the next row's values are loaded while this row is computed
  T nv[VPT];
  if (blockIdx.x < B) {
#pragma unroll
    for (int u = 0; u < VPT; u++) {
      const int j = tid + 128 * u;
      nv[u] = j < C ? __ldg(x + (int64_t)blockIdx.x * C + j) : (T)(-INFINITY);
    }
  }
  for (int64_t i = blockIdx.x; i < B; i += gridDim.x) {
    const int32_t y = labels[i];
    const bool bad = y < 0 || y >= C;
    if (bad && tid == 0 && bad_label) *bad_label = 1;
    T v[VPT];
#pragma unroll
    for (int u = 0; u < VPT; u++) v[u] = nv[u];
    if (i + gridDim.x < B) {
#pragma unroll
      for (int u = 0; u < VPT; u++) {
        const int j = tid + 128 * u;
        nv[u] = j < C ? __ldg(x + (i + gridDim.x) * C + j) : (T)(-INFINITY);
      }
    }
    T m = (T)(-INFINITY);
#pragma unroll
    for (int u = 0; u < VPT; u++)
      if (tid + 128 * u < C) m = go_max(m, v[u]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = go_max(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) red[w] = m;
    if (tid == 0) nonfin = 0, pick = (T)0;
    __syncthreads();
    m = go_max(go_max(red[0], red[1]), go_max(red[2], red[3]));
    __syncthreads();  // red is reused below
    T S = (T)0;
    bool nf = false;
#pragma unroll
    for (int u = 0; u < VPT; u++) {
      const int j = tid + 128 * u;
      if (j < C) {
        const T sv = sub_rn(v[u], m);
        if (j == y) pick = sv;  // the label's shifted logit (one thread)
        else if (!isfinite(sv)) nf = true;
        v[u] = (T)exp((double)sv);
        S = add_rn(S, v[u]);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) S = add_rn(S, __shfl_xor_sync(0xffffffffu, S, off));
    if (lane == 0) red[w] = S;
    if (__any_sync(0xffffffffu, nf) && lane == 0) nonfin = 1;
    __syncthreads();
    S = add_rn(add_rn(add_rn(red[0], red[1]), red[2]), red[3]);
    const T Lse = (T)log((double)S);
    const T q = div_rn(c, S);
    if (dx) {
      T* dr = dx + i * C;
#pragma unroll
      for (int u = 0; u < VPT; u++) {
        const int j = tid + 128 * u;
        if (j < C) {
          const T g = mul_rn(q, v[u]);
          const T d = j == y ? add_rn(-c, g) : g;
          dr[j] = d;
          if constexpr (COLS) cs[u] = add_rn(cs[u], d);
        }
      }
    }
    if (tid == 0) {
      const bool nonfinite = nonfin || (!isfinite(Lse) && C > 1);
      row_terms[i] = (nonfinite || bad) ? (T)NAN : add_rn(sub_rn(pick, Lse), (T)0);
    }
    __syncthreads();  // red, pick and nonfin are rewritten by the next row
  }
  if constexpr (COLS) {
#pragma unroll
    for (int u = 0; u < VPT; u++) {
      const int j = tid + 128 * u;
      if (j < C) col_part[(int64_t)blockIdx.x * C + j] = cs[u];
    }
  }
}

// The row kernel with column sums for rows of at most 1024 classes (a block
// of 4 warps, at most 8 blocks per SM: one partial row per block, which
// column_sums_kernel adds); returns false for wider rows.
template <typename T>
static bool xent_rows_cols_launch(gt_ctx* ctx, const T* x, const int32_t* labels, int64_t B, int64_t C, T c,
                                  T* terms, T* dx, int32_t* bad, T* col_part, int grid) {
  const size_t sm = 4 * (size_t)C * sizeof(T);
  if (C <= 32)
    xent_rows_reg_kernel<T, 1, true><<<grid, 128, sm, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad, col_part);
  else if (C <= 128)
    xent_rows_reg_kernel<T, 4, true><<<grid, 128, sm, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad, col_part);
  else if (C <= 512)
    xent_rows_blk_kernel<T, 4, true><<<grid, 128, 0, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad, col_part);
  else if (C <= 1024)
    xent_rows_blk_kernel<T, 8, true><<<grid, 128, 0, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad, col_part);
  else
    return false;
  return true;
}

// Blocks for the block-per-row kernel: up to 16 per SM, the rows loop over them.
static int xent_blk_grid(const gt_ctx* ctx, int64_t B) {
  return (int)std::min<int64_t>(B, 16 * (int64_t)ctx->sm_count);
}

// Launches the row kernel that fits C: a warp per row up to 128 classes, a
// block per row up to 1024, else the streaming kernel.
template <typename T>
static void xent_rows_launch(gt_ctx* ctx, const T* x, const int32_t* labels, int64_t B, int64_t C, T c, T* terms,
                             T* dx, int32_t* bad) {
  const int grid = grid_for(ctx, B * 32, 256);
  if (C <= 32)
    xent_rows_reg_kernel<T, 1><<<grid, 256, 0, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad);
  else if (C <= 128)
    xent_rows_reg_kernel<T, 4><<<grid, 256, 0, ctx->stream>>>(x, labels, B, (int)C, c, terms, dx, bad);
  else if (C <= 512)
    xent_rows_blk_kernel<T, 4, false><<<xent_blk_grid(ctx, B), 128, 0, ctx->stream>>>(x, labels, B, (int)C, c, terms,
                                                                                      dx, bad, nullptr);
  else if (C <= 1024)
    xent_rows_blk_kernel<T, 8, false><<<xent_blk_grid(ctx, B), 128, 0, ctx->stream>>>(x, labels, B, (int)C, c, terms,
                                                                                      dx, bad, nullptr);
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
  const int grid = C <= 128 ? (int)std::min<int64_t>(ceil_div(B, 4), 8 * (int64_t)ctx->sm_count)
                            : xent_blk_grid(ctx, B);
  void *terms = nullptr, *part = nullptr;
  GT_TRY(scratch(ctx, B * es, &terms));
  char* err = scratch(ctx, (size_t)grid * C * es, &part);
  if (!err) {
    GT_DISPATCH(dtype, {
      T c = (T)(1.0 / (double)B);
      xent_rows_cols_launch<T>(ctx, (const T*)logits, labels, B, C, c, (T*)terms, (T*)dlogits, bad_label, (T*)part,
                               grid);
      xent_sum_kernel<T><<<1, 1024, 0, ctx->stream>>>((const T*)terms, B, c, (T*)loss);
      column_sums_kernel<T><<<(unsigned)ceil_div(C, 32), 1024, 0, ctx->stream>>>((const T*)part, grid, C, (T*)db);
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
