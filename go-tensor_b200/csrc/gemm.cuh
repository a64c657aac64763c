// Internal GEMM interface shared by the matmul, linear and conv entry points.
//
//   C[m, n] = epilogue( sum_k A(m, k) * B(k, n) )
//   A(m, k) = trans_a ? A[k * lda + m] : A[m * lda + k]
//   B(k, n) = trans_b ? B[n * ldb + k] : B[k * ldb + n]
//
// The epilogue rounds the fp32/fp64 accumulator to T and then applies, in the
// reference's order: + bias[n] (rounded), the forward activation, or the
// backward factor act'(dmask[m, n]); finally it stores to out[m * ldc + n].
#pragma once
#include "gt_common.cuh"

namespace gt {

template <typename T>
struct Epi {
  T* out = nullptr;
  int64_t ldc = 0;
  const T* bias = nullptr;   // added before act: bias[n], or bias[m] if bias_by_row
  bool bias_by_row = false;
  int act = GT_ACT_NONE;     // forward activation
  const T* dmask = nullptr;  // out = act_bwd(dact, acc, dmask[m * ldm + n])
  int dact = GT_ACT_NONE;
  int64_t ldm = 0;
  // nchw_L > 0 stores C (M = channels, N = images * L) into an (images, M, L)
  // tensor: out[(n / L) * M * L + m * L + n % L], with M given in nchw_M.
  int64_t nchw_L = 0, nchw_M = 0;
  // ReLU bit masks in column words: bit m % 32 of bits[(m / 32) * ldw + n],
  // ldw = the number of columns, so a thread that owns column n of 32 rows
  // reads or writes one word, and a warp's 32 columns are 128 contiguous
  // bytes. bits_out (forward): bit = (stored value > 0), written by
  // the tcgen05 epilogues only (other paths leave it to gt_relu_bits). dbits
  // (dX): out = acc * (bit ? 1 : 0), ReLU's derivative g * Step(y) read from
  // the forward's bits instead of the activation itself.
  uint32_t* bits_out = nullptr;
  const uint32_t* dbits = nullptr;
  int64_t ldw = 0;

  // The finished value of C(m, n): bias, activation, activation derivative.
  __device__ __forceinline__ T finish(int64_t m, int64_t n, T acc) const {
    T v = acc;
    if (bias) v = add_rn(v, bias[bias_by_row ? m : n]);
    if (act != GT_ACT_NONE) v = act_fwd(act, v);
    if (dmask) v = act_bwd(dact, v, dmask[m * ldm + n]);
    if (dbits) v = mul_rn(v, ((dbits[(m >> 5) * ldw + n] >> (m & 31)) & 1u) ? (T)1 : (T)0);
    return v;
  }

  __device__ __forceinline__ void store(int64_t m, int64_t n, T acc) const { put(m, n, finish(m, n, acc)); }

  // Writes the finished value of C(m, n) (row-major or the NCHW order).
  __device__ __forceinline__ void put(int64_t m, int64_t n, T v) const {
    if (nchw_L > 0) {
      int64_t img = n / nchw_L;
      out[(img * nchw_M + m) * nchw_L + (n - img * nchw_L)] = v;
    } else {
      out[m * ldc + n] = v;
    }
  }
};

struct GemmShape {
  int64_t M, N, K;
  bool trans_a, trans_b;
  int64_t lda, ldb;
};

// SIMT path (FFMA/DFMA). Any shape, any alignment.
template <typename T>
char* gemm_simt(gt_ctx* ctx, const GemmShape& s, const T* A, const T* B, const Epi<T>& epi);

// tcgen05 3xTF32 path for float32. Returns nullptr and sets *done = false
// when the shape or alignment does not qualify (the caller falls back).
char* gemm_tc_f32(gt_ctx* ctx, const GemmShape& s, const float* A, const float* B, const Epi<float>& epi,
                  bool* done);

// Dispatches to the fastest qualifying path.
template <typename T>
char* gemm(gt_ctx* ctx, const GemmShape& s, const T* A, const T* B, const Epi<T>& epi);

// Test hook: 0 = automatic, 1 = force SIMT, 2 = require tcgen05 (error if the
// shape does not qualify).
void set_gemm_path(int path);
int gemm_path();
void set_gemm_splits(int splits);  // tcgen05 path: 0 = automatic, else this many K-splits
void set_tc_wait_limit_us(int64_t us);  // tcgen05 barrier-wait limit (0: the default 2 s)
void tc_withhold_next_arrive();         // the next tcgen05 GEMM's first slice never reaches its MMA

}  // namespace gt
