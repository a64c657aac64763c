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
  // pos_major (with nchw_L > 0) swaps the roles in the NCHW store: m is the
  // position (image m / L, offset m % L) and n the channel, nchw_M channels:
  // out[((m / L) * nchw_M + n) * L + m % L] (an implicit-GEMM convolution,
  // positions on M).
  bool pos_major = false;
  // col_major stores C transposed, out[n * ldc + m]; row rowsum_m of C goes to
  // rowsum_out[n] instead (a weight gradient whose extra row of ones in A
  // makes that row the bias gradient).
  bool col_major = false;
  T* rowsum_out = nullptr;
  int64_t rowsum_m = -1;
  // Column partial sums of the stored values (tcgen05 plain, mask and bit-mask
  // epilogues): colsum_ws[(m / 32) * ldcs + n] = sum over the 32-row block
  // of C(m, n), rows in order; a second kernel adds the blocks. With dX of a
  // Linear as C, the column sums are the bias gradient of the layer before.
  T* colsum_ws = nullptr;
  int64_t ldcs = 0;
  // With pos_major: 2 x 2 / stride-2 max pooling after the bias and
  // activation (tcgen05 implicit convolution only). out receives the pooled
  // (images, nchw_M, OH / 2, OW / 2) values and pool_idx the offset (kh * 2 +
  // kw) of each window's first maximum; the convolution output itself is not
  // stored.
  uint8_t* pool_idx = nullptr;

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

  // Writes the finished value of C(m, n) (row-major, transposed or an NCHW order).
  __device__ __forceinline__ void put(int64_t m, int64_t n, T v) const {
    if (col_major) {
      if (m == rowsum_m) {
        if (rowsum_out) rowsum_out[n] = v;
      } else {
        out[n * ldc + m] = v;
      }
    } else if (nchw_L > 0 && pos_major) {
      int64_t img = m / nchw_L;
      out[(img * nchw_M + n) * nchw_L + (m - img * nchw_L)] = v;
    } else if (nchw_L > 0) {
      int64_t img = n / nchw_L;
      out[(img * nchw_M + m) * nchw_L + (n - img * nchw_L)] = v;
    } else {
      out[m * ldc + n] = v;
    }
  }
};

// Rounds to the nearest tf32 value (ties away from zero) on the integer ALU:
// add half a tf32 ulp to the magnitude bits, clear the 13 dropped bits. The
// 3xTF32 operands are x = hi + lo with hi = tf32(x), lo = tf32(x - hi).
// Infinities stay infinities; a NaN stays NaN or becomes an infinity whose lo
// part is NaN, so a product with it is NaN either way.
__device__ __forceinline__ float tf32_round(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// Output-channel tile width of an implicit-GEMM convolution with `cols`
// output channels (the narrowest of 64, 128, 256 that holds them), and the
// row count its pre-split weight planes are padded to.
inline int64_t conv_tile_width(int64_t cols) { return cols <= 64 ? 64 : cols <= 128 ? 128 : 256; }
inline int64_t conv_weight_rows(int64_t cols) {
  const int64_t t = conv_tile_width(cols);
  return (cols + t - 1) / t * t;
}

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

// Implicit-GEMM convolutions on the tcgen05 path (float32), with no im2col
// columns in memory. Both return nullptr with *done = false when the geometry
// does not qualify (the caller then uses the explicit path).
//   conv_fwd_tc: y (N, O, OH, OW) = act(conv2d(x, w) + bias) (stride 1); the
//     weight comes pre-split into tf32 planes: ws rows [0, O) = tf32(w) and
//     rows [wrows, wrows + O) = tf32(w - tf32(w)), wrows =
//     conv_weight_rows(O), every row of w_pitch elements (a multiple of 4,
//     16-byte aligned base), padding rows and columns zero; act is none or
//     ReLU.
//   conv_wgrad_tc: dw (O, C*KH*KW) and db (O, or NULL) from x and dy
//     (N, O, OH, OW); needs OH * OW % 16 == 0.
//   With pool_idx, conv_fwd_tc also applies 2 x 2 / stride-2 max pooling
//     (MaxPool2d(2) after the convolution and its activation): y receives the
//     pooled (N, O, OH / 2, OW / 2) values and pool_idx each window's
//     first-max offset; needs even OH and OW.
char* conv_fwd_tc(gt_ctx* ctx, const float* x, const float* ws, int64_t w_pitch, const float* bias, float* y,
                  const gt_geom& g, int64_t O, int act, bool* done, uint8_t* pool_idx = nullptr);
char* conv_wgrad_tc(gt_ctx* ctx, const float* x, const float* dy, float* dw, float* db, const gt_geom& g, int64_t O,
                    bool* done);

// The same through the GEMM launch timer (gemm.cu); the conv entry points call these.
char* conv_fwd_gemm(gt_ctx* ctx, const float* x, const float* w, int64_t w_pitch, const float* bias, float* y,
                    const gt_geom& g, int64_t O, int act, bool* done, uint8_t* pool_idx = nullptr);
char* conv_wgrad_gemm(gt_ctx* ctx, const float* x, const float* dy, float* dw, float* db, const gt_geom& g,
                      int64_t O, bool* done);

// Runs run(arg) between the GEMM launch timer's events, recorded as an
// M x N x K GEMM on `path`: kernels that compute a GEMM's result another way
// (5: the fused pool-backward weight gradient, 7: the direct first-conv +
// ReLU + pool forward, conv.cu).
char* timed_gemm_like(gt_ctx* ctx, int64_t M, int64_t N, int64_t K, int path, char* (*run)(void*), void* arg);

// Whether a float32 GEMM with this epilogue, if it runs on the tcgen05 path,
// writes its column partial sums (Epi::colsum_ws).
bool tc_writes_colsums(const Epi<float>& epi, int64_t n_cols);

// Thin GEMMs (gemm_simt.cu): N <= 32 with B transposed (a classifier's
// forward), or M <= 32 with A transposed and a plain epilogue (its weight
// gradient). *done = false when the shape does not qualify.
template <typename T>
char* gemm_thin(gt_ctx* ctx, const GemmShape& s, const T* A, const T* B, const Epi<T>& epi, bool* done);

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
