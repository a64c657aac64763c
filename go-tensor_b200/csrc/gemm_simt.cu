// SIMT GEMM: the FP64 path (DFMA; tcgen05 has no f64 kind) and the float32
// path for shapes the tensor-core kernel does not take (tiny or unaligned
// operands, such as the K = 9 or 27 convolutions and N = 10 classifiers).
//
// Classic register-blocked tiling: a CTA computes a BM x BN tile, staging
// BK-deep slices of A and B in shared memory (k-major, so the inner product
// reads contiguous rows); each thread accumulates a TM x TN block in
// registers with FMA in the dtype. Loads are coalesced along whichever of
// (m, k) / (k, n) is contiguous for the transpose flags.
#include "gemm.cuh"

namespace gt {

template <typename T, int BM, int BN, int BK, int TM, int TN>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    gemm_simt_kernel(GemmShape s, const T* __restrict__ A, const T* __restrict__ B, Epi<T> epi) {
  constexpr int NT = (BM / TM) * (BN / TN);
  __shared__ T As[BK][BM];
  __shared__ T Bs[BK][BN];
  const int tid = threadIdx.x;
  const int tx = tid % (BN / TN), ty = tid / (BN / TN);
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int64_t M = s.M, N = s.N, K = s.K;

  T acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = (T)0;

  for (int64_t k0 = 0; k0 < K; k0 += BK) {
#pragma unroll 4
    for (int e = tid; e < BM * BK; e += NT) {
      int mm, kk;
      if (s.trans_a) {
        kk = e / BM;
        mm = e % BM;
      } else {
        mm = e / BK;
        kk = e % BK;
      }
      int64_t gm = m0 + mm, gk = k0 + kk;
      T v = (T)0;
      if (gm < M && gk < K) v = s.trans_a ? A[gk * s.lda + gm] : A[gm * s.lda + gk];
      As[kk][mm] = v;
    }
#pragma unroll 4
    for (int e = tid; e < BN * BK; e += NT) {
      int nn, kk;
      if (s.trans_b) {
        nn = e / BK;
        kk = e % BK;
      } else {
        kk = e / BN;
        nn = e % BN;
      }
      int64_t gn = n0 + nn, gk = k0 + kk;
      T v = (T)0;
      if (gn < N && gk < K) v = s.trans_b ? B[gn * s.ldb + gk] : B[gk * s.ldb + gn];
      Bs[kk][nn] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; kk++) {
      T a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; i++) a[i] = As[kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; j++) b[j] = Bs[kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = fma(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < TM; i++) {
    int64_t m = m0 + ty * TM + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; j++) {
      int64_t n = n0 + tx * TN + j;
      if (n < N) epi.store(m, n, acc[i][j]);
    }
  }
}

template <typename T>
char* gemm_simt(gt_ctx* ctx, const GemmShape& s, const T* A, const T* B, const Epi<T>& epi) {
  if (s.M <= 0 || s.N <= 0) return nullptr;
  if (sizeof(T) == 4) {
    constexpr int BM = 128, BN = 128, BK = 8, TM = 8, TN = 8;
    dim3 grid((unsigned)ceil_div(s.N, BN), (unsigned)ceil_div(s.M, BM));
    if (grid.y > 65535) return errorf("gemm_simt: M = %lld is too large", (long long)s.M);
    gemm_simt_kernel<T, BM, BN, BK, TM, TN><<<grid, (BM / TM) * (BN / TN), 0, ctx->stream>>>(s, A, B, epi);
  } else {
    constexpr int BM = 64, BN = 64, BK = 8, TM = 4, TN = 4;
    dim3 grid((unsigned)ceil_div(s.N, BN), (unsigned)ceil_div(s.M, BM));
    if (grid.y > 65535) return errorf("gemm_simt: M = %lld is too large", (long long)s.M);
    gemm_simt_kernel<T, BM, BN, BK, TM, TN><<<grid, (BM / TM) * (BN / TN), 0, ctx->stream>>>(s, A, B, epi);
  }
  GT_LAUNCH_CHECK();
  return nullptr;
}

template char* gemm_simt<float>(gt_ctx*, const GemmShape&, const float*, const float*, const Epi<float>&);
template char* gemm_simt<double>(gt_ctx*, const GemmShape&, const double*, const double*, const Epi<double>&);

}  // namespace gt
