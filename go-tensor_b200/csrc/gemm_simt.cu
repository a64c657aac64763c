// SIMT GEMM: the FP64 path (DFMA; tcgen05 has no f64 kind) and the float32
// path for shapes the tensor-core kernel does not take (tiny or unaligned
// operands, such as the K = 9 or 27 convolutions and N = 10 classifiers).
//
// K-split: when the output has too few tiles to occupy the SMs and K is long
// (the weight gradient of a convolution's first layer: 64 x 27 outputs over
// K = batch x pixels, a million), blockIdx.z takes a K range and writes its
// partial tile to a workspace; a second kernel adds the partials in split
// order and applies the epilogue, so the result does not depend on timing.
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
    gemm_simt_kernel(GemmShape s, const T* __restrict__ A, const T* __restrict__ B, Epi<T> epi, int64_t k_per_split,
                     T* __restrict__ ws) {
  constexpr int NT = (BM / TM) * (BN / TN);
  __shared__ T As[BK][BM];
  __shared__ T Bs[BK][BN];
  const int tid = threadIdx.x;
  const int tx = tid % (BN / TN), ty = tid / (BN / TN);
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int64_t M = s.M, N = s.N;
  const int64_t k_begin = (int64_t)blockIdx.z * k_per_split;
  const int64_t K = k_begin + k_per_split < s.K ? k_begin + k_per_split : s.K;  // this split's end

  T acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = (T)0;

  for (int64_t k0 = k_begin; k0 < K; k0 += BK) {
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
      if (n >= N) continue;
      if (ws)
        ws[((int64_t)blockIdx.z * M + m) * N + n] = acc[i][j];
      else
        epi.store(m, n, acc[i][j]);
    }
  }
}

// out(m, n) = epilogue(sum of the splits' partials in split order).
template <typename T>
__global__ void simt_split_reduce_kernel(const T* __restrict__ ws, int splits, int64_t M, int64_t N, Epi<T> epi) {
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    T acc = ws[i];
    for (int k = 1; k < splits; k++) acc = add_rn(acc, ws[k * total + i]);
    const int64_t m = i / N;
    epi.store(m, i - m * N, acc);
  }
}

// Splits for a launch of `blocks` output tiles: enough to give every SM two
// blocks, each split at least 128 deep in K, at most 1024 splits and a 256 MB
// workspace.
static int simt_splits(const gt_ctx* ctx, int64_t blocks, int64_t M, int64_t N, int64_t K, size_t es) {
  const int64_t want = 2 * (int64_t)ctx->sm_count;
  if (blocks >= want) return 1;
  int64_t S = ceil_div(want, blocks);
  S = S < K / 128 ? S : K / 128;
  S = S < 1024 ? S : 1024;
  while (S > 1 && (double)S * M * N * es > (double)(256u << 20)) S /= 2;
  return S > 1 ? (int)S : 1;
}

template <typename T, int BM, int BN, int BK, int TM, int TN>
static char* simt_launch(gt_ctx* ctx, const GemmShape& s, const T* A, const T* B, const Epi<T>& epi) {
  const int64_t gx = ceil_div(s.N, BN), gy = ceil_div(s.M, BM);
  if (gy > 65535) return errorf("gemm_simt: M = %lld is too large", (long long)s.M);
  const int splits = simt_splits(ctx, gx * gy, s.M, s.N, s.K, sizeof(T));
  auto kern = gemm_simt_kernel<T, BM, BN, BK, TM, TN>;
  if (splits == 1) {
    kern<<<dim3((unsigned)gx, (unsigned)gy), (BM / TM) * (BN / TN), 0, ctx->stream>>>(s, A, B, epi, s.K, nullptr);
    GT_LAUNCH_CHECK();
    return nullptr;
  }
  // K ranges in whole BK slices; splits that would start past K are dropped
  const int64_t k_per = ceil_div(ceil_div(s.K, (int64_t)splits), (int64_t)BK) * BK;
  const int S = (int)ceil_div(s.K, k_per);
  void* ws = nullptr;
  GT_TRY(scratch(ctx, (size_t)S * s.M * s.N * sizeof(T), &ws));
  kern<<<dim3((unsigned)gx, (unsigned)gy, (unsigned)S), (BM / TM) * (BN / TN), 0, ctx->stream>>>(s, A, B, epi, k_per,
                                                                                               (T*)ws);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    simt_split_reduce_kernel<T><<<grid_for(ctx, s.M * s.N, 256), 256, 0, ctx->stream>>>((const T*)ws, S, s.M, s.N, epi);
    count_launch();
    e = cudaGetLastError();
  }
  release(ctx, ws);
  if (e != cudaSuccess) return cuda_error(e, "gemm_simt launch", __FILE__, __LINE__);
  return nullptr;
}

template <typename T>
char* gemm_simt(gt_ctx* ctx, const GemmShape& s, const T* A, const T* B, const Epi<T>& epi) {
  if (s.M <= 0 || s.N <= 0) return nullptr;
  if (sizeof(T) == 4) {
    // Block tile by shape (always 16 x 16 threads): skinny outputs such as a
    // conv's first-layer weight gradient (64 x 27) would leave most of a
    // 128 x 128 tile idle.
    const bool short_m = s.M <= 64, narrow_n = s.N <= 32;
    if (short_m && narrow_n) return simt_launch<T, 64, 32, 8, 4, 2>(ctx, s, A, B, epi);
    if (short_m) return simt_launch<T, 64, 128, 8, 4, 8>(ctx, s, A, B, epi);
    if (narrow_n) return simt_launch<T, 128, 32, 8, 8, 2>(ctx, s, A, B, epi);
    return simt_launch<T, 128, 128, 8, 8, 8>(ctx, s, A, B, epi);
  }
  return simt_launch<T, 64, 64, 8, 4, 4>(ctx, s, A, B, epi);
}

template char* gemm_simt<float>(gt_ctx*, const GemmShape&, const float*, const float*, const Epi<float>&);
template char* gemm_simt<double>(gt_ctx*, const GemmShape&, const double*, const double*, const Epi<double>&);

}  // namespace gt
