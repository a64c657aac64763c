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
#include <algorithm>

#include "gemm.cuh"

namespace gt {

// Float tiles up to 64 x 128 ask for 3 resident blocks per SM: the first
// conv's GEMMs (K = 27 or 9) wait on global loads most of the time, and the
// extra warps hide that (measured: conv stack 4.91 to 4.81 ms per step).
template <typename T, int BM, int BN, int BK, int TM, int TN>
__global__ void __launch_bounds__((BM / TM) * (BN / TN), (sizeof(T) == 4 && BM * BN <= 64 * 128) ? 3 : 1)
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

  if (!ws && epi.nchw_L > 0) {
    // NCHW store (a convolution's output): the thread's TN consecutive
    // columns are split into (image, position) once and then stepped, not
    // divided per element.
    const int64_t nb = n0 + tx * TN;
    int64_t img = nb / epi.nchw_L, pos = nb - img * epi.nchw_L;
#pragma unroll
    for (int j = 0; j < TN; j++) {
      if (nb + j < N) {
        T* col = epi.out + img * epi.nchw_M * epi.nchw_L + pos;
#pragma unroll
        for (int i = 0; i < TM; i++) {
          const int64_t m = m0 + ty * TM + i;
          if (m < M) col[m * epi.nchw_L] = epi.finish(m, nb + j, acc[i][j]);
        }
      }
      if (++pos == epi.nchw_L) pos = 0, img++;
    }
    return;
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

// Four consecutive elements from a 4-element-aligned address, as vectors.
__device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
  const float4 q = __ldg((const float4*)p);
  v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
}
__device__ __forceinline__ void load4(const double* p, double (&v)[4]) {
  const double2 q0 = __ldg((const double2*)p), q1 = __ldg((const double2*)p + 1);
  v[0] = q0.x, v[1] = q0.y, v[2] = q1.x, v[3] = q1.y;
}

// Small K (the input gradient of a classifier: K = its 10 classes): C = A
// (M x K, row-major) @ B (K x N, row-major), a thread per four consecutive
// columns of a row. B's row k is read as one four-element vector per thread
// (coalesced), A(m, k) is the same for the warp's threads (broadcast), and
// each output is the same FMA chain over k, in order, as gemm_simt_kernel's,
// so the results are identical; the outputs leave as contiguous runs.
template <typename T>
__global__ void gemm_smallk_kernel(GemmShape s, const T* __restrict__ A, const T* __restrict__ B, Epi<T> epi) {
  const int64_t qn = s.N / 4, total = s.M * qn;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = u / qn, n = 4 * (u - m * qn);
    T acc[4] = {(T)0, (T)0, (T)0, (T)0};
    const T* a = A + m * s.lda;
#pragma unroll 4
    for (int64_t k = 0; k < s.K; k++) {
      const T av = __ldg(a + k);
      T bv[4];
      load4(B + k * s.ldb + n, bv);
#pragma unroll
      for (int j = 0; j < 4; j++) acc[j] = fma(av, bv[j], acc[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; j++) epi.store(m, n + j, acc[j]);
  }
}

// Thin GEMMs, where a classifier's 10 classes make one dimension tiny and
// the cost is streaming the other operand once:
//
// gemm_thin_n_kernel, N <= NN (the forward x @ W^T of a classifier): WR
// warps per row of C (8 / WR rows per 256-thread block), warp w of a row
// taking the w-th of WR equal K ranges; lane l accumulates k = l, l + 32, ...
// of its range for all N dot products (A's row read once, coalesced; W's N
// rows stay in L1). The lanes' sums are added by a xor butterfly (the same
// order on every lane), the row's WR warp sums in warp order through shared
// memory, and lane n stores C(m, n) through the epilogue.
template <typename T, int NN>
__global__ void __launch_bounds__(256) gemm_thin_n_kernel(GemmShape s, const T* __restrict__ A,
                                                          const T* __restrict__ B, Epi<T> epi, int WR) {
  __shared__ T part[8][NN];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rows_per_block = 8 / WR, r = warp / WR, w = warp - r * WR;
  const int N = (int)s.N;
  const int64_t kr = (s.K + WR - 1) / WR, k_lo = w * kr, k_hi = k_lo + kr < s.K ? k_lo + kr : s.K;
  for (int64_t m0 = (int64_t)blockIdx.x * rows_per_block; m0 < s.M; m0 += (int64_t)gridDim.x * rows_per_block) {
    const int64_t m = m0 + r;
    T acc[NN];
#pragma unroll
    for (int n = 0; n < NN; n++) acc[n] = (T)0;
    if (m < s.M) {
      const T* a = A + m * s.lda;
#pragma unroll 2
      for (int64_t k = k_lo + lane; k < k_hi; k += 32) {
        const T av = a[k];
#pragma unroll
        for (int n = 0; n < NN; n++)
          if (n < N) acc[n] = fma(av, __ldg(B + n * s.ldb + k), acc[n]);
      }
    }
    T mine = (T)0;
#pragma unroll
    for (int n = 0; n < NN; n++) {
      if (n < N) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc[n] = acc[n] + __shfl_xor_sync(0xffffffffu, acc[n], off);
      }
      if (lane == n) mine = acc[n];
    }
    if (WR == 1) {
      if (m < s.M && lane < N) epi.store(m, lane, mine);
      continue;
    }
    if (lane < N) part[warp][lane] = mine;
    __syncthreads();
    if (w == 0 && m < s.M && lane < N) {
      T sum = part[warp][lane];
      for (int j = 1; j < WR; j++) sum = sum + part[warp + j][lane];
      epi.store(m, lane, sum);
    }
    __syncthreads();
  }
}

// gemm_thin_m_kernel, M <= MM (a classifier's weight gradient dY^T @ X): a
// thread per column n of C over the block's K range; the range's rows of A
// (M values each) are staged in shared memory and broadcast, B's row is read
// coalesced. part[y][m][n] holds the partial sums of K range y; the ranges are
// added in order afterwards (column_sums_kernel over the y rows).
template <typename T, int MM>
__global__ void __launch_bounds__(256) gemm_thin_m_kernel(GemmShape s, const T* __restrict__ A,
                                                          const T* __restrict__ B, int64_t k_per,
                                                          T* __restrict__ part) {
  __shared__ T as[64][MM];
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t k0 = (int64_t)blockIdx.y * k_per, k1 = k0 + k_per < s.K ? k0 + k_per : s.K;
  const int M = (int)s.M;
  T acc[MM];
#pragma unroll
  for (int m = 0; m < MM; m++) acc[m] = (T)0;
  for (int64_t kc = k0; kc < k1; kc += 64) {
    const int kn = (int)(k1 - kc < 64 ? k1 - kc : 64);
    __syncthreads();
    for (int e = threadIdx.x; e < 64 * MM; e += blockDim.x) {
      const int kk = e / MM, mm = e - kk * MM;
      as[kk][mm] = kk < kn && mm < M ? A[(kc + kk) * s.lda + mm] : (T)0;
    }
    __syncthreads();
    if (n < s.N) {
      const T* b = B + kc * s.ldb + n;
#pragma unroll 4
      for (int kk = 0; kk < kn; kk++) {
        const T bv = b[(int64_t)kk * s.ldb];
#pragma unroll
        for (int m = 0; m < MM; m++) acc[m] = fma(as[kk][m], bv, acc[m]);
      }
    }
  }
  if (n < s.N)
#pragma unroll
    for (int m = 0; m < MM; m++)
      if (m < M) part[((int64_t)blockIdx.y * M + m) * s.N + n] = acc[m];
}

template <typename T>
char* gemm_thin(gt_ctx* ctx, const GemmShape& s, const T* A, const T* B, const Epi<T>& epi, bool* done) {
  *done = false;
  if (s.M <= 0 || s.N <= 0 || s.K <= 0) return nullptr;
  const bool generic_out = epi.nchw_L == 0 && !epi.col_major && !epi.pos_major && !epi.colsum_ws && !epi.bits_out &&
                           !epi.pool_idx && !epi.dbits;
  if (!generic_out) return nullptr;
  if (s.N <= 32 && !s.trans_a && s.trans_b && s.M >= 16 && s.K >= 32) {
    // warps per row: K ranges of at least 256, while the rows alone leave
    // fewer than 32 warps per SM
    int wr = 1;
    while (wr < 8 && s.K / (2 * wr) >= 256 && s.M * wr < 32 * (int64_t)ctx->sm_count) wr *= 2;
    const int64_t rows_per_block = 8 / wr;
    const int grid = (int)std::min<int64_t>(ceil_div(s.M, rows_per_block), (int64_t)ctx->sm_count * 8);
    if (s.N <= 16)
      gemm_thin_n_kernel<T, 16><<<grid, 256, 0, ctx->stream>>>(s, A, B, epi, wr);
    else
      gemm_thin_n_kernel<T, 32><<<grid, 256, 0, ctx->stream>>>(s, A, B, epi, wr);
    GT_LAUNCH_CHECK();
    *done = true;
    return nullptr;
  }
  const bool plain = !epi.bias && epi.act == GT_ACT_NONE && !epi.dmask && epi.ldc == s.N;
  if (s.M <= 32 && s.trans_a && !s.trans_b && plain && s.N >= 64 && s.K >= 64) {
    const int64_t gx = ceil_div(s.N, 256);
    int64_t S = ceil_div(4 * (int64_t)ctx->sm_count, gx);
    S = std::min<int64_t>(S, ceil_div(s.K, 32));
    const int64_t k_per = ceil_div(s.K, S);
    S = ceil_div(s.K, k_per);
    if (S > 65535) return nullptr;
    void* part = nullptr;
    GT_TRY(scratch(ctx, (size_t)(S * s.M * s.N) * sizeof(T), &part));
    if (s.M <= 16)
      gemm_thin_m_kernel<T, 16><<<dim3((unsigned)gx, (unsigned)S), 256, 0, ctx->stream>>>(s, A, B, k_per, (T*)part);
    else
      gemm_thin_m_kernel<T, 32><<<dim3((unsigned)gx, (unsigned)S), 256, 0, ctx->stream>>>(s, A, B, k_per, (T*)part);
    column_sums_kernel<T><<<(unsigned)ceil_div(s.M * s.N, 32), 1024, 0, ctx->stream>>>((const T*)part, S, s.M * s.N,
                                                                                     epi.out);
    count_launch(2);
    cudaError_t e = cudaGetLastError();
    release(ctx, part);
    if (e != cudaSuccess) return cuda_error(e, "gemm_thin_m launch", __FILE__, __LINE__);
    *done = true;
    return nullptr;
  }
  return nullptr;
}

template char* gemm_thin<float>(gt_ctx*, const GemmShape&, const float*, const float*, const Epi<float>&, bool*);
template char* gemm_thin<double>(gt_ctx*, const GemmShape&, const double*, const double*, const Epi<double>&, bool*);

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

// FP64 main kernel on the FP64 tensor-core path (mma.sync m8n8k4 f64, 256
// fused multiply-adds per warp instruction, so sixteen warps per SM keep the
// pipe busy where DFMA would be issue-bound): a 128 x 128 tile per CTA over
// 32-deep K slices, staged k-major in shared memory by cp.async (8-byte
// elements, out-of-range ones zero-filled) in a three-slice ring with one
// barrier per slice, so two slices' loads run under the MMAs. Sixteen warps
// (four per scheduler, which the MMA latency needs): warp w computes rows
// 32 * (w / 4) .. +32 and columns 32 * (w % 4) .. +32 as 4 x 4 MMA tiles.
// Each operand keeps its memory order in shared memory, so every 32-byte
// sector a copy brings lands in one contiguous run: an operand whose K index
// is contiguous is stored [row][k] in rows of 36 doubles, the other [k][row]
// in rows of 132. Fragment reads (thread t takes k = t % 4 and row t / 4 of
// an 8 x 4 block) then fall in distinct banks in both layouts. Copies are 16
// bytes (two elements) when both operands' bases and leading dimensions allow
// it, else 8.
//
// Work units: units 0 .. whole-1 are whole tiles; after them each remaining
// tile is `splits` units over consecutive K ranges of k_per, whose partial
// tiles go to ws and are added in K order by f64_tail_reduce_kernel, so the
// last wave's tiles spread over all SMs instead of leaving most of them idle.
namespace f64k {
constexpr int BM = 128, BN = 128, BK = 32, THREADS = 512;
constexpr int PITCH = 132;  // [k][row] layout: row stride of a k
constexpr int PK = 36;      // [row][k] layout: row stride of a row
constexpr int STAGES = 3;   // slices in the shared-memory ring
constexpr int OPS = BK * PITCH > 128 * PK ? BK * PITCH : 128 * PK;  // doubles per operand and stage
constexpr size_t SMEM = (size_t)STAGES * 2 * OPS * sizeof(double);
static_assert(BM == 128 && BN == 128 && 128 * BK % (2 * THREADS) == 0 && BK % 4 == 0, "copy mapping");

struct Plan {
  int whole = 0;        // units that are whole tiles
  int splits = 1;       // units per remaining tile
  int64_t k_per = 0;    // K range of a split unit (a multiple of BK)
  int64_t gx = 1;       // tiles along N
};

__device__ __forceinline__ void cp_async8(double* dst, const double* src, bool valid) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(d), "l"(src), "r"(valid ? 8 : 0) : "memory");
}

__device__ __forceinline__ void cp_async16(double* dst, const double* src, int bytes) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mma_f64(double (&c)[2], double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
               : "+d"(c[0]), "+d"(c[1])
               : "d"(a), "d"(b));
}

// Copies the BK x 128 slice [k0, k0 + BK) x [r0, r0 + 128) of an operand
// into one stage. KC: element (k, r) is at src[r * ld + k] (stored [row][k],
// rows of PK); otherwise at src[k * ld + r] (stored [k][row], rows of
// PITCH). Elements past k_end or rlim are zero-filled without being read.
template <bool KC, bool V16>
__device__ __forceinline__ void copy_slice(double* dst, const double* __restrict__ src, int64_t ld, int64_t k0,
                                           int64_t k_end, int64_t r0, int64_t rlim, int tid) {
  if constexpr (V16) {
#pragma unroll
    for (int q = 0; q < 128 * BK / (2 * THREADS); q++) {
      const int e = tid + THREADS * q;
      if constexpr (KC) {  // two consecutive k of one row
        const int r = e / (BK / 2), k = 2 * (e % (BK / 2));
        const int64_t gr = r0 + r, gk = k0 + k;
        const int bytes = gr < rlim ? (gk + 1 < k_end ? 16 : gk < k_end ? 8 : 0) : 0;
        cp_async16(dst + r * PK + k, bytes ? src + gr * ld + gk : src, bytes);
      } else {  // two consecutive rows of one k
        const int k = e / 64, r = 2 * (e % 64);
        const int64_t gr = r0 + r, gk = k0 + k;
        const int bytes = gk < k_end ? (gr + 1 < rlim ? 16 : gr < rlim ? 8 : 0) : 0;
        cp_async16(dst + k * PITCH + r, bytes ? src + gk * ld + gr : src, bytes);
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < 128 * BK / THREADS; q++) {
      const int e = tid + THREADS * q;
      const int k = KC ? e % BK : e / 128, r = KC ? e / BK : e % 128;
      const int64_t gr = r0 + r, gk = k0 + k;
      const bool ok = gr < rlim && gk < k_end;
      cp_async8(dst + (KC ? r * PK + k : k * PITCH + r), ok ? (KC ? src + gr * ld + gk : src + gk * ld + gr) : src,
                ok);
    }
  }
}

// Element (k, r) of a stage in its layout.
template <bool KC>
__device__ __forceinline__ int stage_at(int k, int r) {
  return KC ? r * PK + k : k * PITCH + r;
}
}  // namespace f64k

template <bool TA, bool TB, bool V16>
__global__ void __launch_bounds__(f64k::THREADS, 1)
    gemm_f64_kernel(GemmShape s, const double* __restrict__ A, const double* __restrict__ B, Epi<double> epi,
                    f64k::Plan plan, double* __restrict__ ws) {
  using namespace f64k;
  extern __shared__ double sm[];
  double* As = sm;                 // [STAGES][OPS]
  double* Bs = sm + STAGES * OPS;  // [STAGES][OPS]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = 32 * (warp >> 2), wn = 32 * (warp & 3);
  const int u = blockIdx.x;
  int64_t tile, k_begin = 0, k_end = s.K;
  int split = -1;
  if (u < plan.whole) {
    tile = u;
  } else {
    const int r = u - plan.whole;
    tile = plan.whole + r / plan.splits;
    split = r % plan.splits;
    k_begin = (int64_t)split * plan.k_per;
    k_end = k_begin + plan.k_per < s.K ? k_begin + plan.k_per : s.K;
  }
  const int64_t m0 = (tile / plan.gx) * BM, n0 = (tile % plan.gx) * BN;
  const int slices = (int)((k_end - k_begin + BK - 1) / BK);

  // A is K-contiguous unless transposed; B is K-contiguous when transposed.
  auto load = [&](int slice, int stage) {
    const int64_t k0 = k_begin + (int64_t)slice * BK;
    copy_slice<!TA, V16>(As + stage * OPS, A, s.lda, k0, k_end, m0, s.M, tid);
    copy_slice<TB, V16>(Bs + stage * OPS, B, s.ldb, k0, k_end, n0, s.N, tid);
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  double acc[4][4][2];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j][0] = acc[i][j][1] = 0.0;

  const int fk = lane & 3, fr = lane >> 2;  // fragment k and row / column
  // One commit group per slice (empty past the end). At slice t: waiting
  // until at most STAGES - 2 groups are pending means slice t has landed;
  // the barrier then makes every thread's copies visible and frees the
  // stage slice t - 1 used, which the load of slice t + STAGES - 1 refills.
#pragma unroll
  for (int p = 0; p < STAGES - 1; p++) {
    if (p < slices) load(p, p);
    else asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int t = 0; t < slices; t++) {
    asm volatile("cp.async.wait_group %0;" ::"n"(STAGES - 2) : "memory");
    __syncthreads();
    const int next = t + STAGES - 1;
    if (next < slices) load(next, next % STAGES);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    const double* as = As + (t % STAGES) * OPS + stage_at<!TA>(fk, wm + fr);
    const double* bs = Bs + (t % STAGES) * OPS + stage_at<TB>(fk, wn + fr);
#pragma unroll
    for (int k4 = 0; k4 < BK; k4 += 4) {
      double a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = as[stage_at<!TA>(k4, 8 * i)];
#pragma unroll
      for (int j = 0; j < 4; j++) b[j] = bs[stage_at<TB>(k4, 8 * j)];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) mma_f64(acc[i][j], a[i], b[j]);
    }
  }

  // Thread t holds C(8 i + t / 4, 8 j + 2 (t % 4) + {0, 1}) of the warp's tile;
  // a split unit writes its partial tile, row-major 128 x 128, to ws.
  double* part = split < 0 ? nullptr : ws + ((tile - plan.whole) * plan.splits + split) * (int64_t)(BM * BN);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t m = m0 + wm + 8 * i + fr;
    if (m >= s.M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int64_t n = n0 + wn + 8 * j + 2 * fk + h;
        if (n >= s.N) continue;
        if (part)
          part[(m - m0) * BN + (n - n0)] = acc[i][j][h];
        else
          epi.store(m, n, acc[i][j][h]);
      }
    }
  }
}

// The split tiles: C = epilogue(sum of a tile's partials in K order).
__global__ void f64_tail_reduce_kernel(const double* __restrict__ ws, f64k::Plan plan, int64_t tiles, GemmShape s,
                                       Epi<double> epi) {
  using namespace f64k;
  const int64_t total = (tiles - plan.whole) * (int64_t)(BM * BN);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (BM * BN), e = i - r * (BM * BN), tile = plan.whole + r;
    const int64_t m = (tile / plan.gx) * BM + e / BN, n = (tile % plan.gx) * BN + e % BN;
    if (m >= s.M || n >= s.N) continue;
    const double* p = ws + r * plan.splits * (int64_t)(BM * BN) + e;
    double acc = p[0];
    for (int k = 1; k < plan.splits; k++) acc = add_rn(acc, p[(int64_t)k * BM * BN]);
    epi.store(m, n, acc);
  }
}

// The unit plan: whole tiles while they fill every SM, then the remaining
// tiles in the number of K ranges that minimises (rounds of units) x (unit
// depth) plus the partials' traffic (one CTA per SM; ranges at least 128 deep).
static f64k::Plan f64_plan(int64_t tiles, int64_t gx, int64_t K, int64_t sms) {
  using namespace f64k;
  Plan best;
  best.gx = gx;
  best.whole = (int)tiles;
  best.k_per = K;
  const int64_t rest = tiles % sms, whole = tiles - rest;
  if (rest == 0) return best;
  const double tile_s = 2.0 * BM * BN * (double)K / (37e12 / (double)sms);  // one tile on one SM
  auto cost = [&](int64_t S) {
    const int64_t k_per = ceil_div(ceil_div(K, S), (int64_t)BK) * BK, units = rest * ceil_div(K, k_per);
    const double depth = (double)k_per / (double)K;
    const double traffic = S > 1 ? 2.0 * (double)units * BM * BN * 8 / 6.5e12 : 0.0;
    return (double)((whole + sms - 1) / sms) * tile_s + (double)ceil_div(units, sms) * depth * tile_s + traffic;
  };
  double best_cost = cost(1);
  for (int64_t S = 2; S <= 32 && K / S >= 128; S++) {
    const double c = cost(S);
    if (c < 0.97 * best_cost) {
      best_cost = c;
      best.k_per = ceil_div(ceil_div(K, S), (int64_t)BK) * BK;
      best.splits = (int)ceil_div(K, best.k_per);
      best.whole = (int)whole;
    }
  }
  return best;
}

template <bool TA, bool TB, bool V16>
static char* f64_launch(gt_ctx* ctx, const GemmShape& s, const double* A, const double* B, const Epi<double>& epi) {
  using namespace f64k;
  const int64_t gx = ceil_div(s.N, BN), gy = ceil_div(s.M, BM), tiles = gx * gy;
  auto kern = gemm_f64_kernel<TA, TB, V16>;
  static bool configured[64] = {};
  if (ctx->device < 0 || ctx->device >= 64 || !configured[ctx->device]) {
    GT_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM));
    if (ctx->device >= 0 && ctx->device < 64) configured[ctx->device] = true;
  }
  Plan plan = f64_plan(tiles, gx, s.K, ctx->sm_count);
  // keep the partials under 256 MB
  while (plan.splits > 1 && (double)(tiles - plan.whole) * plan.splits * BM * BN * 8 > (double)(256u << 20)) {
    plan.k_per = ceil_div(ceil_div(s.K, (int64_t)plan.splits / 2), (int64_t)BK) * BK;
    plan.splits = (int)ceil_div(s.K, plan.k_per);
  }
  if (plan.splits <= 1) plan.whole = (int)tiles;
  const int64_t units = plan.whole + (tiles - plan.whole) * plan.splits;
  if (units > INT32_MAX) return errorf("gemm_f64: %lld output tiles", (long long)units);
  double* ws = nullptr;
  if (plan.splits > 1) {
    void* w = nullptr;
    GT_TRY(scratch(ctx, (size_t)(tiles - plan.whole) * plan.splits * BM * BN * sizeof(double), &w));
    ws = (double*)w;
  }
  kern<<<(unsigned)units, THREADS, SMEM, ctx->stream>>>(s, A, B, epi, plan, ws);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && ws) {
    f64_tail_reduce_kernel<<<grid_for(ctx, (tiles - plan.whole) * BM * BN, 256), 256, 0, ctx->stream>>>(
        ws, plan, tiles, s, epi);
    count_launch();
    e = cudaGetLastError();
  }
  if (ws) release(ctx, ws);
  if (e != cudaSuccess) return cuda_error(e, "gemm_f64 launch", __FILE__, __LINE__);
  return nullptr;
}

template <bool V16>
static char* f64_layouts(gt_ctx* ctx, const GemmShape& s, const double* A, const double* B, const Epi<double>& epi) {
  if (s.trans_a)
    return s.trans_b ? f64_launch<true, true, V16>(ctx, s, A, B, epi) : f64_launch<true, false, V16>(ctx, s, A, B, epi);
  return s.trans_b ? f64_launch<false, true, V16>(ctx, s, A, B, epi) : f64_launch<false, false, V16>(ctx, s, A, B, epi);
}

// 16-byte copies need 16-byte aligned bases and even leading dimensions
// (every copied pair then starts on a 16-byte boundary).
static char* f64_main(gt_ctx* ctx, const GemmShape& s, const double* A, const double* B, const Epi<double>& epi) {
  const bool v16 = !((uintptr_t)A & 15) && !((uintptr_t)B & 15) && !(s.lda & 1) && !(s.ldb & 1);
  return v16 ? f64_layouts<true>(ctx, s, A, B, epi) : f64_layouts<false>(ctx, s, A, B, epi);
}

template <typename T>
char* gemm_simt(gt_ctx* ctx, const GemmShape& s, const T* A, const T* B, const Epi<T>& epi) {
  if (s.M <= 0 || s.N <= 0) return nullptr;
  // K of a few classes over a wide output (row-major operands, N a multiple
  // of 4): the output is the cost, written in contiguous runs
  if (s.K <= 32 && !s.trans_a && !s.trans_b && s.N % 4 == 0 && s.ldb % 4 == 0 && s.M * s.N >= 4096 &&
      !((uintptr_t)B & (4 * sizeof(T) - 1)) && epi.nchw_L == 0 && !epi.col_major) {
    gemm_smallk_kernel<T><<<grid_for(ctx, s.M * s.N / 4, 256), 256, 0, ctx->stream>>>(s, A, B, epi);
    GT_LAUNCH_CHECK();
    return nullptr;
  }
  // float64 outputs of at least 128 x 128 with K long enough to amortise the
  // one-CTA-per-SM epilogue go to the tensor-core kernel.
  if constexpr (sizeof(T) == 8)
    if (s.M >= 128 && s.N >= 128 && s.K >= 128) return f64_main(ctx, s, A, B, epi);
  // Block tile by shape (always 16 x 16 threads): skinny outputs such as a
  // conv's first-layer weight gradient (64 x 27) or a 10-class classifier
  // (and its 10-row weight gradient) would leave most of a square tile idle.
  const bool tiny_m = s.M <= 16, short_m = s.M <= 64, narrow_n = s.N <= 32;
  if (tiny_m) return narrow_n ? simt_launch<T, 16, 32, 8, 1, 2>(ctx, s, A, B, epi)
                              : simt_launch<T, 16, 128, 8, 1, 8>(ctx, s, A, B, epi);
  // long K over a skinny output (a first-layer conv's weight gradient): 32-deep
  // slices, so each row of A is read 128 contiguous bytes at a time
  if (short_m && narrow_n && s.K >= 65536 && !s.trans_a) return simt_launch<T, 64, 32, 32, 4, 2>(ctx, s, A, B, epi);
  if (short_m && narrow_n) return simt_launch<T, 64, 32, 8, 4, 2>(ctx, s, A, B, epi);
  if (short_m) return simt_launch<T, 64, 128, 8, 4, 8>(ctx, s, A, B, epi);
  if (narrow_n) return simt_launch<T, 128, 32, 8, 8, 2>(ctx, s, A, B, epi);
  if constexpr (sizeof(T) == 4)
    return simt_launch<T, 128, 128, 8, 8, 8>(ctx, s, A, B, epi);
  else
    return simt_launch<T, 64, 64, 8, 4, 4>(ctx, s, A, B, epi);
}

template char* gemm_simt<float>(gt_ctx*, const GemmShape&, const float*, const float*, const Epi<float>&);
template char* gemm_simt<double>(gt_ctx*, const GemmShape&, const double*, const double*, const Epi<double>&);

}  // namespace gt
