// GEMM dispatch and the entry points built on it: Backend.MatMul
// (internal/backend/backend.go:150) and the fused Linear forward/backward.
#include <vector>

#include "gemm.cuh"

namespace gt {

static int g_gemm_path = 0;
static int g_gemm_taken = 0;
void set_gemm_path(int path) { g_gemm_path = path; }
int gemm_path() { return g_gemm_path; }

}  // namespace gt

// Per-launch device times of the GEMMs issued on a context: a CUDA event on
// the context's stream before and after each GEMM kernel, so the figures are
// the kernels' own durations inside whatever step issues them.
struct gt_gemm_timer {
  struct Launch {
    int64_t m, n, k;
    int path;
    cudaEvent_t start, end;
  };
  std::vector<Launch> launches;
  int64_t used = 0, dropped = 0;
};

namespace gt {

// Brackets one GEMM with the context's timer events (when a timer is on and
// the stream is not being captured into a graph).
// With `done`, a call that ends with *done false launched nothing and leaves
// no record.
template <typename F>
static char* timed_gemm(gt_ctx* ctx, const GemmShape& s, F&& run, const bool* done = nullptr) {
  gt_gemm_timer* t = ctx->gemm_timer;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (t) GT_CUDA(cudaStreamIsCapturing(ctx->stream, &cap));
  if (!t || cap != cudaStreamCaptureStatusNone) return run();
  if (t->used >= (int64_t)t->launches.size()) {
    char* err = run();
    if (!done || *done) t->dropped++;
    return err;
  }
  auto& l = t->launches[t->used++];
  l.m = s.M, l.n = s.N, l.k = s.K;
  GT_CUDA(cudaEventRecord(l.start, ctx->stream));
  char* err = run();
  l.path = g_gemm_taken;
  GT_CUDA(cudaEventRecord(l.end, ctx->stream));
  if (done && !*done) t->used--;
  return err;
}

static char* gemm_f32(gt_ctx* ctx, const GemmShape& s, const float* A, const float* B, const Epi<float>& epi);

// The implicit-GEMM convolutions, timed like any GEMM (path 4). The timer
// records the convolution's own GEMM shape (M = positions or patch entries
// without the bias-gradient row), so its flops are the algorithmic ones.
char* conv_fwd_gemm(gt_ctx* ctx, const float* x, const float* w, int64_t w_pitch, const float* bias, float* y,
                    const gt_geom& g, int64_t O, int act, bool* done, uint8_t* pool_idx) {
  *done = false;
  if (g_gemm_path == 1) return nullptr;  // SIMT pinned: the explicit path
  GemmShape ts{g.N * g.OH * g.OW, O, g.C * g.KH * g.KW, false, true, 0, 0};
  return timed_gemm(
      ctx, ts,
      [&] {
        char* e = conv_fwd_tc(ctx, x, w, w_pitch, bias, y, g, O, act, done, pool_idx);
        if (*done) g_gemm_taken = 4;
        return e;
      },
      done);
}

char* conv_wgrad_gemm(gt_ctx* ctx, const float* x, const float* dy, float* dw, float* db, const gt_geom& g,
                      int64_t O, bool* done) {
  *done = false;
  if (g_gemm_path == 1) return nullptr;
  GemmShape ts{O, g.C * g.KH * g.KW, g.N * g.OH * g.OW, true, false, 0, 0};
  return timed_gemm(
      ctx, ts,
      [&] {
        char* e = conv_wgrad_tc(ctx, x, dy, dw, db, g, O, done);
        if (*done) g_gemm_taken = 4;
        return e;
      },
      done);
}

// A kernel that computes a GEMM's result by other means, timed and recorded
// like the GEMMs under `path` (the fused pool-backward weight gradient).
char* timed_gemm_like(gt_ctx* ctx, int64_t M, int64_t N, int64_t K, int path, char* (*run)(void*), void* arg) {
  GemmShape ts{M, N, K, false, false, 0, 0};
  return timed_gemm(ctx, ts, [&] {
    char* e = run(arg);
    g_gemm_taken = path;
    return e;
  });
}

template <>
char* gemm<double>(gt_ctx* ctx, const GemmShape& s, const double* A, const double* B, const Epi<double>& epi) {
  if (g_gemm_path == 2) return errorf("gemm: the tcgen05 path has no float64 kind");
  return timed_gemm(ctx, s, [&] {
    if (g_gemm_path == 0) {  // the thin kernels only on the automatic path
      bool done = false;
      char* e = gemm_thin<double>(ctx, s, A, B, epi, &done);
      if (e || done) {
        g_gemm_taken = 6;
        return e;
      }
    }
    g_gemm_taken = 1;
    return gemm_simt<double>(ctx, s, A, B, epi);
  });
}

template <>
char* gemm<float>(gt_ctx* ctx, const GemmShape& s, const float* A, const float* B, const Epi<float>& epi) {
  return timed_gemm(ctx, s, [&] {
    if (g_gemm_path == 0) {  // the thin kernels only on the automatic path
      bool done = false;
      char* e = gemm_thin<float>(ctx, s, A, B, epi, &done);
      if (e || done) {
        g_gemm_taken = 6;
        return e;
      }
    }
    return gemm_f32(ctx, s, A, B, epi);
  });
}

static char* gemm_f32(gt_ctx* ctx, const GemmShape& s, const float* A, const float* B, const Epi<float>& epi) {
  if (g_gemm_path != 1) {
    bool done = false;
    GT_TRY(gemm_tc_f32(ctx, s, A, B, epi, &done));
    if (done) {
      g_gemm_taken = 2;
      return nullptr;
    }
    if (g_gemm_path == 2)
      return errorf("gemm: shape M=%lld N=%lld K=%lld does not qualify for the tcgen05 path", (long long)s.M,
                    (long long)s.N, (long long)s.K);
  }
  g_gemm_taken = 1;
  return gemm_simt<float>(ctx, s, A, B, epi);
}

}  // namespace gt

using namespace gt;

namespace gt {

// bits[b * N + n] bit j = (y[32 b + j][n] > 0): a thread per word;
// consecutive threads take consecutive columns, so the 32 row reads and the
// word stores are coalesced.
template <typename T>
__global__ void relu_bits_kernel(const T* __restrict__ y, uint32_t* __restrict__ bits, int64_t M, int64_t N) {
  const int64_t words = (M + 31) / 32 * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / N, n = i - b * N;
    uint32_t w = 0;
    for (int j = 0; j < 32 && 32 * b + j < M; j++) w |= (uint32_t)(y[(32 * b + j) * N + n] > (T)0) << j;
    bits[i] = w;
  }
}

// dx = the GEMM of s with epilogue e (a Linear's input gradient, M x K), and
// db_prev (K) = its column sums: the bias gradient of the Linear that
// produced this layer's input (sumTo over the batch, tensor/ops.go:418-433).
// On the float32 tcgen05 path the epilogue adds each 32-row block's columns
// while it stores them, and one small kernel adds the blocks; elsewhere a
// reduction over dx follows the GEMM.
static char* bwd_data_with_db(gt_ctx* ctx, int dtype, const GemmShape& s, const void* dy, const void* w, void* dx,
                              void* db_prev, const Epi<float>& ef, const Epi<double>& ed, int64_t M, int64_t K) {
  if (dtype == GT_FLOAT32 && tc_writes_colsums(ef, K)) {
    const int64_t blocks = ceil_div(M, 32);
    void* ws = nullptr;
    GT_TRY(scratch(ctx, (size_t)(blocks * K) * sizeof(float), &ws));
    Epi<float> e = ef;
    e.colsum_ws = (float*)ws;
    e.ldcs = K;
    char* err = gemm<float>(ctx, s, (const float*)dy, (const float*)w, e);
    const bool fused = !err && g_gemm_taken == 2;
    if (fused) {
      column_sums_kernel<float><<<(unsigned)ceil_div(K, 32), 1024, 0, ctx->stream>>>((const float*)ws, blocks, K,
                                                                                     (float*)db_prev);
      count_launch();
      cudaError_t ce = cudaGetLastError();
      if (ce != cudaSuccess) err = cuda_error(ce, "column_sums_kernel launch", __FILE__, __LINE__);
    }
    release(ctx, ws);
    if (err || fused) return err;
  } else if (dtype == GT_FLOAT32) {
    GT_TRY(gemm<float>(ctx, s, (const float*)dy, (const float*)w, ef));
  } else {
    GT_TRY(gemm<double>(ctx, s, (const double*)dy, (const double*)w, ed));
  }
  return gt_reduce(ctx, dtype, GT_SUM, dx, db_prev, 1, M, K);
}

}  // namespace gt

extern "C" {

char* gt_linear_bwd_data_db(gt_ctx* ctx, int dtype, const void* dy, const void* w, const void* y_prev, int act_prev,
                            void* dx, void* db_prev, int64_t M, int64_t K, int64_t N) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (M <= 0 || K <= 0 || N <= 0 || !db_prev) return errorf("gt_linear_bwd_data_db: bad arguments");
  GemmShape s{M, K, N, false, false, N, K};
  Epi<float> ef;
  Epi<double> ed;
  ef.out = (float*)dx, ed.out = (double*)dx;
  ef.ldc = ed.ldc = K;
  if (y_prev && act_prev != GT_ACT_NONE) {
    ef.dmask = (const float*)y_prev, ed.dmask = (const double*)y_prev;
    ef.dact = ed.dact = act_prev;
    ef.ldm = ed.ldm = K;
  }
  return bwd_data_with_db(ctx, dtype, s, dy, w, dx, db_prev, ef, ed, M, K);
}

char* gt_linear_bwd_data_bits_db(gt_ctx* ctx, int dtype, const void* dy, const void* w, const uint32_t* bits,
                                 void* dx, void* db_prev, int64_t M, int64_t K, int64_t N) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (M <= 0 || K <= 0 || N <= 0 || !bits || !db_prev) return errorf("gt_linear_bwd_data_bits_db: bad arguments");
  GemmShape s{M, K, N, false, false, N, K};
  Epi<float> ef;
  Epi<double> ed;
  ef.out = (float*)dx, ed.out = (double*)dx;
  ef.ldc = ed.ldc = K;
  ef.dbits = ed.dbits = bits;
  ef.ldw = ed.ldw = K;
  return bwd_data_with_db(ctx, dtype, s, dy, w, dx, db_prev, ef, ed, M, K);
}

char* gt_set_gemm_sm_reserve(gt_ctx* ctx, int sms) {
  GT_ENTER(ctx);
  if (sms < 0 || sms > ctx->sm_count - 2) return errorf("gt_set_gemm_sm_reserve: %d of %d SMs", sms, ctx->sm_count);
  ctx->gemm_sm_reserve = sms;
  return nullptr;
}

void gt_debug_set_gemm_path(int path) { set_gemm_path(path); }
void gt_debug_set_gemm_splits(int splits) { set_gemm_splits(splits < 0 ? 0 : splits); }
void gt_debug_set_tc_wait_limit_us(int64_t us) { set_tc_wait_limit_us(us); }
void gt_debug_tc_withhold_arrive(void) { tc_withhold_next_arrive(); }
int gt_gemm_path_taken(void) { return g_gemm_taken; }

char* gt_gemm_timer_start(gt_ctx* ctx, int64_t capacity) {
  GT_ENTER(ctx);
  if (capacity <= 0 || capacity > (1 << 20)) return errorf("gt_gemm_timer_start: capacity %lld out of range",
                                                           (long long)capacity);
  GT_TRY(gt_gemm_timer_stop(ctx));
  auto* t = new gt_gemm_timer();
  t->launches.resize(capacity);
  for (auto& l : t->launches) {
    cudaError_t e1 = cudaEventCreate(&l.start), e2 = cudaEventCreate(&l.end);
    if (e1 != cudaSuccess || e2 != cudaSuccess) {
      ctx->gemm_timer = t;
      gt_free_error(gt_gemm_timer_stop(ctx));
      return cuda_error(e1 != cudaSuccess ? e1 : e2, "cudaEventCreate", __FILE__, __LINE__);
    }
  }
  ctx->gemm_timer = t;
  return nullptr;
}

char* gt_gemm_timer_stop(gt_ctx* ctx) {
  GT_ENTER(ctx);
  gt_gemm_timer* t = ctx->gemm_timer;
  if (!t) return nullptr;
  ctx->gemm_timer = nullptr;
  GT_CUDA(cudaStreamSynchronize(ctx->stream));
  for (auto& l : t->launches) {
    if (l.start) cudaEventDestroy(l.start);
    if (l.end) cudaEventDestroy(l.end);
  }
  delete t;
  return nullptr;
}

char* gt_gemm_timer_count(gt_ctx* ctx, int64_t* launches, int64_t* dropped) {
  GT_ENTER(ctx);
  gt_gemm_timer* t = ctx->gemm_timer;
  if (!t) return errorf("gt_gemm_timer_count: no timer on this context");
  if (launches) *launches = t->used;
  if (dropped) *dropped = t->dropped;
  return nullptr;
}

char* gt_gemm_timer_read(gt_ctx* ctx, int64_t i, int64_t mnk[3], int* path, float* ms) {
  GT_ENTER(ctx);
  gt_gemm_timer* t = ctx->gemm_timer;
  if (!t) return errorf("gt_gemm_timer_read: no timer on this context");
  if (i < 0 || i >= t->used) return errorf("gt_gemm_timer_read: launch %lld of %lld", (long long)i,
                                           (long long)t->used);
  const auto& l = t->launches[i];
  GT_CUDA(cudaEventSynchronize(l.end));
  if (ms) GT_CUDA(cudaEventElapsedTime(ms, l.start, l.end));
  if (mnk) mnk[0] = l.m, mnk[1] = l.n, mnk[2] = l.k;
  if (path) *path = l.path;
  return nullptr;
}

char* gt_matmul(gt_ctx* ctx, int dtype, const void* a, const void* b, void* c, int64_t m, int64_t k, int64_t n,
                int trans_a, int trans_b) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (m < 0 || k < 0 || n < 0) return errorf("gt_matmul: negative size");
  if (m == 0 || n == 0) return nullptr;
  if (k == 0) {  // empty inner dimension: the product is zero
    GT_CUDA(cudaMemsetAsync(c, 0, m * n * (dtype == GT_FLOAT64 ? 8 : 4), ctx->stream));
    return nullptr;
  }
  // C = op(A) @ op(B); B(k, n) = trans_b ? B[n*K + k] : B[k*N + n].
  GemmShape s{m, n, k, trans_a != 0, trans_b != 0, trans_a ? m : k, trans_b ? k : n};
  GT_DISPATCH(dtype, {
    Epi<T> e;
    e.out = (T*)c;
    e.ldc = n;
    return gemm<T>(ctx, s, (const T*)a, (const T*)b, e);
  });
  return nullptr;
}

char* gt_linear_fwd(gt_ctx* ctx, int dtype, const void* x, const void* w, const void* bias, void* y, int64_t M,
                    int64_t K, int64_t N, int act) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (M < 0 || K < 0 || N < 0) return errorf("gt_linear_fwd: negative size");
  if (M == 0 || N == 0) return nullptr;
  // y = x (M, K) @ w (N, K)^T: B(k, n) = w[n*K + k].
  GemmShape s{M, N, K, false, true, K, K};
  GT_DISPATCH(dtype, {
    Epi<T> e;
    e.out = (T*)y;
    e.ldc = N;
    e.bias = (const T*)bias;
    e.act = act;
    if (K == 0) return errorf("gt_linear_fwd: K must be positive");
    return gemm<T>(ctx, s, (const T*)x, (const T*)w, e);
  });
  return nullptr;
}

char* gt_linear_bwd_data(gt_ctx* ctx, int dtype, const void* dy, const void* w, const void* y_prev, int act_prev,
                         void* dx, int64_t M, int64_t K, int64_t N) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (M <= 0 || K <= 0 || N <= 0) return errorf("gt_linear_bwd_data: sizes must be positive");
  // dx (M, K) = dy (M, N) @ w (N, K): B(k=N-index, n=K-index) = w[k*K + n].
  GemmShape s{M, K, N, false, false, N, K};
  GT_DISPATCH(dtype, {
    Epi<T> e;
    e.out = (T*)dx;
    e.ldc = K;
    if (y_prev && act_prev != GT_ACT_NONE) {
      e.dmask = (const T*)y_prev;
      e.dact = act_prev;
      e.ldm = K;
    }
    return gemm<T>(ctx, s, (const T*)dy, (const T*)w, e);
  });
  return nullptr;
}

char* gt_relu_bits(gt_ctx* ctx, int dtype, const void* y, uint32_t* bits, int64_t M, int64_t N) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (M < 0 || N < 0 || (M > 0 && N > 0 && (!y || !bits))) return errorf("gt_relu_bits: bad arguments");
  if (M == 0 || N == 0) return nullptr;
  GT_DISPATCH(dtype, {
    relu_bits_kernel<T><<<grid_for(ctx, (M + 31) / 32 * N, 256), 256, 0, ctx->stream>>>((const T*)y, bits, M, N);
  });
  GT_LAUNCH_CHECK();
  return nullptr;
}

char* gt_linear_fwd_bits(gt_ctx* ctx, int dtype, const void* x, const void* w, const void* bias, void* y,
                         uint32_t* bits, int64_t M, int64_t K, int64_t N) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (M < 0 || K <= 0 || N < 0 || !bits) return errorf("gt_linear_fwd_bits: bad arguments");
  if (M == 0 || N == 0) return nullptr;
  GemmShape s{M, N, K, false, true, K, K};
  bool fused = false;
  GT_DISPATCH(dtype, {
    Epi<T> e;
    e.out = (T*)y;
    e.ldc = N;
    e.bias = (const T*)bias;
    e.act = GT_ACT_RELU;
    e.bits_out = (uint32_t*)bits;
    e.ldw = N;
    GT_TRY(gemm<T>(ctx, s, (const T*)x, (const T*)w, e));
    fused = sizeof(T) == 4 && g_gemm_taken == 2;  // the tcgen05 epilogues wrote the mask
  });
  return fused ? nullptr : gt_relu_bits(ctx, dtype, y, bits, M, N);
}

char* gt_linear_bwd_data_bits(gt_ctx* ctx, int dtype, const void* dy, const void* w, const uint32_t* bits, void* dx,
                              int64_t M, int64_t K, int64_t N) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (M <= 0 || K <= 0 || N <= 0 || !bits) return errorf("gt_linear_bwd_data_bits: bad arguments");
  GemmShape s{M, K, N, false, false, N, K};
  GT_DISPATCH(dtype, {
    Epi<T> e;
    e.out = (T*)dx;
    e.ldc = K;
    e.dbits = bits;
    e.ldw = K;
    return gemm<T>(ctx, s, (const T*)dy, (const T*)w, e);
  });
  return nullptr;
}

char* gt_linear_bwd_weight_rows(gt_ctx* ctx, int dtype, const void* x, const void* dy, void* dw, int64_t M,
                                int64_t K, int64_t N, int64_t r0, int64_t r1) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (M <= 0 || K <= 0 || N <= 0 || r0 < 0 || r1 > N || r0 >= r1)
    return errorf("gt_linear_bwd_weight_rows: bad sizes or row range [%lld, %lld) of %lld", (long long)r0,
                  (long long)r1, (long long)N);
  // dw rows [r0, r1) = dy[:, r0:r1]^T @ x: A(m, k) = dy[k*N + r0 + m], the
  // full row pitch N kept.
  GemmShape s{r1 - r0, K, M, true, false, N, K};
  GT_DISPATCH(dtype, {
    Epi<T> e;
    e.out = (T*)dw + r0 * K;
    e.ldc = K;
    return gemm<T>(ctx, s, (const T*)dy + r0, (const T*)x, e);
  });
  return nullptr;
}

char* gt_linear_bwd_weight(gt_ctx* ctx, int dtype, const void* x, const void* dy, void* dw, void* db, int64_t M,
                           int64_t K, int64_t N) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (M <= 0 || K <= 0 || N <= 0) return errorf("gt_linear_bwd_weight: sizes must be positive");
  // dw (N, K) = dy (M, N)^T @ x (M, K): A(m=N-index, k=M-index) = dy[k*N + m].
  GemmShape s{N, K, M, true, false, N, K};
  GT_DISPATCH(dtype, {
    Epi<T> e;
    e.out = (T*)dw;
    e.ldc = K;
    GT_TRY(gemm<T>(ctx, s, (const T*)dy, (const T*)x, e));
  });
  if (db) GT_TRY(gt_reduce(ctx, dtype, GT_SUM, dy, db, 1, M, N));
  return nullptr;
}

}  // extern "C"
