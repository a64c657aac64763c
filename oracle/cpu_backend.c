/*
 * ORACLE — test infrastructure only. Not part of the product.
 *
 * A C restatement of go-tensor's pure-Go CPU backend, the reference
 * implementation every device backend is checked against. It follows the
 * reference op for op:
 *
 *   internal/cpu/cpu.go:103-167   unary (transcendentals computed in float64,
 *                                 then rounded to T; scalars rounded to T)
 *   internal/cpu/cpu.go:169-231   binary with broadcast views (contiguous fast
 *                                 path + odometer walk)
 *   internal/cpu/cpu.go:233-244   contiguous()
 *   internal/cpu/cpu.go:246-268   gather (Copy)
 *   internal/cpu/cpu.go:270-296   reduce over the middle axis, sequential
 *                                 accumulation in T, Go max() semantics
 *   internal/cpu/linalg.go:15-62  matmulT / matmul: transposes materialized,
 *                                 i-k-j loop folding four rows of b per pass,
 *                                 accumulation in T
 *   internal/cpu/linalg.go:65-81  parallelRows: row split over worker threads
 *                                 above 2^16 multiply-adds
 *   internal/cpu/linalg.go:84-92  transpose2d
 *   internal/cpu/linalg.go:94-146 im2col / col2im / eachPatch
 *   internal/cpu/linalg.go:148-191 maxPool forward and first-max backward
 *
 * Build with -ffp-contract=off: Go on amd64 rounds every multiply and add
 * separately (no FMA fusion), and so must this restatement.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * the shared library built from this file.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OC_MAXDIMS 8

typedef struct {
  int32_t ndim;
  int32_t _pad;
  int64_t offset;
  int64_t shape[OC_MAXDIMS];
  int64_t strides[OC_MAXDIMS];
} oc_view;

typedef struct {
  int64_t N, C, H, W, KH, KW, OH, OW, stride, pad;
} oc_geom;

/* Op codes follow internal/backend/backend.go:72-106. */
enum { U_NEG, U_EXP, U_LOG, U_SQRT, U_ABS, U_RELU, U_SIGMOID, U_TANH, U_SIGN, U_STEP,
       U_ADD_SCALAR, U_MUL_SCALAR, U_POW };
enum { B_ADD, B_SUB, B_MUL, B_DIV };
enum { R_SUM, R_MAX };

/* Go's builtin max for floats (Go spec, "Min and max"): NaN wins, and
 * max(-0.0, +0.0) is +0.0. */
static inline double go_max_d(double a, double b) {
  if (isnan(a) || isnan(b)) return NAN;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
static inline float go_max_f(float a, float b) {
  if (isnan(a) || isnan(b)) return NAN;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}

static int64_t numel(const oc_view* v) {
  int64_t n = 1;
  for (int d = 0; d < v->ndim; d++) n *= v->shape[d];
  return n;
}

/* internal/cpu/cpu.go:233-244 */
static int contiguous(const oc_view* v) {
  if (v->offset != 0) return 0;
  int64_t s = 1;
  for (int d = v->ndim - 1; d >= 0; d--) {
    if (v->shape[d] != 1 && v->strides[d] != s) return 0;
    s *= v->shape[d];
  }
  return 1;
}

/* ---- generic kernels, instantiated for float (f32) and double (f64) ---- */

#define DEFINE_KERNELS(T, SFX, MAXF)                                                          \
  void oc_unary_##SFX(int op, double s, const T* x, T* y, int64_t n) {                       \
    int64_t i;                                                                                \
    T c = (T)s;                                                                               \
    switch (op) {                                                                             \
      case U_NEG: for (i = 0; i < n; i++) y[i] = -x[i]; break;                                \
      case U_EXP: for (i = 0; i < n; i++) y[i] = (T)exp((double)x[i]); break;                 \
      case U_LOG: for (i = 0; i < n; i++) y[i] = (T)log((double)x[i]); break;                 \
      case U_SQRT: for (i = 0; i < n; i++) y[i] = (T)sqrt((double)x[i]); break;               \
      case U_ABS: for (i = 0; i < n; i++) y[i] = (T)fabs((double)x[i]); break;                \
      case U_RELU: for (i = 0; i < n; i++) y[i] = MAXF(x[i], (T)0); break;                    \
      case U_SIGMOID:                                                                         \
        for (i = 0; i < n; i++) y[i] = (T)(1.0 / (1.0 + exp(-(double)x[i])));                 \
        break;                                                                                \
      case U_TANH: for (i = 0; i < n; i++) y[i] = (T)tanh((double)x[i]); break;               \
      case U_SIGN:                                                                            \
        for (i = 0; i < n; i++) y[i] = x[i] > 0 ? (T)1 : (x[i] < 0 ? (T)-1 : (T)0);           \
        break;                                                                                \
      case U_STEP: for (i = 0; i < n; i++) y[i] = x[i] > 0 ? (T)1 : (T)0; break;              \
      case U_ADD_SCALAR: for (i = 0; i < n; i++) y[i] = x[i] + c; break;                      \
      case U_MUL_SCALAR: for (i = 0; i < n; i++) y[i] = x[i] * c; break;                      \
      case U_POW: for (i = 0; i < n; i++) y[i] = (T)pow((double)x[i], s); break;              \
      default: break;                                                                         \
    }                                                                                         \
  }                                                                                           \
                                                                                              \
  static inline T binop_##SFX(int op, T x, T y) {                                             \
    switch (op) {                                                                             \
      case B_ADD: return x + y;                                                               \
      case B_SUB: return x - y;                                                               \
      case B_MUL: return x * y;                                                               \
      default: return x / y;                                                                  \
    }                                                                                         \
  }                                                                                           \
                                                                                              \
  void oc_binary_##SFX(int op, const T* a, const oc_view* av, const T* b, const oc_view* bv, \
                       T* out) {                                                              \
    int64_t n = numel(av), k;                                                                 \
    if (contiguous(av) && contiguous(bv)) {                                                   \
      for (k = 0; k < n; k++) out[k] = binop_##SFX(op, a[k], b[k]);                           \
      return;                                                                                 \
    }                                                                                         \
    int64_t idx[OC_MAXDIMS] = {0};                                                            \
    int64_t ia = av->offset, ib = bv->offset;                                                 \
    for (k = 0; k < n; k++) {                                                                 \
      out[k] = binop_##SFX(op, a[ia], b[ib]);                                                 \
      for (int d = av->ndim - 1; d >= 0; d--) {                                               \
        idx[d]++;                                                                             \
        ia += av->strides[d];                                                                 \
        ib += bv->strides[d];                                                                 \
        if (idx[d] < av->shape[d]) break;                                                     \
        ia -= av->strides[d] * av->shape[d];                                                  \
        ib -= bv->strides[d] * av->shape[d];                                                  \
        idx[d] = 0;                                                                           \
      }                                                                                       \
    }                                                                                         \
  }                                                                                           \
                                                                                              \
  void oc_copy_##SFX(const T* src, const oc_view* v, T* out) {                                \
    int64_t n = numel(v), k;                                                                  \
    int64_t idx[OC_MAXDIMS] = {0};                                                            \
    int64_t off = v->offset;                                                                  \
    for (k = 0; k < n; k++) {                                                                 \
      out[k] = src[off];                                                                      \
      for (int d = v->ndim - 1; d >= 0; d--) {                                                \
        idx[d]++;                                                                             \
        off += v->strides[d];                                                                 \
        if (idx[d] < v->shape[d]) break;                                                      \
        off -= v->strides[d] * v->shape[d];                                                   \
        idx[d] = 0;                                                                           \
      }                                                                                       \
    }                                                                                         \
  }                                                                                           \
                                                                                              \
  void oc_reduce_##SFX(int op, const T* x, T* out, int64_t outer, int64_t n, int64_t inner) { \
    for (int64_t o = 0; o < outer; o++) {                                                     \
      T* dst = out + o * inner;                                                               \
      if (op == R_MAX) {                                                                      \
        memcpy(dst, x + o * n * inner, sizeof(T) * (size_t)inner);                            \
      } else {                                                                                \
        memset(dst, 0, sizeof(T) * (size_t)inner);                                            \
      }                                                                                       \
      for (int64_t k = 0; k < n; k++) {                                                       \
        const T* src = x + (o * n + k) * inner;                                               \
        if (op == R_MAX) {                                                                    \
          for (int64_t i = 0; i < inner; i++) dst[i] = MAXF(dst[i], src[i]);                  \
        } else {                                                                              \
          for (int64_t i = 0; i < inner; i++) dst[i] += src[i];                               \
        }                                                                                     \
      }                                                                                       \
    }                                                                                         \
  }                                                                                           \
                                                                                              \
  static void transpose2d_##SFX(const T* a, T* out, int64_t r, int64_t c) {                   \
    for (int64_t i = 0; i < r; i++)                                                           \
      for (int64_t j = 0; j < c; j++) out[j * r + i] = a[i * c + j];                          \
  }                                                                                           \
                                                                                              \
  typedef struct {                                                                            \
    const T *a, *b;                                                                           \
    T* c;                                                                                     \
    int64_t k, n, lo, hi;                                                                     \
  } rows_arg_##SFX;                                                                           \
                                                                                              \
  static void* matmul_rows_##SFX(void* p) {                                                   \
    rows_arg_##SFX* r = (rows_arg_##SFX*)p;                                                   \
    const T *a = r->a, *b = r->b;                                                             \
    int64_t k = r->k, n = r->n;                                                               \
    for (int64_t i = r->lo; i < r->hi; i++) {                                                 \
      T* ci = r->c + i * n;                                                                   \
      const T* ai = a + i * k;                                                                \
      int64_t p = 0;                                                                          \
      for (; p + 4 <= k; p += 4) {                                                            \
        T a0 = ai[p], a1 = ai[p + 1], a2 = ai[p + 2], a3 = ai[p + 3];                         \
        const T *b0 = b + p * n, *b1 = b + (p + 1) * n, *b2 = b + (p + 2) * n,                \
                *b3 = b + (p + 3) * n;                                                        \
        for (int64_t j = 0; j < n; j++) {                                                     \
          T t = a0 * b0[j];                                                                   \
          t = t + a1 * b1[j];                                                                 \
          t = t + a2 * b2[j];                                                                 \
          t = t + a3 * b3[j];                                                                 \
          ci[j] = ci[j] + t;                                                                  \
        }                                                                                     \
      }                                                                                       \
      for (; p < k; p++) {                                                                    \
        T aip = ai[p];                                                                        \
        const T* bp = b + p * n;                                                              \
        for (int64_t j = 0; j < n; j++) ci[j] = ci[j] + aip * bp[j];                          \
      }                                                                                       \
    }                                                                                         \
    return NULL;                                                                              \
  }                                                                                           \
                                                                                              \
  /* threads plays the role of runtime.GOMAXPROCS(0). */                                      \
  void oc_matmul_##SFX(const T* a, const T* b, T* c, int64_t m, int64_t k, int64_t n, int ta, \
                       int tb, int threads) {                                                 \
    T *at = NULL, *bt = NULL;                                                                 \
    if (ta) {                                                                                 \
      at = (T*)malloc(sizeof(T) * (size_t)(m * k + 1));                                       \
      transpose2d_##SFX(a, at, k, m);                                                         \
      a = at;                                                                                 \
    }                                                                                         \
    if (tb) {                                                                                 \
      bt = (T*)malloc(sizeof(T) * (size_t)(k * n + 1));                                       \
      transpose2d_##SFX(b, bt, n, k);                                                         \
      b = bt;                                                                                 \
    }                                                                                         \
    memset(c, 0, sizeof(T) * (size_t)(m * n));                                                \
    int64_t workers = threads < m ? threads : m;                                              \
    if (m * k * n < (1 << 16) || workers <= 1) {                                              \
      rows_arg_##SFX r = {a, b, c, k, n, 0, m};                                               \
      matmul_rows_##SFX(&r);                                                                  \
    } else {                                                                                  \
      int64_t chunk = (m + workers - 1) / workers;                                            \
      int64_t nt = (m + chunk - 1) / chunk;                                                   \
      pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nt);                     \
      rows_arg_##SFX* args = (rows_arg_##SFX*)malloc(sizeof(rows_arg_##SFX) * (size_t)nt);    \
      for (int64_t t = 0; t < nt; t++) {                                                      \
        int64_t lo = t * chunk, hi = lo + chunk < m ? lo + chunk : m;                         \
        rows_arg_##SFX r = {a, b, c, k, n, lo, hi};                                           \
        args[t] = r;                                                                          \
        pthread_create(&th[t], NULL, matmul_rows_##SFX, &args[t]);                            \
      }                                                                                       \
      for (int64_t t = 0; t < nt; t++) pthread_join(th[t], NULL);                             \
      free(th);                                                                               \
      free(args);                                                                             \
    }                                                                                         \
    free(at);                                                                                 \
    free(bt);                                                                                 \
  }                                                                                           \
                                                                                              \
  /* internal/cpu/linalg.go:122-146: eachPatch drives im2col (assign) and col2im (+=). */     \
  static void each_patch_##SFX(const oc_geom* g, const T* src, T* dst, int to_cols) {         \
    int64_t k = g->C * g->KH * g->KW, row = 0;                                                \
    for (int64_t nn = 0; nn < g->N; nn++)                                                     \
      for (int64_t oh = 0; oh < g->OH; oh++)                                                  \
        for (int64_t ow = 0; ow < g->OW; ow++) {                                              \
          int64_t idx = row * k;                                                              \
          for (int64_t c = 0; c < g->C; c++) {                                                \
            int64_t plane = (nn * g->C + c) * g->H;                                           \
            for (int64_t kh = 0; kh < g->KH; kh++) {                                          \
              int64_t ih = oh * g->stride - g->pad + kh;                                      \
              for (int64_t kw = 0; kw < g->KW; kw++) {                                        \
                int64_t iw = ow * g->stride - g->pad + kw;                                    \
                if (ih >= 0 && ih < g->H && iw >= 0 && iw < g->W) {                           \
                  int64_t xi = (plane + ih) * g->W + iw;                                      \
                  if (to_cols)                                                                \
                    dst[idx] = src[xi];                                                       \
                  else                                                                        \
                    dst[xi] = dst[xi] + src[idx];                                             \
                }                                                                             \
                idx++;                                                                        \
              }                                                                               \
            }                                                                                 \
          }                                                                                   \
          row++;                                                                              \
        }                                                                                     \
  }                                                                                           \
                                                                                              \
  void oc_im2col_##SFX(const T* x, T* cols, const oc_geom* g) {                               \
    memset(cols, 0, sizeof(T) * (size_t)(g->N * g->OH * g->OW * g->C * g->KH * g->KW));       \
    each_patch_##SFX(g, x, cols, 1);                                                          \
  }                                                                                           \
                                                                                              \
  void oc_col2im_##SFX(const T* cols, T* x, const oc_geom* g) {                               \
    memset(x, 0, sizeof(T) * (size_t)(g->N * g->C * g->H * g->W));                            \
    each_patch_##SFX(g, cols, x, 0);                                                          \
  }                                                                                           \
                                                                                              \
  /* internal/cpu/linalg.go:160-191; grad == NULL selects the forward pass. */                \
  void oc_maxpool_##SFX(const T* x, const T* grad, T* out, const oc_geom* g) {                \
    int64_t planes = g->N * g->C, i = 0;                                                      \
    if (grad) memset(out, 0, sizeof(T) * (size_t)(planes * g->H * g->W));                     \
    for (int64_t pl = 0; pl < planes; pl++) {                                                 \
      int64_t base = pl * g->H * g->W;                                                        \
      for (int64_t oh = 0; oh < g->OH; oh++)                                                  \
        for (int64_t ow = 0; ow < g->OW; ow++) {                                              \
          T best = (T)(-INFINITY);                                                            \
          int64_t best_idx = -1;                                                              \
          for (int64_t kh = 0; kh < g->KH; kh++)                                              \
            for (int64_t kw = 0; kw < g->KW; kw++) {                                          \
              int64_t idx = base + (oh * g->stride + kh) * g->W + ow * g->stride + kw;        \
              T v = x[idx];                                                                   \
              if (v > best || best_idx < 0) {                                                 \
                best = v;                                                                     \
                best_idx = idx;                                                               \
              }                                                                               \
            }                                                                                 \
          if (!grad)                                                                          \
            out[i] = best;                                                                    \
          else                                                                                \
            out[best_idx] = out[best_idx] + grad[i];                                          \
          i++;                                                                                \
        }                                                                                     \
    }                                                                                         \
  }

DEFINE_KERNELS(float, f32, go_max_f)
DEFINE_KERNELS(double, f64, go_max_d)

/* internal/cpu/cpu.go:75-90 */
void oc_cast_f32_f64(const float* x, double* y, int64_t n) {
  for (int64_t i = 0; i < n; i++) y[i] = (double)x[i];
}
void oc_cast_f64_f32(const double* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; i++) y[i] = (float)x[i];
}
