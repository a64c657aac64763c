// Element-wise primitives: Backend.Unary/Binary/Copy/Cast
// (internal/backend/backend.go:136-144), restated from internal/cpu/cpu.go.
//
// All are HBM-bound. Contiguous operands take a vectorized path (16-byte
// loads and stores, grid-stride over a grid sized to the SM count); strided
// views are first coalesced on the host (adjacent dimensions that are
// contiguous in every operand are merged), so the common broadcasts reach the
// kernel as one or two dimensions.
#include "gt_common.cuh"

namespace gt {

struct Strided {
  int ndim;
  int nops;
  int64_t shape[GT_MAX_DIMS];
  int64_t stride[2][GT_MAX_DIMS];
  int64_t offset[2];
};

// Merges adjacent dimensions that are laid out contiguously in every operand.
static Strided coalesce(const int64_t* shape, int ndim, const gt_view* const* views, int nops) {
  Strided s{};
  s.nops = nops;
  for (int o = 0; o < nops; o++) s.offset[o] = views[o]->offset;
  // Walk from the innermost dimension outwards; drop size-1 dimensions.
  int nd = 0;
  int64_t sh[GT_MAX_DIMS], st[2][GT_MAX_DIMS];
  for (int d = ndim - 1; d >= 0; d--) {
    if (shape[d] == 1) continue;
    if (nd > 0) {
      bool merge = true;
      for (int o = 0; o < nops; o++)
        if (views[o]->strides[d] != st[o][nd - 1] * sh[nd - 1]) merge = false;
      if (merge) {
        sh[nd - 1] *= shape[d];
        continue;
      }
    }
    sh[nd] = shape[d];
    for (int o = 0; o < nops; o++) st[o][nd] = views[o]->strides[d];
    nd++;
  }
  if (nd == 0) {  // a single element
    sh[0] = 1;
    for (int o = 0; o < nops; o++) st[o][0] = 0;
    nd = 1;
  }
  s.ndim = nd;
  for (int d = 0; d < nd; d++) {  // back to outermost-first order
    s.shape[d] = sh[nd - 1 - d];
    for (int o = 0; o < nops; o++) s.stride[o][d] = st[o][nd - 1 - d];
  }
  return s;
}

static bool is_contiguous(const gt_view* v) {
  if (v->offset != 0) return false;
  int64_t s = 1;
  for (int d = v->ndim - 1; d >= 0; d--) {
    if (v->shape[d] != 1 && v->strides[d] != s) return false;
    s *= v->shape[d];
  }
  return true;
}

static int64_t view_numel(const gt_view* v) {
  int64_t n = 1;
  for (int d = 0; d < v->ndim; d++) n *= v->shape[d];
  return n;
}

template <typename T>
struct UnaryF {
  int op;
  double s;
  T c;
  __device__ __forceinline__ T operator()(T v) const {
    switch (op) {
      case GT_NEG: return -v;
      case GT_EXP: return (T)exp((double)v);
      case GT_LOG: return (T)log((double)v);
      case GT_SQRT: return (T)sqrt((double)v);
      case GT_ABS: return (T)fabs((double)v);
      case GT_RELU: return go_max(v, (T)0);
      case GT_SIGMOID: return (T)(1.0 / (1.0 + exp(-(double)v)));
      case GT_TANH: return (T)tanh((double)v);
      case GT_SIGN: return v > (T)0 ? (T)1 : (v < (T)0 ? (T)-1 : (T)0);
      case GT_STEP: return v > (T)0 ? (T)1 : (T)0;
      case GT_ADD_SCALAR: return add_rn(v, c);
      case GT_MUL_SCALAR: return mul_rn(v, c);
      default: return (T)pow((double)v, s);
    }
  }
};

template <typename T>
struct BinaryF {
  int op;
  __device__ __forceinline__ T operator()(T a, T b) const {
    switch (op) {
      case GT_ADD: return add_rn(a, b);
      case GT_SUB: return sub_rn(a, b);
      case GT_MUL: return mul_rn(a, b);
      default: return div_rn(a, b);
    }
  }
};

template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
  using type = float4;
  static constexpr int n = 4;
};
template <>
struct Vec16<double> {
  using type = double2;
  static constexpr int n = 2;
};

template <typename T>
__device__ __forceinline__ T& lane(typename Vec16<T>::type& v, int i) {
  return reinterpret_cast<T*>(&v)[i];
}

// y = f(x) over n contiguous elements; VEC selects 16-byte accesses.
template <typename T, bool VEC, typename F>
__global__ void map1_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n, F f) {
  int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, step = (int64_t)gridDim.x * blockDim.x;
  if (VEC) {
    using V = typename Vec16<T>::type;
    constexpr int W = Vec16<T>::n;
    int64_t nv = n / W;
    const V* xv = reinterpret_cast<const V*>(x);
    V* yv = reinterpret_cast<V*>(y);
    for (int64_t i = tid; i < nv; i += step) {
      V v = xv[i];
#pragma unroll
      for (int j = 0; j < W; j++) lane<T>(v, j) = f(lane<T>(v, j));
      yv[i] = v;
    }
    for (int64_t i = nv * W + tid; i < n; i += step) y[i] = f(x[i]);
  } else {
    for (int64_t i = tid; i < n; i += step) y[i] = f(x[i]);
  }
}

template <typename T, bool VEC, typename F>
__global__ void map2_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y, int64_t n, F f) {
  int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, step = (int64_t)gridDim.x * blockDim.x;
  if (VEC) {
    using V = typename Vec16<T>::type;
    constexpr int W = Vec16<T>::n;
    int64_t nv = n / W;
    const V* av = reinterpret_cast<const V*>(a);
    const V* bv = reinterpret_cast<const V*>(b);
    V* yv = reinterpret_cast<V*>(y);
    for (int64_t i = tid; i < nv; i += step) {
      V p = av[i], q = bv[i];
#pragma unroll
      for (int j = 0; j < W; j++) lane<T>(p, j) = f(lane<T>(p, j), lane<T>(q, j));
      yv[i] = p;
    }
    for (int64_t i = nv * W + tid; i < n; i += step) y[i] = f(a[i], b[i]);
  } else {
    for (int64_t i = tid; i < n; i += step) y[i] = f(a[i], b[i]);
  }
}

__device__ __forceinline__ void strided_offsets(const Strided& s, int64_t i, int64_t* off) {
  off[0] = s.offset[0];
  off[1] = s.offset[1];
  for (int d = s.ndim - 1; d >= 0; d--) {
    int64_t sz = s.shape[d];
    int64_t q = i / sz, r = i - q * sz;
    i = q;
    off[0] += r * s.stride[0][d];
    off[1] += r * s.stride[1][d];
  }
}

template <typename T>
__global__ void binary_strided_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y,
                                      int64_t n, Strided s, BinaryF<T> f) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t off[2];
    strided_offsets(s, i, off);
    y[i] = f(a[off[0]], b[off[1]]);
  }
}

template <typename T>
__global__ void gather_kernel(const T* __restrict__ src, T* __restrict__ y, int64_t n, Strided s) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t off[2];
    strided_offsets(s, i, off);
    y[i] = src[off[0]];
  }
}

template <typename S, typename D>
__global__ void cast_kernel(const S* __restrict__ x, D* __restrict__ y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = (D)x[i];
}

template <typename T>
struct ActBwdF {
  int act;
  __device__ __forceinline__ T operator()(T g, T y) const { return act_bwd(act, g, y); }
};

template <typename T>
__global__ void bias_act_kernel(T* __restrict__ y, const T* __restrict__ bias, int64_t total, int64_t C, int64_t L,
                                int act) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    T v = y[i];
    if (bias) v = add_rn(v, bias[(i / L) % C]);
    y[i] = act_fwd(act, v);
  }
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <typename T, typename F>
static char* launch_map1(gt_ctx* ctx, const T* x, T* y, int64_t n, F f) {
  if (n <= 0) return nullptr;
  const int threads = 256;
  if (aligned16(x) && aligned16(y)) {
    map1_kernel<T, true><<<grid_for(ctx, n, threads, 16 / sizeof(T)), threads, 0, ctx->stream>>>(x, y, n, f);
  } else {
    map1_kernel<T, false><<<grid_for(ctx, n, threads), threads, 0, ctx->stream>>>(x, y, n, f);
  }
  GT_LAUNCH_CHECK();
  return nullptr;
}

template <typename T, typename F>
static char* launch_map2(gt_ctx* ctx, const T* a, const T* b, T* y, int64_t n, F f) {
  if (n <= 0) return nullptr;
  const int threads = 256;
  if (aligned16(a) && aligned16(b) && aligned16(y)) {
    map2_kernel<T, true><<<grid_for(ctx, n, threads, 16 / sizeof(T)), threads, 0, ctx->stream>>>(a, b, y, n, f);
  } else {
    map2_kernel<T, false><<<grid_for(ctx, n, threads), threads, 0, ctx->stream>>>(a, b, y, n, f);
  }
  GT_LAUNCH_CHECK();
  return nullptr;
}

static char* check_view(const gt_view* v, const char* what) {
  if (!v) return errorf("%s: null view", what);
  if (v->ndim < 0 || v->ndim > GT_MAX_DIMS) return errorf("%s: %d dimensions (at most %d)", what, v->ndim, GT_MAX_DIMS);
  for (int d = 0; d < v->ndim; d++)
    if (v->shape[d] < 0) return errorf("%s: negative dimension", what);
  return nullptr;
}

}  // namespace gt

using namespace gt;

extern "C" {

char* gt_unary(gt_ctx* ctx, int dtype, int op, double s, const void* x, void* y, int64_t n) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (op < GT_NEG || op > GT_POW) return errorf("gt_unary: unknown op %d", op);
  GT_DISPATCH(dtype, {
    UnaryF<T> f{op, s, (T)s};
    return launch_map1<T>(ctx, (const T*)x, (T*)y, n, f);
  });
  return nullptr;
}

char* gt_binary(gt_ctx* ctx, int dtype, int op, const void* a, const gt_view* va, const void* b, const gt_view* vb,
                void* out) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_view(va, "gt_binary"));
  GT_TRY(check_view(vb, "gt_binary"));
  if (op < GT_ADD || op > GT_DIV) return errorf("gt_binary: unknown op %d", op);
  if (va->ndim != vb->ndim) return errorf("gt_binary: views have %d and %d dimensions", va->ndim, vb->ndim);
  for (int d = 0; d < va->ndim; d++)
    if (va->shape[d] != vb->shape[d]) return errorf("gt_binary: view shapes differ in dimension %d", d);
  int64_t n = view_numel(va);
  if (n == 0) return nullptr;
  GT_DISPATCH(dtype, {
    BinaryF<T> f{op};
    if (is_contiguous(va) && is_contiguous(vb)) return launch_map2<T>(ctx, (const T*)a, (const T*)b, (T*)out, n, f);
    const gt_view* vs[2] = {va, vb};
    Strided s = coalesce(va->shape, va->ndim, vs, 2);
    binary_strided_kernel<T><<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>((const T*)a, (const T*)b, (T*)out, n, s, f);
    GT_LAUNCH_CHECK();
  });
  return nullptr;
}

char* gt_copy(gt_ctx* ctx, int dtype, const void* src, const gt_view* v, void* out) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_view(v, "gt_copy"));
  int64_t n = view_numel(v);
  if (n == 0) return nullptr;
  size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  gt_view base = *v;
  base.offset = 0;
  if (is_contiguous(&base)) {  // a plain slice starting at v->offset
    GT_CUDA(cudaMemcpyAsync(out, (const char*)src + v->offset * es, n * es, cudaMemcpyDeviceToDevice, ctx->stream));
    return nullptr;
  }
  GT_DISPATCH(dtype, {
    const gt_view* vs[1] = {v};
    Strided s = coalesce(v->shape, v->ndim, vs, 1);
    gather_kernel<T><<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>((const T*)src, (T*)out, n, s);
    GT_LAUNCH_CHECK();
  });
  return nullptr;
}

char* gt_cast(gt_ctx* ctx, const void* x, int from_dtype, void* y, int to_dtype, int64_t n) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(from_dtype);
  GT_CHECK_DTYPE(to_dtype);
  if (n <= 0) return nullptr;
  if (from_dtype == to_dtype) {
    GT_CUDA(cudaMemcpyAsync(y, x, n * (from_dtype == GT_FLOAT64 ? 8 : 4), cudaMemcpyDeviceToDevice, ctx->stream));
    return nullptr;
  }
  if (from_dtype == GT_FLOAT32)
    cast_kernel<float, double><<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>((const float*)x, (double*)y, n);
  else
    cast_kernel<double, float><<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>((const double*)x, (float*)y, n);
  GT_LAUNCH_CHECK();
  return nullptr;
}

char* gt_act_bwd(gt_ctx* ctx, int dtype, int act, const void* dy, const void* y, void* dx, int64_t n) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_DISPATCH(dtype, { return launch_map2<T>(ctx, (const T*)dy, (const T*)y, (T*)dx, n, ActBwdF<T>{act}); });
  return nullptr;
}

char* gt_bias_act(gt_ctx* ctx, int dtype, void* y, const void* bias, int64_t N, int64_t C, int64_t L, int act) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  int64_t total = N * C * L;
  if (total <= 0) return nullptr;
  GT_DISPATCH(dtype, {
    bias_act_kernel<T><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>((T*)y, (const T*)bias, total, C, L, act);
    GT_LAUNCH_CHECK();
  });
  return nullptr;
}

}  // extern "C"
