// Single-pass SGD and Adam updates over flat parameter buffers.
//
// The reference expresses each update as a chain of tensor ops
// (optim/optim.go:48-70 and 110-132), about ten HBM passes per parameter.
// Here one coalesced pass reads p, g (and the state) once and writes p (and
// the state) once: SGD with momentum moves 20 bytes per float32 parameter,
// Adam 28. Each intermediate is rounded exactly where the reference rounds it
// (every op is a separate correctly rounded fp op, no FMA contraction, and
// every scalar is rounded to the dtype as MulScalar/AddScalar do), so given
// the same gradients the updated parameters are bit-identical to the
// reference's.
#include <cmath>

#include "gt_common.cuh"

namespace gt {

template <typename T>
struct SgdScalars {
  T wd, mom, lr;
  bool has_wd, has_mom;
};

template <typename T>
__device__ __forceinline__ void sgd_one(T& p, T g, T& v, const SgdScalars<T>& s, bool first) {
  T d = g;
  if (s.has_wd) d = add_rn(d, mul_rn(p, s.wd));       // d.Add(p.MulScalar(wd))
  if (s.has_mom) {
    v = first ? d : add_rn(mul_rn(v, s.mom), d);       // velocity.MulScalar(m).Add(d)
    d = v;
  }
  p = sub_rn(p, mul_rn(d, s.lr));                      // p.Sub(d.MulScalar(lr))
}

// W elements per thread per iteration; W > 1 uses 16-byte loads and stores
// (every pointer must then be 16-byte aligned).
template <typename T, int W>
struct alignas(sizeof(T) * W) Pack {
  T v[W];
};

template <typename T, int W>
__global__ void sgd_kernel(T* __restrict__ p, const T* __restrict__ g, T* __restrict__ vel, int64_t n,
                           SgdScalars<T> s, int first) {
  const int64_t nv = n / W;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    Pack<T, W> pp = reinterpret_cast<const Pack<T, W>*>(p)[i];
    Pack<T, W> gg = reinterpret_cast<const Pack<T, W>*>(g)[i];
    Pack<T, W> vv;
    if (s.has_mom && !first) vv = reinterpret_cast<const Pack<T, W>*>(vel)[i];
#pragma unroll
    for (int j = 0; j < W; j++) sgd_one(pp.v[j], gg.v[j], vv.v[j], s, first != 0);
    reinterpret_cast<Pack<T, W>*>(p)[i] = pp;
    if (s.has_mom) reinterpret_cast<Pack<T, W>*>(vel)[i] = vv;
  }
  for (int64_t i = nv * W + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    T pv = p[i], vv = s.has_mom && !first ? vel[i] : (T)0;
    sgd_one(pv, g[i], vv, s, first != 0);
    p[i] = pv;
    if (s.has_mom) vel[i] = vv;
  }
}

template <typename T>
struct AdamScalars {
  T wd, b1, omb1, b2, omb2, eps;
  bool has_wd;
};

// One Adam element; inv_bc2 = T(1/bc2), lr_bc1 = T(lr/bc1).
template <typename T>
__device__ __forceinline__ void adam_one(T& p, T g, T& m, T& v, const AdamScalars<T>& s, T inv_bc2, T lr_bc1) {
  if (s.has_wd) g = add_rn(g, mul_rn(p, s.wd));
  m = add_rn(mul_rn(m, s.b1), mul_rn(g, s.omb1));
  v = add_rn(mul_rn(v, s.b2), mul_rn(mul_rn(g, g), s.omb2));
  T denom = add_rn(sqrt_rn(mul_rn(v, inv_bc2)), s.eps);  // Sqrt in float64 then rounded == correctly rounded sqrt
  p = sub_rn(p, div_rn(mul_rn(m, lr_bc1), denom));
}

// One pass over the parameters: each thread loads two groups of W elements of
// p, g, m, v before updating either (more loads in flight per thread). With
// DEV_STEP the bias corrections come from the device-side step counter, read
// once per block; the last block to finish advances the counter (every block
// has read it by then: a block counts itself done only after reading), so a
// captured graph replays the update with no second kernel.
template <typename T, int W, bool DEV_STEP>
__global__ void adam_kernel(T* __restrict__ p, const T* __restrict__ g, T* __restrict__ m, T* __restrict__ v,
                            int64_t n, AdamScalars<T> s, T inv_bc2, T lr_bc1, int64_t* step_dev,
                            unsigned int* blocks_done, double lr, double beta1, double beta2) {
  if (DEV_STEP) {  // bias corrections from the device-side step counter, in float64, once per block
    __shared__ T sc[2];
    if (threadIdx.x == 0) {
      const double t = (double)(*step_dev + 1);
      const double bc1 = 1.0 - pow(beta1, t), bc2 = 1.0 - pow(beta2, t);
      sc[0] = (T)(1.0 / bc2);
      sc[1] = (T)(lr / bc1);
    }
    __syncthreads();
    inv_bc2 = sc[0];
    lr_bc1 = sc[1];
  }
  const int64_t nv = n / W;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  using P = Pack<T, W>;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += 2 * stride) {
    const int64_t i2 = i + stride;
    const bool two = i2 < nv;
    P pp[2], gg[2], mm[2], vv[2];
    pp[0] = reinterpret_cast<const P*>(p)[i], gg[0] = reinterpret_cast<const P*>(g)[i];
    mm[0] = reinterpret_cast<const P*>(m)[i], vv[0] = reinterpret_cast<const P*>(v)[i];
    if (two) {
      pp[1] = reinterpret_cast<const P*>(p)[i2], gg[1] = reinterpret_cast<const P*>(g)[i2];
      mm[1] = reinterpret_cast<const P*>(m)[i2], vv[1] = reinterpret_cast<const P*>(v)[i2];
    }
#pragma unroll
    for (int u = 0; u < 2; u++) {
      if (u == 1 && !two) break;
      const int64_t k = u ? i2 : i;
#pragma unroll
      for (int j = 0; j < W; j++) adam_one(pp[u].v[j], gg[u].v[j], mm[u].v[j], vv[u].v[j], s, inv_bc2, lr_bc1);
      reinterpret_cast<P*>(p)[k] = pp[u];
      reinterpret_cast<P*>(m)[k] = mm[u];
      reinterpret_cast<P*>(v)[k] = vv[u];
    }
  }
  for (int64_t i = nv * W + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    T pv = p[i], mv = m[i], vv = v[i];
    adam_one(pv, g[i], mv, vv, s, inv_bc2, lr_bc1);
    p[i] = pv;
    m[i] = mv;
    v[i] = vv;
  }
  if (DEV_STEP) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();  // this block's read of the step is ordered before its count
      if (atomicAdd(blocks_done, 1u) == gridDim.x - 1) {  // the last block: everyone has read the step
        *step_dev += 1;
        *blocks_done = 0;
      }
    }
  }
}

static bool all_aligned16(const void* a, const void* b, const void* c, const void* d) {
  return (((uintptr_t)a | (uintptr_t)b | (uintptr_t)c | (uintptr_t)d) & 15) == 0;
}

__global__ void step_incr_kernel(int64_t* step) { *step += 1; }

// Threads for an elementwise pass of n elements, W per thread, two groups per
// thread: whole blocks of 256, at most the SMs' resident threads.
static int adam_grid(const gt_ctx* ctx, int64_t n, int W) { return grid_for(ctx, n, 256, 2 * W); }

static char* adam_done_counter(gt_ctx* ctx, unsigned int** out) {
  if (!ctx->adam_done) return errorf("gt_adam_step_dev: the context has no block counter");
  *out = ctx->adam_done;
  return nullptr;
}

template <typename T>
static AdamScalars<T> adam_scalars(const gt_adam_cfg& c) {
  AdamScalars<T> s;
  s.wd = (T)c.weight_decay;
  s.b1 = (T)c.beta1;
  s.omb1 = (T)(1.0 - c.beta1);
  s.b2 = (T)c.beta2;
  s.omb2 = (T)(1.0 - c.beta2);
  s.eps = (T)c.eps;
  s.has_wd = c.weight_decay != 0;
  return s;
}

// Zero config fields take PyTorch's defaults, like optim.NewAdam (optim/optim.go:91-106).
static gt_adam_cfg adam_defaults(const gt_adam_cfg* in) {
  gt_adam_cfg c = *in;
  if (c.lr == 0) c.lr = 1e-3;
  if (c.beta1 == 0) c.beta1 = 0.9;
  if (c.beta2 == 0) c.beta2 = 0.999;
  if (c.eps == 0) c.eps = 1e-8;
  return c;
}

}  // namespace gt

using namespace gt;

extern "C" {

char* gt_sgd_step(gt_ctx* ctx, int dtype, void* p, const void* g, void* vel, int64_t n, const gt_sgd_cfg* cfg,
                  int first) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (!cfg) return errorf("gt_sgd_step: null config");
  if (n <= 0) return nullptr;
  if (cfg->momentum != 0 && !vel) return errorf("gt_sgd_step: momentum needs a velocity buffer");
  GT_DISPATCH(dtype, {
    SgdScalars<T> s{(T)cfg->weight_decay, (T)cfg->momentum, (T)cfg->lr, cfg->weight_decay != 0, cfg->momentum != 0};
    constexpr int W = 16 / sizeof(T);
    if (all_aligned16(p, g, vel ? vel : p, p))
      sgd_kernel<T, W><<<grid_for(ctx, n, 256, W), 256, 0, ctx->stream>>>((T*)p, (const T*)g, (T*)vel, n, s, first);
    else
      sgd_kernel<T, 1><<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>((T*)p, (const T*)g, (T*)vel, n, s, first);
  });
  GT_LAUNCH_CHECK();
  return nullptr;
}

char* gt_adam_step(gt_ctx* ctx, int dtype, void* p, const void* g, void* m, void* v, int64_t n,
                   const gt_adam_cfg* cfg_in, int64_t step) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (!cfg_in) return errorf("gt_adam_step: null config");
  if (step < 1) return errorf("gt_adam_step: step must be >= 1");
  if (n <= 0) return nullptr;
  gt_adam_cfg c = adam_defaults(cfg_in);
  double bc1 = 1.0 - std::pow(c.beta1, (double)step), bc2 = 1.0 - std::pow(c.beta2, (double)step);
  GT_DISPATCH(dtype, {
    constexpr int W = 16 / sizeof(T);
    if (all_aligned16(p, g, m, v))
      adam_kernel<T, W, false><<<adam_grid(ctx, n, W), 256, 0, ctx->stream>>>(
          (T*)p, (const T*)g, (T*)m, (T*)v, n, adam_scalars<T>(c), (T)(1.0 / bc2), (T)(c.lr / bc1), nullptr, nullptr,
          c.lr, c.beta1, c.beta2);
    else
      adam_kernel<T, 1, false><<<adam_grid(ctx, n, 1), 256, 0, ctx->stream>>>(
          (T*)p, (const T*)g, (T*)m, (T*)v, n, adam_scalars<T>(c), (T)(1.0 / bc2), (T)(c.lr / bc1), nullptr, nullptr,
          c.lr, c.beta1, c.beta2);
  });
  GT_LAUNCH_CHECK();
  return nullptr;
}

char* gt_adam_step_dev(gt_ctx* ctx, int dtype, void* p, const void* g, void* m, void* v, int64_t n,
                       const gt_adam_cfg* cfg_in, int64_t* step_dev) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  if (!cfg_in || !step_dev) return errorf("gt_adam_step_dev: null argument");
  gt_adam_cfg c = adam_defaults(cfg_in);
  if (n <= 0) {
    step_incr_kernel<<<1, 1, 0, ctx->stream>>>(step_dev);
    GT_LAUNCH_CHECK();
    return nullptr;
  }
  // blocks_done: a counter the kernel's last block resets to zero, so it
  // starts every launch at zero; one per context, shared by every update on
  // its stream (which run one after another).
  unsigned int* done = nullptr;
  GT_TRY(adam_done_counter(ctx, &done));
  GT_DISPATCH(dtype, {
    constexpr int W = 16 / sizeof(T);
    if (all_aligned16(p, g, m, v))
      adam_kernel<T, W, true><<<adam_grid(ctx, n, W), 256, 0, ctx->stream>>>(
          (T*)p, (const T*)g, (T*)m, (T*)v, n, adam_scalars<T>(c), (T)0, (T)0, step_dev, done, c.lr, c.beta1,
          c.beta2);
    else
      adam_kernel<T, 1, true><<<adam_grid(ctx, n, 1), 256, 0, ctx->stream>>>(
          (T*)p, (const T*)g, (T*)m, (T*)v, n, adam_scalars<T>(c), (T)0, (T)0, step_dev, done, c.lr, c.beta1,
          c.beta2);
  });
  GT_LAUNCH_CHECK();
  return nullptr;
}

}  // extern "C"
