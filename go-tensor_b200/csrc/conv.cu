// Convolution helpers and pooling: Backend.Im2col/Col2im/MaxPool2d/
// MaxPool2dBackward (internal/backend/backend.go:152-156), restated from
// internal/cpu/linalg.go:94-191, plus the fused Conv2d and pool-with-argmax
// entry points.
//
// The reference scatters (col2im adds every patch entry into the input;
// the pool backward adds every window's gradient into its first maximum).
// Here each output element gathers instead, visiting its contributions in the
// same order the reference adds them, so both are bit-exact and need no
// atomics.
#include <algorithm>

#include "gemm.cuh"

namespace gt {

// cols[(n*OH + oh)*OW + ow][(c*KH + kh)*KW + kw] = x[n][c][ih][iw] or 0.
template <typename T>
__global__ void im2col_kernel(const T* __restrict__ x, T* __restrict__ cols, gt_geom g, int64_t total) {
  const int64_t K = g.C * g.KH * g.KW;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t row = e / K, k = e - row * K;
    int64_t ow = row % g.OW, t = row / g.OW;
    int64_t oh = t % g.OH, n = t / g.OH;
    int64_t kw = k % g.KW, t2 = k / g.KW;
    int64_t kh = t2 % g.KH, c = t2 / g.KH;
    int64_t ih = oh * g.stride - g.pad + kh, iw = ow * g.stride - g.pad + kw;
    T v = (T)0;
    if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W) v = x[((n * g.C + c) * g.H + ih) * g.W + iw];
    cols[e] = v;
  }
}

// x[n][c][ih][iw] = sum over the patches (oh, ow) that read it, in row order.
// The same, one warp per row of cols: the row's (n, oh, ow) is decoded once
// and each (c, kh, kw) comes from a table in shared memory, so no element
// pays for divisions, and a row's K values are written contiguously.
// 32-bit arithmetic: the host uses it only when every index fits.
template <typename T>
__global__ void im2col_rows_kernel(const T* __restrict__ x, T* __restrict__ cols, gt_geom g64, int rows, int K) {
  extern __shared__ int2 ktab[];  // (offset of (c, kh, kw) in the image, kh << 16 | kw)
  const int C = (int)g64.C, H = (int)g64.H, W = (int)g64.W, KH = (int)g64.KH, KW = (int)g64.KW;
  const int OH = (int)g64.OH, OW = (int)g64.OW, stride = (int)g64.stride, pad = (int)g64.pad;
  const int KHW = KH * KW, HW = H * W, OHW = OH * OW;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const int c = k / KHW, r = k - c * KHW, kh = r / KW, kw = r - kh * KW;
    ktab[k] = make_int2(c * HW + kh * W + kw, (kh << 16) | kw);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = (int)((gridDim.x * blockDim.x) >> 5);
  // Each warp takes a contiguous run of rows: (n, oh, ow) is decomposed once
  // and then stepped, and consecutive rows reuse the same input sectors.
  const int per = (rows + warps - 1) / warps;
  const int first = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * per;
  const int last = first + per < rows ? first + per : rows;
  if (first >= last) return;
  int n = first / OHW, r = first - n * OHW, oh = r / OW, ow = r - oh * OW;
  for (int row = first; row < last; row++) {
    const int h0 = oh * stride - pad, w0 = ow * stride - pad;
    const T* img = x + (int64_t)n * C * HW;
    T* out = cols + (int64_t)row * K;
    for (int k = lane; k < K; k += 32) {
      const int2 t = ktab[k];
      const int ih = h0 + (t.y >> 16), iw = w0 + (t.y & 0xFFFF);
      out[k] = (ih >= 0 && ih < H && iw >= 0 && iw < W) ? img[t.x + h0 * W + w0] : (T)0;
    }
    if (++ow == OW) {
      ow = 0;
      if (++oh == OH) oh = 0, n++;
    }
  }
}

// dy (N, O, L) -> dyp (O, N, L): contiguous runs of L on both sides.
template <typename T>
__global__ void permute_nol_kernel(const T* __restrict__ dy, T* __restrict__ dyp, int64_t N, int64_t O, int64_t L) {
  for (int64_t r = blockIdx.x; r < O * N; r += gridDim.x) {  // r = o * N + n
    const int64_t o = r / N, n = r - o * N;
    const T* src = dy + (n * O + o) * L;
    T* dst = dyp + r * L;
    for (int64_t l = threadIdx.x; l < L; l += blockDim.x) dst[l] = src[l];
  }
}

// The same permute as 16-byte vectors over the whole tensor, a thread per
// vector (L a multiple of 16 bytes, 32-bit indices): short rows (L = 16 or
// 64 positions) no longer leave threads idle or loads unoverlapped.
template <typename V>
__global__ void permute_nol_vec_kernel(const V* __restrict__ dy, V* __restrict__ dyp, int32_t N, int32_t O,
                                       int32_t LV, int32_t total) {
  for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int32_t r = i / LV, l = i - r * LV;  // r = o * N + n
    const int32_t o = r / N, n = r - o * N;
    dyp[i] = dy[(n * O + o) * LV + l];
  }
}

// I: the index type, int32_t when every index of the call fits (chosen on the
// host), which keeps the divisions cheap.
template <typename T, typename I>
__global__ void col2im_kernel(const T* __restrict__ cols, T* __restrict__ x, gt_geom g64, I total) {
  struct {
    I C, H, W, KH, KW, OH, OW, stride, pad;
  } g = {(I)g64.C, (I)g64.H, (I)g64.W, (I)g64.KH, (I)g64.KW, (I)g64.OH, (I)g64.OW, (I)g64.stride, (I)g64.pad};
  const I K = g.C * g.KH * g.KW;
  for (I e = (I)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (I)gridDim.x * blockDim.x) {
    I iw = e % g.W, t = e / g.W;
    I ih = t % g.H, t2 = t / g.H;
    I c = t2 % g.C, n = t2 / g.C;
    I hp = ih + g.pad, wp = iw + g.pad;
    // oh*stride <= hp and oh*stride > hp - KH
    I oh_lo = hp - g.KH + 1 > 0 ? (hp - g.KH + 1 + g.stride - 1) / g.stride : 0;
    I oh_hi = hp / g.stride < g.OH - 1 ? hp / g.stride : g.OH - 1;
    I ow_lo = wp - g.KW + 1 > 0 ? (wp - g.KW + 1 + g.stride - 1) / g.stride : 0;
    I ow_hi = wp / g.stride < g.OW - 1 ? wp / g.stride : g.OW - 1;
    T acc = (T)0;
    for (I oh = oh_lo; oh <= oh_hi; oh++) {
      I kh = hp - oh * g.stride;
      for (I ow = ow_lo; ow <= ow_hi; ow++) {
        I kw = wp - ow * g.stride;
        I row = (n * g.OH + oh) * g.OW + ow;
        acc = add_rn(acc, cols[row * K + (c * g.KH + kh) * g.KW + kw]);
      }
    }
    x[e] = acc;
  }
}

// First maximum of a window, as internal/cpu/linalg.go:169-176:
// `if v > best || bestIdx < 0`.
template <typename T>
__device__ __forceinline__ int window_argmax(const T* __restrict__ plane, const gt_geom& g, int64_t oh, int64_t ow,
                                             T* best_out) {
  T best = (T)(-INFINITY);
  int best_k = -1;
  for (int64_t kh = 0; kh < g.KH; kh++)
    for (int64_t kw = 0; kw < g.KW; kw++) {
      T v = plane[(oh * g.stride + kh) * g.W + ow * g.stride + kw];
      if (v > best || best_k < 0) {
        best = v;
        best_k = (int)(kh * g.KW + kw);
      }
    }
  *best_out = best;
  return best_k;
}

template <typename T>
__global__ void maxpool_fwd_kernel(const T* __restrict__ x, T* __restrict__ out, uint8_t* __restrict__ idx, gt_geom g,
                                   int64_t total) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t ow = e % g.OW, t = e / g.OW;
    int64_t oh = t % g.OH, pl = t / g.OH;
    T best;
    int k = window_argmax(x + pl * g.H * g.W, g, oh, ow, &best);
    out[e] = best;
    if (idx) idx[e] = (uint8_t)k;
  }
}

// 2 x 2 windows with stride 2 that tile the input exactly (H = 2 OH,
// W = 2 OW), the pooling of both conv configurations: a thread per output,
// whose window is two 8-byte pairs of adjacent inputs, so a warp's loads and
// stores are contiguous runs. Same first-maximum rule and outputs as
// maxpool_fwd_kernel / maxpool_bwd_idx_kernel.
template <typename T, typename I>
__global__ void maxpool2_fwd_kernel(const T* __restrict__ x, T* __restrict__ out, uint8_t* __restrict__ idx,
                                    I OH, I OW, I total) {
  for (I e = (I)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (I)gridDim.x * blockDim.x) {
    const I ow = e % OW, t = e / OW;  // t = plane * OH + oh
    const T* r0 = x + (int64_t)t * 4 * OW + 2 * ow;
    const T v[4] = {r0[0], r0[1], r0[2 * OW], r0[2 * OW + 1]};
    T best = v[0];
    int k = 0;
#pragma unroll
    for (int j = 1; j < 4; j++)
      if (v[j] > best) {
        best = v[j];
        k = j;
      }
    out[e] = best;
    if (idx) idx[e] = (uint8_t)k;
  }
}

template <typename T, typename I>
__global__ void maxpool2_bwd_idx_kernel(const T* __restrict__ grad, const uint8_t* __restrict__ idx,
                                        const T* __restrict__ pooled, int relu_mask, T* __restrict__ dx, I OW,
                                        I total) {
  for (I e = (I)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (I)gridDim.x * blockDim.x) {
    const I ow = e % OW, t = e / OW;
    T v = grad[e];
    if (relu_mask) v = mul_rn(v, pooled[e] > (T)0 ? (T)1 : (T)0);
    const int k = idx[e];
    T* r0 = dx + (int64_t)t * 4 * OW + 2 * ow;
    r0[0] = k == 0 ? v : (T)0;
    r0[1] = k == 1 ? v : (T)0;
    r0[2 * OW] = k == 2 ? v : (T)0;
    r0[2 * OW + 1] = k == 3 ? v : (T)0;
  }
}

// The weight operand of an implicit-GEMM convolution, split into its tf32
// planes once per call (the splitter warps would otherwise split the same
// weight slice again for every tile): ws rows [0, rows) = tf32(v) and rows
// [rows_pad, rows_pad + rows) = tf32(v - tf32(v)), rows of `pitch` elements
// (a multiple of 4, for the TMA copy), zero elsewhere. v is row r, column j
// of the GEMM's B operand:
//   forward (flip = 0): w viewed as (O, C*KH*KW), rows = O, cols = C*KH*KW;
//   input gradient (flip = 1): the weight of the forward convolution of dy
//     that gives dx (stride 1): row c, column (o, kh, kw) =
//     w[o][c][KH-1-kh][KW-1-kw], rows = C, cols = O*KH*KW.
__global__ void split_weight_kernel(const float* __restrict__ w, float* __restrict__ ws, int rows, int cols,
                                    int pitch, int rows_pad, int flip, int O, int C, int KH, int KW) {
  const int KHW = KH * KW;
  const int64_t plane = (int64_t)rows_pad * pitch;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < plane; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / pitch), j = (int)(i - (int64_t)r * pitch);
    float v = 0.0f;
    if (r < rows && j < cols) {
      if (flip) {
        const int o = j / KHW, rem = j - o * KHW, kh = rem / KW, kw = rem - kh * KW;
        v = w[((int64_t)(o * C + r) * KH + (KH - 1 - kh)) * KW + (KW - 1 - kw)];
      } else {
        v = w[(int64_t)r * cols + j];
      }
    }
    const float h = tf32_round(v);
    ws[i] = h;
    ws[plane + i] = tf32_round(__fsub_rn(v, h));
  }
}

static bool pool2_tiles(const gt_geom* g) {
  return g->KH == 2 && g->KW == 2 && g->stride == 2 && g->pad == 0 && g->H == 2 * g->OH && g->W == 2 * g->OW;
}

// dx[pl][ih][iw] = sum of grad over the windows whose first maximum is this
// element, visited in increasing window order (the reference's order).
template <typename T>
__global__ void maxpool_bwd_kernel(const T* __restrict__ x, const T* __restrict__ grad, T* __restrict__ dx, gt_geom g,
                                   int64_t total) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t iw = e % g.W, t = e / g.W;
    int64_t ih = t % g.H, pl = t / g.H;
    const T* plane = x + pl * g.H * g.W;
    int64_t oh_lo = ih - g.KH + 1 > 0 ? (ih - g.KH + 1 + g.stride - 1) / g.stride : 0;
    int64_t oh_hi = ih / g.stride < g.OH - 1 ? ih / g.stride : g.OH - 1;
    int64_t ow_lo = iw - g.KW + 1 > 0 ? (iw - g.KW + 1 + g.stride - 1) / g.stride : 0;
    int64_t ow_hi = iw / g.stride < g.OW - 1 ? iw / g.stride : g.OW - 1;
    T acc = (T)0;
    for (int64_t oh = oh_lo; oh <= oh_hi; oh++)
      for (int64_t ow = ow_lo; ow <= ow_hi; ow++) {
        T best;
        int k = window_argmax(plane, g, oh, ow, &best);
        if ((ih - oh * g.stride) * g.KW + (iw - ow * g.stride) == k)
          acc = add_rn(acc, grad[(pl * g.OH + oh) * g.OW + ow]);
      }
    dx[e] = acc;
  }
}

// Non-overlapping windows: each input element lies in at most one window, so
// dx is grad at the recorded maximum (times relu'(pooled) when the pool
// follows a ReLU) and zero elsewhere.
template <typename T, typename I>
__global__ void maxpool_bwd_idx_kernel(const T* __restrict__ grad, const uint8_t* __restrict__ idx,
                                       const T* __restrict__ pooled, int relu_mask, T* __restrict__ dx, gt_geom g64,
                                       I total) {
  struct {
    I H, W, KH, KW, OH, OW, stride;
  } g = {(I)g64.H, (I)g64.W, (I)g64.KH, (I)g64.KW, (I)g64.OH, (I)g64.OW, (I)g64.stride};
  for (I e = (I)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (I)gridDim.x * blockDim.x) {
    I iw = e % g.W, t = e / g.W;
    I ih = t % g.H, pl = t / g.H;
    I oh = ih / g.stride, ow = iw / g.stride;
    I kh = ih - oh * g.stride, kw = iw - ow * g.stride;
    T v = (T)0;
    if (oh < g.OH && ow < g.OW && kh < g.KH && kw < g.KW) {
      I w = (pl * g.OH + oh) * g.OW + ow;
      if (idx[w] == (uint8_t)(kh * g.KW + kw)) {
        v = grad[w];
        if (relu_mask) v = mul_rn(v, pooled[w] > (T)0 ? (T)1 : (T)0);
      }
    }
    dx[e] = v;
  }
}

static char* check_geom(const gt_geom* g, const char* what) {
  if (!g) return errorf("%s: null geometry", what);
  if (g->N < 0 || g->C < 0 || g->H < 0 || g->W < 0 || g->KH <= 0 || g->KW <= 0 || g->stride < 1 || g->pad < 0 ||
      g->OH < 0 || g->OW < 0)
    return errorf("%s: invalid geometry", what);
  if (g->OH != (g->H + 2 * g->pad - g->KH) / g->stride + 1 || g->OW != (g->W + 2 * g->pad - g->KW) / g->stride + 1)
    return errorf("%s: OH/OW do not match the geometry", what);
  return nullptr;
}

template <typename T>
static char* im2col_launch(gt_ctx* ctx, const T* x, T* cols, const gt_geom& g) {
  int64_t total = g.N * g.OH * g.OW * g.C * g.KH * g.KW;
  if (total == 0) return nullptr;
  const int64_t rows = g.N * g.OH * g.OW, K = g.C * g.KH * g.KW;
  const bool fits = K <= 6144 && g.KH < 32768 && g.KW < 32768 && rows < INT32_MAX / 2 &&
                    g.C * g.H * g.W < INT32_MAX / 2 && (g.H + 2 * g.pad) * (g.W + 2 * g.pad) < INT32_MAX / 4;
  if (fits) {
    const int grid = (int)std::min<int64_t>(ceil_div(rows, 8), (int64_t)ctx->sm_count * 16);
    im2col_rows_kernel<T><<<grid, 256, K * sizeof(int2), ctx->stream>>>(x, cols, g, (int)rows, (int)K);
  } else {
    im2col_kernel<T><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>(x, cols, g, total);
  }
  GT_LAUNCH_CHECK();
  return nullptr;
}

template <typename T>
static char* col2im_launch(gt_ctx* ctx, const T* cols, T* x, const gt_geom& g) {
  int64_t total = g.N * g.C * g.H * g.W;
  if (total == 0) return nullptr;
  const int64_t colsize = g.N * g.OH * g.OW * g.C * g.KH * g.KW;
  if (total < INT32_MAX / 2 && colsize < INT32_MAX / 2 && (g.H + g.pad) * g.stride < INT32_MAX / 4)
    col2im_kernel<T, int32_t><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>(cols, x, g, (int32_t)total);
  else
    col2im_kernel<T, int64_t><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>(cols, x, g, total);
  GT_LAUNCH_CHECK();
  return nullptr;
}

}  // namespace gt

using namespace gt;

extern "C" {

char* gt_im2col(gt_ctx* ctx, int dtype, const void* x, void* cols, const gt_geom* g) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_im2col"));
  GT_DISPATCH(dtype, { return im2col_launch<T>(ctx, (const T*)x, (T*)cols, *g); });
  return nullptr;
}

char* gt_col2im(gt_ctx* ctx, int dtype, const void* cols, void* x, const gt_geom* g) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_col2im"));
  GT_DISPATCH(dtype, { return col2im_launch<T>(ctx, (const T*)cols, (T*)x, *g); });
  return nullptr;
}

char* gt_maxpool_fwd(gt_ctx* ctx, int dtype, const void* x, void* out, const gt_geom* g) {
  return gt_maxpool_fwd_idx(ctx, dtype, x, out, nullptr, g);
}

char* gt_maxpool_fwd_idx(gt_ctx* ctx, int dtype, const void* x, void* out, uint8_t* idx, const gt_geom* g) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_maxpool_fwd"));
  if (g->pad != 0) return errorf("gt_maxpool_fwd: pooling has no padding");
  if (idx && g->KH * g->KW > 256) return errorf("gt_maxpool_fwd_idx: window larger than 256 elements");
  int64_t total = g->N * g->C * g->OH * g->OW;
  if (total == 0) return nullptr;
  GT_DISPATCH(dtype, {
    if (pool2_tiles(g) && total < INT32_MAX / 2)
      maxpool2_fwd_kernel<T, int32_t><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>(
          (const T*)x, (T*)out, idx, (int32_t)g->OH, (int32_t)g->OW, (int32_t)total);
    else if (pool2_tiles(g))
      maxpool2_fwd_kernel<T, int64_t><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>(
          (const T*)x, (T*)out, idx, g->OH, g->OW, total);
    else
      maxpool_fwd_kernel<T><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>((const T*)x, (T*)out, idx, *g,
                                                                               total);
  });
  GT_LAUNCH_CHECK();
  return nullptr;
}

char* gt_maxpool_bwd(gt_ctx* ctx, int dtype, const void* x, const void* grad, void* dx, const gt_geom* g) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_maxpool_bwd"));
  if (g->pad != 0) return errorf("gt_maxpool_bwd: pooling has no padding");
  int64_t total = g->N * g->C * g->H * g->W;
  if (total == 0) return nullptr;
  GT_DISPATCH(dtype, {
    maxpool_bwd_kernel<T><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>((const T*)x, (const T*)grad, (T*)dx, *g,
                                                                             total);
  });
  GT_LAUNCH_CHECK();
  return nullptr;
}

char* gt_maxpool_bwd_idx(gt_ctx* ctx, int dtype, const void* grad, const uint8_t* idx, const void* pooled,
                         int relu_mask, void* dx, const gt_geom* g) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_maxpool_bwd_idx"));
  if (g->pad != 0) return errorf("gt_maxpool_bwd_idx: pooling has no padding");
  if (g->stride < g->KH || g->stride < g->KW) return errorf("gt_maxpool_bwd_idx: windows overlap; use gt_maxpool_bwd");
  if (relu_mask && !pooled) return errorf("gt_maxpool_bwd_idx: relu_mask needs the pooled output");
  int64_t total = g->N * g->C * g->H * g->W;
  if (total == 0) return nullptr;
  if (pool2_tiles(g)) {  // a thread per window
    const int64_t outs = g->N * g->C * g->OH * g->OW;
    GT_DISPATCH(dtype, {
      if (outs < INT32_MAX / 2)
        maxpool2_bwd_idx_kernel<T, int32_t><<<grid_for(ctx, outs, 256), 256, 0, ctx->stream>>>(
            (const T*)grad, idx, (const T*)pooled, relu_mask, (T*)dx, (int32_t)g->OW, (int32_t)outs);
      else
        maxpool2_bwd_idx_kernel<T, int64_t><<<grid_for(ctx, outs, 256), 256, 0, ctx->stream>>>(
            (const T*)grad, idx, (const T*)pooled, relu_mask, (T*)dx, g->OW, outs);
    });
    GT_LAUNCH_CHECK();
    return nullptr;
  }
  GT_DISPATCH(dtype, {
    if (total < INT32_MAX / 2)
      maxpool_bwd_idx_kernel<T, int32_t><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>(
          (const T*)grad, idx, (const T*)pooled, relu_mask, (T*)dx, *g, (int32_t)total);
    else
      maxpool_bwd_idx_kernel<T, int64_t><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>(
          (const T*)grad, idx, (const T*)pooled, relu_mask, (T*)dx, *g, total);
  });
  GT_LAUNCH_CHECK();
  return nullptr;
}

// The implicit-GEMM forward (float32, tcgen05): no columns in memory. The
// weight is first split into its tf32 planes (split_weight_kernel). *done is
// false if the geometry does not qualify.
static char* conv_implicit(gt_ctx* ctx, const float* x, const float* w, int flip, int64_t rows, int64_t cols,
                           const float* bias, float* y, const gt_geom& g, int act, int64_t O_w, int64_t C_w,
                           bool* done) {
  *done = false;
  if ((act != GT_ACT_NONE && act != GT_ACT_RELU) || g.stride != 1) return nullptr;
  const int64_t pitch = (cols + 3) / 4 * 4, rows_pad = conv_weight_rows(rows);
  if (2 * rows_pad * pitch >= INT32_MAX / 2) return nullptr;
  void* ws = nullptr;
  GT_TRY(scratch(ctx, (size_t)(2 * rows_pad * pitch) * sizeof(float), &ws));
  split_weight_kernel<<<grid_for(ctx, rows_pad * pitch, 256), 256, 0, ctx->stream>>>(
      w, (float*)ws, (int)rows, (int)cols, (int)pitch, (int)rows_pad, flip, (int)O_w, (int)C_w, (int)g.KH,
      (int)g.KW);
  count_launch();
  cudaError_t e = cudaGetLastError();
  char* err = e != cudaSuccess ? cuda_error(e, "split_weight_kernel launch", __FILE__, __LINE__)
                               : conv_fwd_gemm(ctx, x, (const float*)ws, pitch, bias, y, g, rows, act, done);
  release(ctx, ws);
  return err;
}

static char* conv_fwd_implicit(gt_ctx* ctx, const float* x, const float* w, const float* bias, float* y,
                               const gt_geom& g, int64_t O, int act, bool* done) {
  return conv_implicit(ctx, x, w, 0, O, g.C * g.KH * g.KW, bias, y, g, act, O, g.C, done);
}

// The implicit-GEMM input gradient of a stride-1 convolution with a square
// window: dx = conv2d(dy, flip(w)^T) with padding KH-1-pad (dy plays the
// input, C the output channels).
static char* conv_dgrad_implicit(gt_ctx* ctx, const float* dy, const float* w, float* dx, const gt_geom& g,
                                 int64_t O, bool* done) {
  *done = false;
  if (g.stride != 1 || g.KH != g.KW || g.pad > g.KH - 1) return nullptr;
  gt_geom gd = g;
  gd.C = O, gd.H = g.OH, gd.W = g.OW, gd.OH = g.H, gd.OW = g.W, gd.pad = g.KH - 1 - g.pad;
  return conv_implicit(ctx, dy, w, 1, g.C, O * g.KH * g.KW, nullptr, dx, gd, GT_ACT_NONE, O, g.C, done);
}

// Conv2d forward. float32 runs as an implicit GEMM on the tensor cores
// (conv_fwd_implicit); otherwise cols = im2col(x) (scratch), then C (O, N*L)
// = W (O, CKK) @ cols^T stored straight into NCHW with the bias and
// activation fused.
char* gt_conv_fwd(gt_ctx* ctx, int dtype, const void* x, const void* w, const void* bias, void* y, const gt_geom* g,
                  int64_t O, int act) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_conv_fwd"));
  if (O <= 0) return errorf("gt_conv_fwd: out_channels must be positive");
  const int64_t L = g->OH * g->OW, NL = g->N * L, CKK = g->C * g->KH * g->KW;
  if (NL == 0) return nullptr;
  if (dtype == GT_FLOAT32) {
    bool done = false;
    GT_TRY(conv_fwd_implicit(ctx, (const float*)x, (const float*)w, (const float*)bias, (float*)y, *g, O, act, &done));
    if (done) return nullptr;
  }
  const size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  void* cols = nullptr;
  GT_TRY(scratch(ctx, (size_t)(NL * CKK) * es, &cols));
  char* err = nullptr;
  GT_DISPATCH(dtype, {
    err = im2col_launch<T>(ctx, (const T*)x, (T*)cols, *g);
    if (!err) {
      // B(k, j) = cols[j * CKK + k]
      GemmShape s{O, NL, CKK, false, true, CKK, CKK};
      Epi<T> e;
      e.out = (T*)y;
      e.bias = (const T*)bias;
      e.bias_by_row = true;
      e.act = act;
      e.nchw_L = L;
      e.nchw_M = O;
      err = gemm<T>(ctx, s, (const T*)w, (const T*)cols, e);
    }
  });
  release(ctx, cols);
  return err;
}

// dy (N, O, L) -> dyp (O, N*L): the layout of the GEMMs below.
static char* permute_nol(gt_ctx* ctx, int dtype, const void* dy, void* dyp, int64_t N, int64_t O, int64_t L) {
  if (N * O * L == 0) return nullptr;
  const size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  if ((L * (int64_t)es) % 16 == 0 && ((uintptr_t)dy & 15) == 0 && ((uintptr_t)dyp & 15) == 0 &&
      N * O * L * (int64_t)es / 16 < INT32_MAX / 2) {
    const int64_t LV = L * (int64_t)es / 16, total = N * O * LV;
    permute_nol_vec_kernel<float4><<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>(
        (const float4*)dy, (float4*)dyp, (int32_t)N, (int32_t)O, (int32_t)LV, (int32_t)total);
    GT_LAUNCH_CHECK();
    return nullptr;
  }
  const int threads = L >= 256 ? 256 : L >= 64 ? 64 : 32;
  const int blocks = (int)std::min<int64_t>(N * O, (int64_t)ctx->sm_count * 32);
  GT_DISPATCH(dtype, {
    permute_nol_kernel<T><<<blocks, threads, 0, ctx->stream>>>((const T*)dy, (T*)dyp, N, O, L);
  });
  GT_LAUNCH_CHECK();
  return nullptr;
}

char* gt_conv_bwd_weight(gt_ctx* ctx, int dtype, const void* x, const void* dy, void* dw, void* db, const gt_geom* g,
                         int64_t O) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_conv_bwd_weight"));
  if (O <= 0) return errorf("gt_conv_bwd_weight: out_channels must be positive");
  const int64_t L = g->OH * g->OW, NL = g->N * L, CKK = g->C * g->KH * g->KW;
  const size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  if (NL == 0) {
    GT_CUDA(cudaMemsetAsync(dw, 0, O * CKK * es, ctx->stream));
    if (db) GT_CUDA(cudaMemsetAsync(db, 0, O * es, ctx->stream));
    return nullptr;
  }
  if (dtype == GT_FLOAT32) {  // implicit GEMM: no columns, dy read in place, db as one more row
    bool done = false;
    GT_TRY(conv_wgrad_gemm(ctx, (const float*)x, (const float*)dy, (float*)dw, (float*)db, *g, O, &done));
    if (done) return nullptr;
  }
  void *cols = nullptr, *dyp = nullptr;
  GT_TRY(scratch(ctx, (size_t)(NL * CKK) * es, &cols));
  char* err = scratch(ctx, (size_t)(O * NL) * es, &dyp);
  if (!err) err = permute_nol(ctx, dtype, dy, dyp, g->N, O, L);
  GT_DISPATCH(dtype, {
    if (!err) err = im2col_launch<T>(ctx, (const T*)x, (T*)cols, *g);
    if (!err) {
      // dW (O, CKK) = dyp (O, NL) @ cols (NL, CKK)
      GemmShape s{O, CKK, NL, false, false, NL, CKK};
      Epi<T> e;
      e.out = (T*)dw;
      e.ldc = CKK;
      err = gemm<T>(ctx, s, (const T*)dyp, (const T*)cols, e);
    }
  });
  if (!err && db) err = gt_reduce(ctx, dtype, GT_SUM, dyp, db, O, NL, 1);
  release(ctx, cols);
  release(ctx, dyp);
  return err;
}

char* gt_conv_bwd_data(gt_ctx* ctx, int dtype, const void* dy, const void* w, void* dx, const gt_geom* g, int64_t O) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_conv_bwd_data"));
  if (O <= 0) return errorf("gt_conv_bwd_data: out_channels must be positive");
  const int64_t L = g->OH * g->OW, NL = g->N * L, CKK = g->C * g->KH * g->KW;
  const size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  if (NL == 0) {  // no output positions: nothing reaches the input
    GT_CUDA(cudaMemsetAsync(dx, 0, g->N * g->C * g->H * g->W * es, ctx->stream));
    return nullptr;
  }
  if (dtype == GT_FLOAT32) {  // implicit GEMM: no dcols, no col2im
    bool done = false;
    GT_TRY(conv_dgrad_implicit(ctx, (const float*)dy, (const float*)w, (float*)dx, *g, O, &done));
    if (done) return nullptr;
  }
  void *dcols = nullptr, *dyp = nullptr;
  GT_TRY(scratch(ctx, (size_t)(NL * CKK) * es, &dcols));
  char* err = scratch(ctx, (size_t)(O * NL) * es, &dyp);
  if (!err) err = permute_nol(ctx, dtype, dy, dyp, g->N, O, L);
  GT_DISPATCH(dtype, {
    if (!err) {
      // dcols (NL, CKK) = dyp^T (NL, O) @ W (O, CKK): A(m=j, k=o) = dyp[o*NL + j]
      GemmShape s{NL, CKK, O, true, false, NL, CKK};
      Epi<T> e;
      e.out = (T*)dcols;
      e.ldc = CKK;
      err = gemm<T>(ctx, s, (const T*)dyp, (const T*)w, e);
    }
    if (!err) err = col2im_launch<T>(ctx, (const T*)dcols, (T*)dx, *g);
  });
  release(ctx, dcols);
  release(ctx, dyp);
  return err;
}

// Conv2d forward that keeps its im2col columns in `cols` (N*L x C*KH*KW
// elements, the caller's buffer) for gt_conv_bwd: the same kernels and result
// as gt_conv_fwd.
char* gt_conv_fwd_cols(gt_ctx* ctx, int dtype, const void* x, const void* w, const void* bias, void* y, void* cols,
                       const gt_geom* g, int64_t O, int act) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_conv_fwd_cols"));
  if (O <= 0 || !cols) return errorf("gt_conv_fwd_cols: bad arguments");
  const int64_t L = g->OH * g->OW, NL = g->N * L, CKK = g->C * g->KH * g->KW;
  if (NL == 0) return nullptr;
  GT_DISPATCH(dtype, {
    GT_TRY(im2col_launch<T>(ctx, (const T*)x, (T*)cols, *g));
    GemmShape s{O, NL, CKK, false, true, CKK, CKK};
    Epi<T> e;
    e.out = (T*)y;
    e.bias = (const T*)bias;
    e.bias_by_row = true;
    e.act = act;
    e.nchw_L = L;
    e.nchw_M = O;
    return gemm<T>(ctx, s, (const T*)w, (const T*)cols, e);
  });
  return nullptr;
}

// Conv2d backward from the forward's columns: dy is permuted to (O, N*L)
// once for both GEMMs, dW = dyp @ cols, db = row sums of dyp, and (dx not
// NULL) dx = col2im(dyp^T @ W). The same kernels, in the same order, as
// gt_conv_bwd_weight followed by gt_conv_bwd_data.
char* gt_conv_bwd(gt_ctx* ctx, int dtype, const void* cols, const void* dy, const void* w, void* dx, void* dw,
                  void* db, const gt_geom* g, int64_t O) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_conv_bwd"));
  if (O <= 0 || !cols || !dw) return errorf("gt_conv_bwd: bad arguments");
  const int64_t L = g->OH * g->OW, NL = g->N * L, CKK = g->C * g->KH * g->KW;
  const size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  if (NL == 0) {
    GT_CUDA(cudaMemsetAsync(dw, 0, O * CKK * es, ctx->stream));
    if (db) GT_CUDA(cudaMemsetAsync(db, 0, O * es, ctx->stream));
    if (dx) GT_CUDA(cudaMemsetAsync(dx, 0, g->N * g->C * g->H * g->W * es, ctx->stream));
    return nullptr;
  }
  void *dyp = nullptr, *dcols = nullptr;
  GT_TRY(scratch(ctx, (size_t)(O * NL) * es, &dyp));
  char* err = permute_nol(ctx, dtype, dy, dyp, g->N, O, L);
  GT_DISPATCH(dtype, {
    if (!err) {
      GemmShape s{O, CKK, NL, false, false, NL, CKK};
      Epi<T> e;
      e.out = (T*)dw;
      e.ldc = CKK;
      err = gemm<T>(ctx, s, (const T*)dyp, (const T*)cols, e);
    }
  });
  if (!err && db) err = gt_reduce(ctx, dtype, GT_SUM, dyp, db, O, NL, 1);
  if (!err && dx) err = scratch(ctx, (size_t)(NL * CKK) * es, &dcols);
  if (!err && dx) {
    GT_DISPATCH(dtype, {
      GemmShape s{NL, CKK, O, true, false, NL, CKK};
      Epi<T> e;
      e.out = (T*)dcols;
      e.ldc = CKK;
      err = gemm<T>(ctx, s, (const T*)dyp, (const T*)w, e);
      if (!err) err = col2im_launch<T>(ctx, (const T*)dcols, (T*)dx, *g);
    });
  }
  release(ctx, dcols);
  release(ctx, dyp);
  return err;
}

}  // extern "C"
