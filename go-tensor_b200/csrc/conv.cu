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


// Weight and bias gradients of a convolution whose output went through
// [ReLU ->] MaxPool2d with k x k windows at stride k that tile it exactly,
// computed from the pooled gradient. The reference's output gradient is
// MaxPool2dBackward of it (the pooled gradient at each window's first
// maximum, zero elsewhere: tensor/conv.go:63-70, internal/cpu/linalg.go:
// 169-191) times ReLU's Step factor (tensor/ops.go:110), and the weight
// gradient sums it against the patches (tensor/conv.go:40-59). Only window
// maxima carry a nonzero term, so pooled position q adds g_q * patch(p_q) to
// dW and g_q to db, with p_q its window's maximum and g_q = grad_q *
// Step(pooled_q). A zero term still counts when its patch value is infinite
// or NaN (0 * inf = NaN), so an image holding a non-finite value takes every
// window position, zeros included, as the dense sum does.
//
// One block per image. The zero-padded image is staged in shared memory;
// warp w takes output channels w, w + 8, ...; lane l takes pooled positions
// l, l + 32, ... and keeps CKK + 1 running sums (fused multiply-adds). The
// warp adds its lanes' sums in lane order through shared memory and writes
// the image's partials part_w[n][o * CKK + k] and part_b[n][o];
// column_sums_kernel then adds the images in a fixed order.
constexpr int kPoolWgradWarps = 8;

template <typename T>
__host__ __device__ constexpr size_t pool_wgrad_red_bytes(int nk) {
  return (size_t)kPoolWgradWarps * (nk + 1) * 33 * sizeof(T);
}
// The patch offset table, padded to 16 bytes so that the image after it is
// aligned for any T.
__host__ __device__ constexpr size_t pool_wgrad_koff_bytes(int nk) { return ((size_t)nk * sizeof(int) + 15) / 16 * 16; }

// KS = 3: 3 x 3 windows over at most NK / 9 channels, the patch offsets
// computed in registers; KS = 0: any window, offsets from a shared table.
template <typename T, int NK, int KS>
__global__ void __launch_bounds__(32 * kPoolWgradWarps)
    conv_wgrad_pool_kernel(const T* __restrict__ x, const T* __restrict__ grad, const uint8_t* __restrict__ idx,
                           const T* __restrict__ pooled, int relu, int C, int H, int W, int KH, int KW, int stride,
                           int pad, int kp, int PH, int PW, int O, T* __restrict__ part_w, T* __restrict__ part_b) {
  extern __shared__ __align__(16) unsigned char pool_wgrad_smem[];
  const int Hs = H + 2 * pad, Ws = W + 2 * pad, plane = Hs * Ws, KHW = KH * KW, CKK = C * KHW;
  T* red = reinterpret_cast<T*>(pool_wgrad_smem);
  int* koff = reinterpret_cast<int*>(pool_wgrad_smem + pool_wgrad_red_bytes<T>(NK));
  T* xs = reinterpret_cast<T*>(pool_wgrad_smem + pool_wgrad_red_bytes<T>(NK) + pool_wgrad_koff_bytes(NK));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t n = blockIdx.x;
  const T* xn = x + n * C * H * W;
  bool bad = false;
  for (int e = tid; e < C * plane; e += blockDim.x) {
    const int c = e / plane, r = e - c * plane, hs = r / Ws, ws = r - hs * Ws, h = hs - pad, w = ws - pad;
    const T v = (h >= 0 && h < H && w >= 0 && w < W) ? xn[((int64_t)c * H + h) * W + w] : (T)0;
    bad |= !isfinite(v);
    xs[e] = v;
  }
  for (int k = tid; k < NK; k += blockDim.x) {
    int off = 0;
    if (k < CKK) {
      const int c = k / KHW, r = k - c * KHW, kh = r / KW, kw = r - kh * KW;
      off = c * plane + kh * Ws + kw;
    }
    koff[k] = off;
  }
  const bool dense = __syncthreads_or(bad);
  const int P = PH * PW, win = kp * kp;
  T* rw = red + warp * (NK + 1) * 33;
  for (int o = warp; o < O; o += kPoolWgradWarps) {
    T acc[NK + 1];
#pragma unroll
    for (int k = 0; k <= NK; k++) acc[k] = (T)0;
    const int64_t qbase = (n * O + o) * P;
    for (int q = lane; q < P; q += 32) {
      T g = grad[qbase + q];
      if (relu) g = mul_rn(g, pooled[qbase + q] > (T)0 ? (T)1 : (T)0);
      const int m = idx[qbase + q];
      const int qh = q / PW, qw = q - qh * PW;
      const int i0 = dense ? 0 : m, i1 = dense ? win : min(m + 1, win);  // an index past the window adds nothing
      for (int i = i0; i < i1; i++) {
        const T gi = i == m ? g : (T)0;
        const int ih = i / kp, iw = i - ih * kp;
        // the patch of output position (qh*kp + ih, qw*kp + iw), in the padded image
        const T* xp = xs + (qh * kp + ih) * stride * Ws + (qw * kp + iw) * stride;
        if constexpr (KS == 3) {
#pragma unroll
          for (int c = 0; c < NK / 9; c++)
            if (c < C) {
              const T* xc = xp + c * plane;
#pragma unroll
              for (int kh = 0; kh < 3; kh++)
#pragma unroll
                for (int kw = 0; kw < 3; kw++) acc[c * 9 + kh * 3 + kw] = fma(gi, xc[kh * Ws + kw], acc[c * 9 + kh * 3 + kw]);
            }
        } else {
#pragma unroll
          for (int k = 0; k < NK; k++)
            if (k < CKK) acc[k] = fma(gi, xp[koff[k]], acc[k]);
        }
        acc[NK] = acc[NK] + gi;
      }
    }
#pragma unroll
    for (int k = 0; k <= NK; k++) rw[k * 33 + lane] = acc[k];
    __syncwarp();
    for (int k = lane; k <= NK; k += 32) {
      if (k < CKK || k == NK) {
        T s = rw[k * 33];
        for (int j = 1; j < 32; j++) s = s + rw[k * 33 + j];
        if (k == NK)
          part_b[n * O + o] = s;
        else
          part_w[(n * O + o) * CKK + k] = s;
      }
    }
    __syncwarp();
  }
}

// Shared memory of conv_wgrad_pool_kernel: the lane-sum buffer, the patch
// offset table and the padded image.
template <typename T, int NK>
static size_t pool_wgrad_smem_bytes(const gt_geom& g) {  // the same for both KS
  return pool_wgrad_red_bytes<T>(NK) + pool_wgrad_koff_bytes(NK) +
         (size_t)g.C * (g.H + 2 * g.pad) * (g.W + 2 * g.pad) * sizeof(T);
}

template <typename T, int NK, int KS>
static char* pool_wgrad_launch(gt_ctx* ctx, const T* x, const T* grad, const uint8_t* idx, const T* pooled, int relu,
                               const gt_geom& g, const gt_geom& pg, int64_t O, T* part_w, T* part_b) {
  const size_t smem = pool_wgrad_smem_bytes<T, NK>(g);
  static bool configured[64] = {};
  int dev = 0;
  GT_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !configured[dev]) {
    GT_CUDA(cudaFuncSetAttribute(conv_wgrad_pool_kernel<T, NK, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 200 * 1024));
    configured[dev] = true;
  }
  conv_wgrad_pool_kernel<T, NK, KS><<<(unsigned)g.N, 32 * kPoolWgradWarps, smem, ctx->stream>>>(
      x, grad, idx, pooled, relu, (int)g.C, (int)g.H, (int)g.W, (int)g.KH, (int)g.KW, (int)g.stride, (int)g.pad,
      (int)pg.KH, (int)pg.OH, (int)pg.OW, (int)O, part_w, part_b);
  GT_LAUNCH_CHECK();
  return nullptr;
}

// The arguments of one gt_conv_bwd_weight_pool launch, and the choice of
// kernel variant: 3 x 3 windows with the patch offsets in registers, or the
// offset table for other windows.
struct PoolWgradArgs {
  gt_ctx* ctx;
  int dtype, relu;
  const void *x, *grad, *pooled;
  const uint8_t* idx;
  const gt_geom *g, *pg;
  int64_t O;
  void *part_w, *part_b;
};

template <typename T>
static char* pool_wgrad_dispatch(const PoolWgradArgs& a) {
  const int64_t ckk = a.g->C * a.g->KH * a.g->KW;
  const bool k3 = a.g->KH == 3 && a.g->KW == 3;
  const T *x = (const T*)a.x, *grad = (const T*)a.grad, *pooled = (const T*)a.pooled;
  T *pw = (T*)a.part_w, *pb = (T*)a.part_b;
  if (k3 && ckk <= 9) return pool_wgrad_launch<T, 9, 3>(a.ctx, x, grad, a.idx, pooled, a.relu, *a.g, *a.pg, a.O, pw, pb);
  if (k3 && ckk <= 27)
    return pool_wgrad_launch<T, 27, 3>(a.ctx, x, grad, a.idx, pooled, a.relu, *a.g, *a.pg, a.O, pw, pb);
  if (ckk <= 16) return pool_wgrad_launch<T, 16, 0>(a.ctx, x, grad, a.idx, pooled, a.relu, *a.g, *a.pg, a.O, pw, pb);
  return pool_wgrad_launch<T, 32, 0>(a.ctx, x, grad, a.idx, pooled, a.relu, *a.g, *a.pg, a.O, pw, pb);
}

// Conv2d (3 x 3 windows, stride 1, at most CM input channels: a first
// convolution) [+ ReLU] then 2 x 2 / stride-2 max pooling, computed directly:
// at K = C*9 a GEMM tile has nothing to hide its epilogue behind, and only the
// pooled values are needed. A block stages one image (zero-padded), the
// weights and the biases in shared memory; a thread takes a pooled position,
// keeps the 4 x 4 x C input region its window's four patches cover in
// registers, and for each output channel forms the four outputs as FMA
// chains over (c, kh, kw) in order (the weights broadcast to the warp), adds
// the bias, applies ReLU and stores the first maximum (MaxPool2d's v > best
// rule, offsets kh * 2 + kw) and its offset.
template <typename T, int CM>
__global__ void __launch_bounds__(256)
    conv_pool_small_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bias, int relu,
                           int C, int H, int W, int pad, int O, int PH, int PW, T* __restrict__ pooled,
                           uint8_t* __restrict__ idx) {
  extern __shared__ __align__(16) unsigned char conv_pool_smem[];
  const int Hs = H + 2 * pad, Ws = W + 2 * pad, plane = Hs * Ws, CKK = C * 9;
  T* wsm = reinterpret_cast<T*>(conv_pool_smem);  // O x CKK weights
  T* bsm = wsm + O * CKK;                         // O biases
  T* xs = bsm + O;                                // C x Hs x Ws padded image
  const int tid = threadIdx.x;
  const int64_t n = blockIdx.y;
  const T* xn = x + n * C * H * W;
  for (int e = tid; e < C * plane; e += blockDim.x) {
    const int c = e / plane, r = e - c * plane, hs = r / Ws, ws = r - hs * Ws, h = hs - pad, ww = ws - pad;
    xs[e] = (h >= 0 && h < H && ww >= 0 && ww < W) ? xn[((int64_t)c * H + h) * W + ww] : (T)0;
  }
  for (int e = tid; e < O * CKK; e += blockDim.x) wsm[e] = w[e];
  for (int e = tid; e < O; e += blockDim.x) bsm[e] = bias ? bias[e] : (T)0;
  __syncthreads();
  const int P = PH * PW;
  for (int pp = blockIdx.x * blockDim.x + tid; pp < P; pp += gridDim.x * blockDim.x) {
    const int ph = pp / PW, pw = pp - ph * PW;
    T v[CM][4][4];
#pragma unroll
    for (int c = 0; c < CM; c++)
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int q = 0; q < 4; q++) v[c][r][q] = c < C ? xs[c * plane + (2 * ph + r) * Ws + 2 * pw + q] : (T)0;
    for (int o = 0; o < O; o++) {
      const T* wo = wsm + o * CKK;
      T a[4] = {(T)0, (T)0, (T)0, (T)0};
#pragma unroll
      for (int c = 0; c < CM; c++) {
        if (c >= C) break;
#pragma unroll
        for (int kh = 0; kh < 3; kh++)
#pragma unroll
          for (int kw = 0; kw < 3; kw++) {
            const T wv = wo[c * 9 + kh * 3 + kw];
            a[0] = fma(v[c][kh][kw], wv, a[0]);
            a[1] = fma(v[c][kh][kw + 1], wv, a[1]);
            a[2] = fma(v[c][kh + 1][kw], wv, a[2]);
            a[3] = fma(v[c][kh + 1][kw + 1], wv, a[3]);
          }
      }
      T best = (T)0;
      int kb = 0;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        T y = add_rn(a[j], bsm[o]);
        if (relu) y = go_max(y, (T)0);
        if (j == 0 || y > best) best = y, kb = j;
      }
      const int64_t out = (n * O + o) * P + pp;
      pooled[out] = best;
      idx[out] = (uint8_t)kb;
    }
  }
}

struct ConvPoolSmallArgs {
  gt_ctx* ctx;
  int dtype, relu;
  const void *x, *w, *bias;
  void* pooled;
  uint8_t* idx;
  const gt_geom *g, *pg;
  int64_t O;
};

static size_t conv_pool_small_smem(const gt_geom& g, int64_t O, size_t es) {
  return (size_t)(O * g.C * 9 + O + g.C * (g.H + 2 * g.pad) * (g.W + 2 * g.pad)) * es;
}

// Whether conv_pool_small_kernel takes this convolution and pooling.
static bool conv_pool_small_fits(const gt_geom& g, const gt_geom& pg, int64_t O, int act, size_t es) {
  return g.KH == 3 && g.KW == 3 && g.stride == 1 && g.C >= 1 && g.C <= 3 && g.pad <= 2 && pg.KH == 2 &&
         pg.KW == 2 && pg.stride == 2 && g.OH % 2 == 0 && g.OW % 2 == 0 && (act == GT_ACT_NONE || act == GT_ACT_RELU) &&
         g.N <= 65535 && O <= 4096 && conv_pool_small_smem(g, O, es) <= 96 * 1024 &&
         (g.H + 2 * g.pad) * (g.W + 2 * g.pad) < (1 << 24) && O * pg.OH * pg.OW < INT32_MAX / 2;
}

template <typename T, int CM>
static char* conv_pool_small_launch(const ConvPoolSmallArgs& a) {
  const gt_geom &g = *a.g, &pg = *a.pg;
  const size_t smem = conv_pool_small_smem(g, a.O, sizeof(T));
  static bool configured[64] = {};
  int dev = 0;
  GT_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !configured[dev]) {
    GT_CUDA(cudaFuncSetAttribute(conv_pool_small_kernel<T, CM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 96 * 1024));
    configured[dev] = true;
  }
  const int64_t P = pg.OH * pg.OW;
  const dim3 grid((unsigned)ceil_div(P, (int64_t)256), (unsigned)g.N);
  conv_pool_small_kernel<T, CM><<<grid, 256, smem, a.ctx->stream>>>(
      (const T*)a.x, (const T*)a.w, (const T*)a.bias, a.relu, (int)g.C, (int)g.H, (int)g.W, (int)g.pad, (int)a.O,
      (int)pg.OH, (int)pg.OW, (T*)a.pooled, a.idx);
  GT_LAUNCH_CHECK();
  return nullptr;
}

static char* conv_pool_small_run(void* p) {
  const ConvPoolSmallArgs& a = *(const ConvPoolSmallArgs*)p;
  const int64_t C = a.g->C;
  if (a.dtype == GT_FLOAT64)
    return C == 1 ? conv_pool_small_launch<double, 1>(a) : conv_pool_small_launch<double, 3>(a);
  return C == 1 ? conv_pool_small_launch<float, 1>(a) : conv_pool_small_launch<float, 3>(a);
}

// Whether gt_conv_bwd_weight_pool runs conv_wgrad_pool_kernel for these
// geometries (otherwise it goes through the full-resolution gradient).
static bool pool_wgrad_fits(const gt_geom& g, const gt_geom& pg, int64_t O, size_t es) {
  const int64_t CKK = g.C * g.KH * g.KW;
  if (pg.KH != pg.KW || pg.stride != pg.KH || pg.OH * pg.KH != pg.H || pg.OW * pg.KW != pg.W || pg.KH > 16) return false;
  if (CKK > 32 || g.N > INT32_MAX || O > 65536) return false;
  const int64_t padded = g.C * (g.H + 2 * g.pad) * (g.W + 2 * g.pad);
  const size_t smem = (es == 8 ? pool_wgrad_red_bytes<double>(32) : pool_wgrad_red_bytes<float>(32)) +
                      pool_wgrad_koff_bytes(32) +
                      (size_t)padded * es;
  return padded < INT32_MAX / 2 && smem <= 200 * 1024 && O * pg.OH * pg.OW < INT32_MAX / 2;
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
                           bool* done, uint8_t* pool_idx = nullptr) {
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
                               : conv_fwd_gemm(ctx, x, (const float*)ws, pitch, bias, y, g, rows, act, done, pool_idx);
  release(ctx, ws);
  return err;
}

static char* conv_fwd_implicit(gt_ctx* ctx, const float* x, const float* w, const float* bias, float* y,
                               const gt_geom& g, int64_t O, int act, bool* done, uint8_t* pool_idx = nullptr) {
  return conv_implicit(ctx, x, w, 0, O, g.C * g.KH * g.KW, bias, y, g, act, O, g.C, done, pool_idx);
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


char* gt_conv_fwd_pool(gt_ctx* ctx, int dtype, const void* x, const void* w, const void* bias, void* pooled,
                       uint8_t* idx, const gt_geom* g, const gt_geom* pg, int64_t O, int act) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_conv_fwd_pool"));
  GT_TRY(check_geom(pg, "gt_conv_fwd_pool"));
  if (O <= 0 || !pooled || !idx) return errorf("gt_conv_fwd_pool: bad arguments");
  if (pg->N != g->N || pg->C != O || pg->H != g->OH || pg->W != g->OW || pg->pad != 0)
    return errorf("gt_conv_fwd_pool: the pooling geometry does not take the convolution's output");
  if (pg->stride < pg->KH || pg->stride < pg->KW) return errorf("gt_conv_fwd_pool: windows overlap");
  if (g->N * O * pg->OH * pg->OW == 0) return nullptr;
  const size_t es0 = dtype == GT_FLOAT64 ? 8 : 4;
  // a first convolution (3 x 3 over at most 3 channels): computed directly,
  // timed like the GEMM it replaces (M = positions, N = O, K = C*9)
  if (conv_pool_small_fits(*g, *pg, O, act, es0)) {
    ConvPoolSmallArgs a{ctx, dtype, act == GT_ACT_RELU ? 1 : 0, x, w, bias, pooled, idx, g, pg, O};
    return timed_gemm_like(ctx, g->N * g->OH * g->OW, O, g->C * 9, 7, conv_pool_small_run, &a);
  }
  // 2 x 2 windows at stride 2 that tile the output: pooled in the epilogue
  if (dtype == GT_FLOAT32 && pg->KH == 2 && pg->KW == 2 && pg->stride == 2 && g->OH % 2 == 0 && g->OW % 2 == 0) {
    bool done = false;
    GT_TRY(conv_fwd_implicit(ctx, (const float*)x, (const float*)w, (const float*)bias, (float*)pooled, *g, O, act,
                             &done, idx));
    if (done) return nullptr;
  }
  const size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  void* y = nullptr;
  GT_TRY(scratch(ctx, (size_t)(g->N * O * g->OH * g->OW) * es, &y));
  char* err = gt_conv_fwd(ctx, dtype, x, w, bias, y, g, O, act);
  if (!err) err = gt_maxpool_fwd_idx(ctx, dtype, y, pooled, idx, pg);
  release(ctx, y);
  return err;
}

char* gt_conv_bwd_weight_pool(gt_ctx* ctx, int dtype, const void* x, const void* grad, const uint8_t* idx,
                              const void* pooled, int relu_mask, void* dw, void* db, const gt_geom* g,
                              const gt_geom* pg, int64_t O) {
  GT_ENTER(ctx);
  GT_CHECK_DTYPE(dtype);
  GT_TRY(check_geom(g, "gt_conv_bwd_weight_pool"));
  GT_TRY(check_geom(pg, "gt_conv_bwd_weight_pool"));
  if (O <= 0 || !dw || !grad || !idx) return errorf("gt_conv_bwd_weight_pool: bad arguments");
  if (relu_mask && !pooled) return errorf("gt_conv_bwd_weight_pool: relu_mask needs the pooled output");
  if (pg->N != g->N || pg->C != O || pg->H != g->OH || pg->W != g->OW || pg->pad != 0)
    return errorf("gt_conv_bwd_weight_pool: the pooling geometry does not take the convolution's output");
  if (pg->stride < pg->KH || pg->stride < pg->KW)
    return errorf("gt_conv_bwd_weight_pool: windows overlap; use gt_maxpool_bwd and gt_conv_bwd_weight");
  const int64_t CKK = g->C * g->KH * g->KW, NL = g->N * g->OH * g->OW;
  const size_t es = dtype == GT_FLOAT64 ? 8 : 4;
  if (NL == 0) {
    GT_CUDA(cudaMemsetAsync(dw, 0, O * CKK * es, ctx->stream));
    if (db) GT_CUDA(cudaMemsetAsync(db, 0, O * es, ctx->stream));
    return nullptr;
  }
  if (!pool_wgrad_fits(*g, *pg, O, es)) {  // through the full-resolution output gradient
    void* dy = nullptr;
    GT_TRY(scratch(ctx, (size_t)(g->N * O * g->OH * g->OW) * es, &dy));
    char* err = gt_maxpool_bwd_idx(ctx, dtype, grad, idx, pooled, relu_mask, dy, pg);
    if (!err) err = gt_conv_bwd_weight(ctx, dtype, x, dy, dw, db, g, O);
    release(ctx, dy);
    return err;
  }
  void *part_w = nullptr, *part_b = nullptr;
  GT_TRY(scratch(ctx, (size_t)(g->N * O * CKK) * es, &part_w));
  char* err = scratch(ctx, (size_t)(g->N * O) * es, &part_b);
  PoolWgradArgs a{ctx, dtype, relu_mask ? 1 : 0, x, grad, pooled, idx, g, pg, O, part_w, part_b};
  auto run = [](void* p) -> char* {
    const PoolWgradArgs& a = *(const PoolWgradArgs*)p;
    return a.dtype == GT_FLOAT64 ? pool_wgrad_dispatch<double>(a) : pool_wgrad_dispatch<float>(a);
  };
  // timed like the GEMM it replaces: dW (O, CKK) over every output position
  if (!err) err = timed_gemm_like(ctx, O, CKK, NL, 5, run, &a);
  if (!err) {
    GT_DISPATCH(dtype, {
      column_sums_kernel<T><<<(unsigned)ceil_div(O * CKK, 32), 1024, 0, ctx->stream>>>((const T*)part_w, g->N,
                                                                                      O * CKK, (T*)dw);
      if (db)
        column_sums_kernel<T><<<(unsigned)ceil_div(O, 32), 1024, 0, ctx->stream>>>((const T*)part_b, g->N, O,
                                                                                  (T*)db);
    });
    count_launch(db ? 2 : 1);
    cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) err = cuda_error(ce, "column_sums_kernel launch", __FILE__, __LINE__);
  }
  release(ctx, part_w);
  release(ctx, part_b);
  return err;
}

}  // extern "C"
