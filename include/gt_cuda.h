/*
 * gt_cuda.h — C interface of libgotensor_cuda.so, the B200 (sm_100a) backend
 * for go-tensor.
 *
 * This is the boundary a Go `internal/cuda` package binds over cgo to
 * implement `backend.Backend` (internal/backend/backend.go:130-157) for
 * `tensor.CUDA(i)`. It has the shape of the Metal backend's C interface
 * (internal/mps/mps.h): plain pointers and sizes, op codes that equal the Go
 * enums, and `char*` error messages (NULL on success) that the caller frees
 * with gt_free_error. Every entry point is non-blocking unless it says
 * otherwise: work is queued on the context's stream, and asynchronous kernel
 * faults surface at the next gt_sync, like mps_sync.
 *
 * Device buffers are raw device pointers from gt_alloc. Element counts and
 * offsets are in elements of the call's dtype unless a name ends in _bytes.
 */
#ifndef GT_CUDA_H
#define GT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define GT_API __attribute__((visibility("default")))
#else
#define GT_API
#endif

#define GT_MAX_DIMS 8 /* backend.MaxDims, internal/backend/backend.go:109 */

/* Per-device context: stream, communicator and the device's stream-ordered
 * memory pool. One per (process, device). */
typedef struct gt_ctx gt_ctx;

/* backend.DType (internal/backend/backend.go:10-15). */
enum { GT_FLOAT32 = 0, GT_FLOAT64 = 1 };

/* backend.UnaryOp (internal/backend/backend.go:71-88). */
enum {
  GT_NEG = 0, GT_EXP, GT_LOG, GT_SQRT, GT_ABS, GT_RELU, GT_SIGMOID, GT_TANH,
  GT_SIGN, GT_STEP, GT_ADD_SCALAR, GT_MUL_SCALAR, GT_POW
};
/* backend.BinaryOp (internal/backend/backend.go:90-98). */
enum { GT_ADD = 0, GT_SUB, GT_MUL, GT_DIV };
/* backend.ReduceOp (internal/backend/backend.go:100-106). */
enum { GT_SUM = 0, GT_MAX };
/* Activation fused into an epilogue or prologue (nn.NewReLU/NewTanh/NewSigmoid,
 * nn/module.go:86-93). */
enum { GT_ACT_NONE = 0, GT_ACT_RELU = 1, GT_ACT_TANH = 2, GT_ACT_SIGMOID = 3 };

/* backend.View (internal/backend/backend.go:111-117): element idx (row-major
 * over shape) is at offset + sum(idx[d]*strides[d]); stride 0 broadcasts.
 * Same layout as mps_view (internal/mps/mps.h:8-13) widened to 64 bits. */
typedef struct {
  int32_t ndim;
  int32_t _pad;
  int64_t offset;
  int64_t shape[GT_MAX_DIMS];
  int64_t strides[GT_MAX_DIMS];
} gt_view;

/* backend.ConvGeom (internal/backend/backend.go:119-125); mps_geom
 * (internal/mps/mps.h:15-18) widened to 64 bits. */
typedef struct {
  int64_t N, C, H, W, KH, KW, OH, OW, stride, pad;
} gt_geom;

/* ---- context and errors -------------------------------------------------- */

/* Opens device `device`: stream, memory pool, kernel attributes. Replaces
 * mps_init (internal/mps/mps.h:20-21) and the per-device factory that
 * tensor/device.go registers (registerBackend, 68-72) and instantiates lazily
 * (backendFor, 74-95). */
GT_API char* gt_init(int device, gt_ctx** out);
/* Frees every resource of the context (communicator, stream). */
GT_API char* gt_destroy(gt_ctx* ctx);
/* Frees an error message returned by any gt_* call. */
GT_API void gt_free_error(char* msg);
/* Device name, e.g. "NVIDIA B200"; mps_device_name (internal/mps/mps.h:22). */
GT_API const char* gt_device_name(const gt_ctx* ctx);
/* Device ordinal and SM count. */
GT_API int gt_device_index(const gt_ctx* ctx);
GT_API int gt_sm_count(const gt_ctx* ctx);
/* The context's CUDA stream (a cudaStream_t), for interoperation. */
GT_API void* gt_stream(gt_ctx* ctx);
/* Waits for all queued work; returns any asynchronous fault. Backend.Sync
 * (internal/backend/backend.go:140), mps_sync (internal/mps/mps.h:31). */
GT_API char* gt_sync(gt_ctx* ctx);

/* ---- memory: Backend.Zeros/FromHost/ToHost/Cast/Write (backend.go:134-139) */

/* Stream-ordered allocation from the device's caching pool; mps_alloc
 * (internal/mps/mps.h:25). */
GT_API char* gt_alloc(gt_ctx* ctx, size_t bytes, void** out);
/* Returns a buffer to the pool, ordered after the work already queued;
 * mps_release (internal/mps/mps.h:28). */
GT_API char* gt_release(gt_ctx* ctx, void* ptr);
/* Bytes of the context's memory pool in use by live allocations and bytes the
 * pool holds from the device (in use plus cached), as of the work queued so
 * far; a diagnostic for callers that budget device memory. No counterpart in
 * the reference. */
GT_API char* gt_pool_usage(gt_ctx* ctx, uint64_t* used_bytes, uint64_t* reserved_bytes);
/* mps_zero (internal/mps/mps.h:27); Backend.Zeros = gt_alloc + gt_zero. */
GT_API char* gt_zero(gt_ctx* ctx, void* dst, size_t bytes);
/* Host -> device copy; Backend.FromHost (mps_alloc_copy, mps.h:26). The host
 * buffer may be reused as soon as the call returns. */
GT_API char* gt_upload(gt_ctx* ctx, void* dst, const void* src, size_t bytes);
/* Device -> host copy after all queued work; Backend.ToHost. Blocking. */
GT_API char* gt_download(gt_ctx* ctx, void* dst, const void* src, size_t bytes);
/* Host <-> device copies that stay ordered on the stream without blocking,
 * for pinned host memory (cudaHostAlloc'd by the caller). */
GT_API char* gt_upload_async(gt_ctx* ctx, void* dst, const void* src, size_t bytes);
GT_API char* gt_download_async(gt_ctx* ctx, void* dst, const void* src, size_t bytes);
/* dst[dst_offset_bytes : +bytes] = src[0 : bytes]; Backend.Write
 * (internal/backend/backend.go:139), mps_write (internal/mps/mps.h:50). */
GT_API char* gt_write(gt_ctx* ctx, void* dst, size_t dst_offset_bytes, const void* src, size_t bytes);
/* y = dtype-converted x, n elements; Backend.Cast (internal/cpu/cpu.go:75-90). */
GT_API char* gt_cast(gt_ctx* ctx, const void* x, int from_dtype, void* y, int to_dtype, int64_t n);

/* ---- element-wise, reductions, linear algebra, convolution helpers -------- */

/* y[i] = op(x[i], s), n elements. Backend.Unary (backend.go:142); internal/cpu/
 * cpu.go:103-167 (transcendentals evaluated in float64, then rounded to the
 * dtype; the scalar is rounded to the dtype for AddScalar/MulScalar). */
GT_API char* gt_unary(gt_ctx* ctx, int dtype, int op, double s, const void* x, void* y, int64_t n);
/* out (contiguous, over va->shape) = a[va] op b[vb]. Backend.Binary
 * (backend.go:143); internal/cpu/cpu.go:169-231. */
GT_API char* gt_binary(gt_ctx* ctx, int dtype, int op, const void* a, const gt_view* va, const void* b,
                const gt_view* vb, void* out);
/* out (contiguous) = src[v]. Backend.Copy (backend.go:144); cpu.go:246-268. */
GT_API char* gt_copy(gt_ctx* ctx, int dtype, const void* src, const gt_view* v, void* out);
/* Reduces the middle axis of x viewed as (outer, n, inner) into (outer, inner).
 * Backend.Reduce (backend.go:147); cpu.go:270-296. */
GT_API char* gt_reduce(gt_ctx* ctx, int dtype, int op, const void* x, void* out, int64_t outer, int64_t n,
                int64_t inner);
/* c (m, n) = op(a) (m, k) @ op(b) (k, n); a is stored (k, m) when trans_a and b
 * is stored (n, k) when trans_b. Backend.MatMul (backend.go:150);
 * internal/cpu/linalg.go:15-62. float32 runs on tcgen05 tensor cores with
 * 3xTF32 split emulation (fp32 accumulation), float64 on the FP64 pipe. */
GT_API char* gt_matmul(gt_ctx* ctx, int dtype, const void* a, const void* b, void* c, int64_t m, int64_t k,
                int64_t n, int trans_a, int trans_b);
/* Backend.Im2col/Col2im/MaxPool2d/MaxPool2dBackward (backend.go:153-156);
 * internal/cpu/linalg.go:94-191. Col2im and the pool backward gather, in the
 * order the reference scatters, so they are bit-exact. */
GT_API char* gt_im2col(gt_ctx* ctx, int dtype, const void* x, void* cols, const gt_geom* g);
GT_API char* gt_col2im(gt_ctx* ctx, int dtype, const void* cols, void* x, const gt_geom* g);
GT_API char* gt_maxpool_fwd(gt_ctx* ctx, int dtype, const void* x, void* out, const gt_geom* g);
GT_API char* gt_maxpool_bwd(gt_ctx* ctx, int dtype, const void* x, const void* grad, void* dx, const gt_geom* g);

/* ---- fused capability entry points ---------------------------------------
 * Each replaces a chain of Backend primitives that the Go tensor/nn/optim code
 * issues today; the Go side reaches them through optional capability
 * interfaces, so the public Go API does not change. */

/* y (M, N) = act(x (M, K) @ w (N, K)^T + bias (N)); bias may be NULL.
 * Replaces Linear.Forward (nn/module.go:51-53: W.T() copy, MatMul, broadcast
 * Add) and the activation module after it (tensor/ops.go:109-125). */
GT_API char* gt_linear_fwd(gt_ctx* ctx, int dtype, const void* x, const void* w, const void* bias, void* y,
                    int64_t M, int64_t K, int64_t N, int act);
/* dx (M, K) = (dy (M, N) @ w (N, K)) * act'(y_prev), where y_prev (M, K) is the
 * output of activation act_prev applied to this layer's input (NULL/NONE: no
 * factor). Replaces the MatMul backward for the input (tensor/ops.go:321-323),
 * the Permute backward and the previous activation's backward closure
 * (tensor/ops.go:110, 116, 123). */
GT_API char* gt_linear_bwd_data(gt_ctx* ctx, int dtype, const void* dy, const void* w, const void* y_prev,
                         int act_prev, void* dx, int64_t M, int64_t K, int64_t N);
/* ReLU bit masks (no counterpart in the reference, which keeps the ReLU
 * input and multiplies by Step(x), tensor/ops.go:110): for y (M, N), bit
 * m % 32 of word bits[(m / 32) * N + n] is (y[m][n] > 0), the factor the ReLU
 * backward applies; ceil(M / 32) * N words in all. The backward then reads
 * 1 bit per element instead of the 4-byte activation. */
/* bits = (y (M, N) > 0), packed. */
GT_API char* gt_relu_bits(gt_ctx* ctx, int dtype, const void* y, uint32_t* bits, int64_t M, int64_t N);
/* gt_linear_fwd with act = ReLU that also writes the output's bit mask
 * (in the GEMM epilogue on the tensor-core path, else by gt_relu_bits). */
GT_API char* gt_linear_fwd_bits(gt_ctx* ctx, int dtype, const void* x, const void* w, const void* bias, void* y,
                                uint32_t* bits, int64_t M, int64_t K, int64_t N);
/* gt_linear_bwd_data with act_prev = ReLU, the factor Step(y_prev) taken from
 * the bit mask of y_prev (M, K): the same result bit for bit. */
GT_API char* gt_linear_bwd_data_bits(gt_ctx* ctx, int dtype, const void* dy, const void* w, const uint32_t* bits,
                                     void* dx, int64_t M, int64_t K, int64_t N);
/* gt_linear_bwd_data and gt_linear_bwd_data_bits that also write db_prev (K)
 * = the column sums of dx: the bias gradient of the Linear that produced this
 * layer's input (the sumTo of its bias, tensor/ops.go:418-433), which
 * follows from dx alone. On the float32 tensor-core path the GEMM's epilogue
 * sums each 32-row block while storing it and one small kernel adds the
 * blocks, so dx is not read again; elsewhere a reduction over dx follows.
 * No counterpart in the reference (whose backward reduces dy per layer). */
GT_API char* gt_linear_bwd_data_db(gt_ctx* ctx, int dtype, const void* dy, const void* w, const void* y_prev,
                                   int act_prev, void* dx, void* db_prev, int64_t M, int64_t K, int64_t N);
GT_API char* gt_linear_bwd_data_bits_db(gt_ctx* ctx, int dtype, const void* dy, const void* w, const uint32_t* bits,
                                        void* dx, void* db_prev, int64_t M, int64_t K, int64_t N);
/* dw (N, K) = dy (M, N)^T @ x (M, K); db (N) = sum over rows of dy (NULL: skip).
 * Replaces the MatMul backward for the weight (tensor/ops.go:324-326), the
 * Permute backward of W.T() and sumTo for the bias (tensor/ops.go:418-433). */
GT_API char* gt_linear_bwd_weight(gt_ctx* ctx, int dtype, const void* x, const void* dy, void* dw, void* db,
                           int64_t M, int64_t K, int64_t N);
/* Rows [r0, r1) of gt_linear_bwd_weight's dw (no db): a weight gradient
 * computed in row chunks, so that a data-parallel step can start averaging
 * the first chunk while the next is computed. No counterpart in the
 * reference (which computes the whole MatMul backward, tensor/ops.go:324). */
GT_API char* gt_linear_bwd_weight_rows(gt_ctx* ctx, int dtype, const void* x, const void* dy, void* dw, int64_t M,
                                       int64_t K, int64_t N, int64_t r0, int64_t r1);
/* Activation backward on its own: dx = dy * act'(y), n elements
 * (tensor/ops.go:110, 116, 123). */
GT_API char* gt_act_bwd(gt_ctx* ctx, int dtype, int act, const void* dy, const void* y, void* dx, int64_t n);
/* Adds bias (C) over an (N, C, L) tensor and applies act in place. */
GT_API char* gt_bias_act(gt_ctx* ctx, int dtype, void* y, const void* bias, int64_t N, int64_t C, int64_t L,
                  int act);

/* y (N, O, OH, OW) = act(conv2d(x (N, C, H, W), w (O, C, KH, KW)) + bias (O)).
 * Replaces tensor.Conv2d (tensor/conv.go:40-59: Im2col, MatMul with the
 * reshaped transposed weight, Permute, broadcast Add) plus the activation. */
GT_API char* gt_conv_fwd(gt_ctx* ctx, int dtype, const void* x, const void* w, const void* bias, void* y,
                  const gt_geom* g, int64_t out_channels, int act);
/* dx (N, C, H, W) = conv2d backward for the input (the Col2im of dy-patches @ W,
 * tensor/conv.go:29-30 and the MatMul backward before it). */
GT_API char* gt_conv_bwd_data(gt_ctx* ctx, int dtype, const void* dy, const void* w, void* dx, const gt_geom* g,
                       int64_t out_channels);
/* dw (O, C, KH, KW) and db (O) (NULL: skip) of a Conv2d given x and dy. */
GT_API char* gt_conv_bwd_weight(gt_ctx* ctx, int dtype, const void* x, const void* dy, void* dw, void* db,
                         const gt_geom* g, int64_t out_channels);
/* gt_conv_fwd that keeps its im2col columns in cols (N*OH*OW x C*KH*KW
 * elements, owned by the caller) for gt_conv_bwd; the same result. No
 * counterpart in the reference, whose backward closure holds the Im2col
 * tensor the same way (tensor/conv.go:40-59). */
GT_API char* gt_conv_fwd_cols(gt_ctx* ctx, int dtype, const void* x, const void* w, const void* bias, void* y,
                              void* cols, const gt_geom* g, int64_t out_channels, int act);
/* Conv2d backward from the forward's columns: dw, db (NULL: skip) and dx
 * (NULL: skip), with dy rearranged once for both GEMMs. The same results as
 * gt_conv_bwd_weight and gt_conv_bwd_data. */
GT_API char* gt_conv_bwd(gt_ctx* ctx, int dtype, const void* cols, const void* dy, const void* w, void* dx, void* dw,
                         void* db, const gt_geom* g, int64_t out_channels);
/* MaxPool2d forward that also records, per output, the window offset of the
 * first maximum (uint8, kh*KW+kw) — the index the backward pass routes to
 * (internal/cpu/linalg.go:169-183). Non-overlapping windows (stride >= KH, KW)
 * only; KH*KW <= 256. */
GT_API char* gt_maxpool_fwd_idx(gt_ctx* ctx, int dtype, const void* x, void* out, uint8_t* idx, const gt_geom* g);
/* dx = scatter of grad to the recorded maxima, times relu'(pooled output) when
 * relu_mask is set (ReLU before the pool). Writes every element of dx. */
GT_API char* gt_maxpool_bwd_idx(gt_ctx* ctx, int dtype, const void* grad, const uint8_t* idx, const void* pooled,
                         int relu_mask, void* dx, const gt_geom* g);
/* Conv2d [+ ReLU] followed by MaxPool2d (geometry pg, non-overlapping windows):
 * pooled and idx as gt_conv_fwd then gt_maxpool_fwd_idx would give them, bit
 * for bit. For float32 2 x 2 windows at stride 2 on the implicit-GEMM path the
 * pooling runs in the convolution's epilogue and the convolution's output is
 * never stored (the backward needs only the pooled values and the indices:
 * gt_maxpool_bwd_idx, gt_conv_bwd_weight_pool); otherwise the output goes
 * through scratch memory. act is GT_ACT_NONE or GT_ACT_RELU on the fused path.
 * No counterpart in the reference (tensor/conv.go:40-70 runs the two ops). */
GT_API char* gt_conv_fwd_pool(gt_ctx* ctx, int dtype, const void* x, const void* w, const void* bias, void* pooled,
                              uint8_t* idx, const gt_geom* g, const gt_geom* pg, int64_t out_channels, int act);
/* dw (O, C, KH, KW) and db (O) (NULL: skip) of a Conv2d (geometry g) whose
 * output went through [ReLU ->] MaxPool2d (geometry pg, non-overlapping
 * windows), from the pooled gradient: the same results as
 * gt_maxpool_bwd_idx(grad, idx, pooled, relu_mask, dy, pg) followed by
 * gt_conv_bwd_weight(x, dy, dw, db, g, O), within rounding. For k x k windows
 * at stride k that tile the output, with C*KH*KW <= 32 (a first convolution),
 * the full-resolution gradient dy is never written: only window maxima carry
 * a nonzero term (MaxPool2dBackward, tensor/conv.go:63-70). Other geometries
 * go through dy in scratch memory. No counterpart in the reference. */
GT_API char* gt_conv_bwd_weight_pool(gt_ctx* ctx, int dtype, const void* x, const void* grad, const uint8_t* idx,
                                     const void* pooled, int relu_mask, void* dw, void* db, const gt_geom* g,
                                     const gt_geom* pg, int64_t out_channels);

/* out[r] (int32) = Tensor.Argmax of row r of x (rows x n) (tensor/ops.go:176-192):
 * the first index of the row's maximum, comparing as the reference does
 * (x[j] > x[best], starting from index 0), so a NaN at index 0 is returned and
 * a NaN elsewhere is never chosen. n >= 1. */
GT_API char* gt_argmax_rows(gt_ctx* ctx, int dtype, const void* x, int64_t rows, int64_t n, int32_t* out);
/* *count (device int64, overwritten) = number of i < n with a[i] == b[i]: the
 * correct-prediction count of the reference's accuracy loop
 * (examples/mnist/main.go:120-133), computed without copying predictions to
 * the host. */
GT_API char* gt_count_equal(gt_ctx* ctx, const int32_t* a, const int32_t* b, int64_t n, int64_t* count);

/* Mean-squared error over n elements: loss (1 element, device) =
 * mean((pred - target)^2) and, if dpred is not NULL, dpred = 2 (pred - target)
 * / n. Replaces MSELoss (nn/loss.go:6-9: Sub, Pow, Mean) and its backward,
 * with the reference's rounding of each intermediate, so dpred equals the
 * tape's bit for bit; n = 0 gives a NaN loss, as Mean of nothing does. */
GT_API char* gt_mse_fwd_bwd(gt_ctx* ctx, int dtype, const void* pred, const void* target, int64_t n, void* loss,
                            void* dpred);
/* Binary cross-entropy of probabilities pred in (0, 1) against targets in
 * [0, 1]: loss = -mean(t log p + (1 - t) log(1 - p)) and, if dpred is not
 * NULL, the gradient the tape forms (t/p and (1 - t)/(1 - p) terms, each
 * scaled by -1/n). Replaces BCELoss (nn/loss.go:17-22) and its backward;
 * the logarithms are evaluated in float64 and rounded, as the reference's
 * Log is. */
GT_API char* gt_bce_fwd_bwd(gt_ctx* ctx, int dtype, const void* pred, const void* target, int64_t n, void* loss,
                            void* dpred);

/* Softmax cross-entropy over logits (B, C) with int32 labels on the device:
 * loss (1 element, device) = -mean_i log softmax(x_i)[y_i] and, if dlogits is
 * not NULL, dlogits = (softmax(x) - onehot(y)) / B. Replaces CrossEntropyLoss
 * (nn/loss.go:12-14: LogSoftmax, host one-hot Pick, Mean, Neg) and its
 * backward, following the reference's rounding of each intermediate.
 * Labels outside [0, C) set *bad_label (device int32, may be NULL) to 1. */
GT_API char* gt_xent_fwd_bwd(gt_ctx* ctx, int dtype, const void* logits, const int32_t* labels, int64_t B,
                      int64_t C, void* loss, void* dlogits, int32_t* bad_label);

/* gt_xent_fwd_bwd that also writes db (C) = the column sums of dlogits: the
 * bias gradient of the Linear that produced the logits (its sumTo over the
 * batch, tensor/ops.go:418-433), summed in the same pass that writes the
 * gradient (rows of up to 1024 classes; wider rows add a reduction over
 * dlogits). dlogits and db must not be NULL. No counterpart in the reference. */
GT_API char* gt_xent_fwd_bwd_db(gt_ctx* ctx, int dtype, const void* logits, const int32_t* labels, int64_t B,
                                int64_t C, void* loss, void* dlogits, void* db, int32_t* bad_label);

/* Largest batch gt_xent_fwd_bwd_noalloc accepts: its per-row loss terms live
 * in a fixed 2 MiB device buffer inside the library (8 bytes per row). */
#define GT_XENT_NOALLOC_MAX_ROWS 262144
/* gt_xent_fwd_bwd for callers that must not allocate device memory during a
 * step, e.g. a host that has already reserved the GPU's memory for its own
 * allocator and cannot let a second pool grow, or one that forbids
 * allocation inside its training loop. Same arguments, same results; no
 * counterpart in the reference (whose backends allocate every result).
 * Instead of pool memory it uses a 2 MiB buffer compiled into this library,
 * which every GPU that loads the library keeps until the process exits.
 * Batches larger than GT_XENT_NOALLOC_MAX_ROWS are rejected with an error.
 * The first call on each device looks up that buffer's device address, so
 * make it before capturing the stream into a graph. The address is kept until
 * the process exits; after a device reset (cudaDeviceReset, which reloads the
 * library's device code) it is stale, so do not call this entry point again
 * after resetting a device it was used on. All calls share the one
 * buffer: two calls that run on the GPU at the same time (different streams
 * or contexts on one device) race and corrupt each other's loss. */
GT_API char* gt_xent_fwd_bwd_noalloc(gt_ctx* ctx, int dtype, const void* logits, const int32_t* labels, int64_t B,
                                     int64_t C, void* loss, void* dlogits, int32_t* bad_label);

/* Optimizer hyperparameters (optim.SGDConfig / optim.AdamConfig,
 * optim/optim.go:22-27, 74-80). */
typedef struct {
  double lr, momentum, weight_decay;
} gt_sgd_cfg;
typedef struct {
  double lr, beta1, beta2, eps, weight_decay;
} gt_adam_cfg;

/* One SGD update over n parameters, in one pass: p, vel updated in place.
 * first != 0 initialises the velocity (the reference's Clone on the first
 * step). Same arithmetic and rounding as SGD.Step (optim/optim.go:48-70). */
GT_API char* gt_sgd_step(gt_ctx* ctx, int dtype, void* p, const void* g, void* vel, int64_t n,
                  const gt_sgd_cfg* cfg, int first);
/* One Adam update (step >= 1) over n parameters in one pass; m and v start at
 * zero. Same arithmetic and rounding as Adam.Step (optim/optim.go:110-132),
 * bias corrections computed in float64 like the reference. */
GT_API char* gt_adam_step(gt_ctx* ctx, int dtype, void* p, const void* g, void* m, void* v, int64_t n,
                   const gt_adam_cfg* cfg, int64_t step);
/* As gt_adam_step but the step number lives on the device (int64, read and
 * incremented by the call's first kernel), so a captured CUDA graph can replay
 * the update. No counterpart in the reference (graph capture). */
GT_API char* gt_adam_step_dev(gt_ctx* ctx, int dtype, void* p, const void* g, void* m, void* v, int64_t n,
                       const gt_adam_cfg* cfg, int64_t* step_dev);

/* ---- data parallelism (no counterpart in the reference) ------------------ */

/* 128-byte unique id for gt_comm_init, made on one rank and shared. */
GT_API char* gt_comm_unique_id(unsigned char id[128]);
/* Joins a communicator of `world` ranks, one per GPU. Fails instead of
 * blocking forever: gives up after timeout_ms. */
GT_API char* gt_comm_init(gt_ctx* ctx, int rank, int world, const unsigned char id[128], int timeout_ms);
/* In-place average over ranks of n elements on the context's stream. */
GT_API char* gt_allreduce_avg(gt_ctx* ctx, int dtype, void* buf, int64_t n);
/* Leaves the communicator (abort when a rank failed, else destroy). */
GT_API char* gt_comm_destroy(gt_ctx* ctx, int abort);
/* Overlapped variant: the average runs on the context's communication stream,
 * after the work queued so far on the compute stream, so later compute
 * (the rest of the backward pass) overlaps it. */
GT_API char* gt_allreduce_avg_async(gt_ctx* ctx, int dtype, void* buf, int64_t n);
/* Makes later compute-stream work wait for every average queued so far. */
GT_API char* gt_comm_wait(gt_ctx* ctx);

/* ---- CUDA graphs (no counterpart in the reference) ------------------------
 * Records the work queued on the context's stream between begin and end into
 * a graph that replays it with one launch (the training step's ~40 kernels).
 * Nothing may synchronize the stream while it records. */
typedef struct gt_graph gt_graph;
GT_API char* gt_capture_begin(gt_ctx* ctx);
GT_API char* gt_capture_end(gt_ctx* ctx, gt_graph** out);
GT_API char* gt_graph_launch(gt_ctx* ctx, gt_graph* graph);
GT_API void gt_graph_free(gt_graph* graph);

/* ---- timing --------------------------------------------------------------- */
/* Device time in milliseconds between two points of the context's stream:
 * gt_mark records a point (slot 0..7), gt_elapsed_ms synchronizes on `to` and
 * returns the interval. */
GT_API char* gt_mark(gt_ctx* ctx, int slot);
GT_API char* gt_elapsed_ms(gt_ctx* ctx, int from, int to, float* ms);

/* GEMM kernels launched on ctx from now on occupy at most sm_count - sms SMs,
 * leaving `sms` free for kernels that run beside them on other streams (the
 * collective kernels of a gradient all-reduce): a persistent GEMM that finds
 * fewer free SMs than it has CTAs runs its remaining tiles in an extra round.
 * 0 (the default) uses every SM. No counterpart in the reference. */
GT_API char* gt_set_gemm_sm_reserve(gt_ctx* ctx, int sms);

/* ---- overlapping uploads ------------------------------------------------- */
/* A context has three streams: compute (every kernel), copy (uploads that
 * overlap compute) and comm (gradient all-reduce). Events order one stream
 * after another, so a host can upload the next batch on the copy stream while
 * the compute stream runs the current step (no counterpart in the reference,
 * whose CPU path has no streams). */
#define GT_STREAM_COMPUTE 0
#define GT_STREAM_COPY 1
#define GT_STREAM_COMM 2
typedef struct gt_event gt_event;
GT_API char* gt_event_new(gt_ctx* ctx, gt_event** out);
GT_API void gt_event_free(gt_event* e);
/* Marks the current end of `stream`'s queued work. */
GT_API char* gt_event_record(gt_ctx* ctx, gt_event* e, int stream);
/* Work queued on `stream` after this call waits for the event's point (an
 * event never recorded is already complete). */
GT_API char* gt_stream_wait_event(gt_ctx* ctx, int stream, gt_event* e);
/* Host -> device copy queued on `stream`; asynchronous for pinned host
 * memory (gt_host_alloc), which must stay unchanged until the copy is done. */
GT_API char* gt_upload_on(gt_ctx* ctx, int stream, void* dst, const void* src, size_t bytes);
/* Page-locked host memory for asynchronous uploads and downloads. */
GT_API char* gt_host_alloc(size_t bytes, void** out);
GT_API void gt_host_free(void* p);

/* Number of kernels this library has launched (or recorded into a graph) in
 * the process so far. */
GT_API int64_t gt_launch_count(void);

/* Per-launch device times of the GEMM kernels issued on ctx (no counterpart
 * in the reference; instrumentation for measuring the hot kernel inside a
 * real step). While a timer is on, every GEMM launched on ctx's stream
 * outside graph capture is bracketed by two CUDA events on that stream, up to
 * `capacity` launches (later ones are counted as dropped, not timed).
 * gt_gemm_timer_start replaces any earlier timer; gt_gemm_timer_read
 * synchronizes on launch i's end event and returns its shape (M, N, K of
 * C[M,N] += A[M,K] B[K,N]), its path (1 SIMT, 2 tcgen05) and its duration.
 * gt_destroy stops the timer. */
GT_API char* gt_gemm_timer_start(gt_ctx* ctx, int64_t capacity);
GT_API char* gt_gemm_timer_stop(gt_ctx* ctx);
GT_API char* gt_gemm_timer_count(gt_ctx* ctx, int64_t* launches, int64_t* dropped);
GT_API char* gt_gemm_timer_read(gt_ctx* ctx, int64_t i, int64_t mnk[3], int* path, float* ms);

/* ---- testing -------------------------------------------------------------- */
/* Pins the float32 GEMM path: 0 automatic, 1 SIMT only, 2 tcgen05 only (shapes
 * that do not qualify then fail). Process-wide; for tests and benchmarks. */
GT_API void gt_debug_set_gemm_path(int path);
/* Pins the number of K-splits of tcgen05 GEMMs (0: chosen per shape). A GEMM
 * with S > 1 splits computes S partial products over consecutive K ranges and
 * sums them in order with its epilogue. Process-wide; for tests. */
GT_API void gt_debug_set_gemm_splits(int splits);
/* Every mbarrier wait of the tcgen05 GEMM gives up after this many
 * microseconds (0: the default, 2 s), records the waiting site in an error
 * word that the next gt_sync reports, and the kernel returns. Process-wide;
 * for tests of that error path. */
GT_API void gt_debug_set_tc_wait_limit_us(int64_t us);
/* Arms a one-shot fault for the next tcgen05 GEMM launch: one splitter warp
 * of each SM pair withholds its arrival for the first K-slice, so the MMA
 * issuer's wait for that slice runs out. Every other wait then runs out too,
 * the kernel frees its tensor memory and returns, and gt_sync reports the
 * timed-out site; the context stays usable. For tests of the error path. */
GT_API void gt_debug_tc_withhold_arrive(void);
/* The path the most recent float32 GEMM took: 1 SIMT, 2 tcgen05 (0: none yet). */
GT_API int gt_gemm_path_taken(void);

#ifdef __cplusplus
}
#endif

#endif /* GT_CUDA_H */
