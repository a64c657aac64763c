/*
 * gt_host.h — C interface of libgotensor_host.so, the native training-step
 * runtime above libgotensor_cuda.so.
 *
 * It runs go-tensor's training loop for a Sequential model,
 *
 *   loss := nn.CrossEntropyLoss(model.Forward(x), y)
 *   opt.ZeroGrad(); loss.Backward(); opt.Step()
 *
 * (examples/mnist/main.go:68-73, nn/nn_mps_test.go:31-36), as a fixed plan of
 * fused kernels instead of a tape of primitives: Linear (+activation) and
 * Conv2d (+ReLU) + MaxPool2d forward in GEMM epilogues, one fused softmax
 * cross-entropy, backward GEMMs with the activation derivative in their
 * epilogue, one optimizer pass over the flat parameter buffer, and (with more
 * than one rank) a bucketed gradient average overlapped with the backward
 * pass. Parameters are laid out flat in Module.Parameters() order
 * (nn/module.go:72-78) and named like nn.NamedParameters ("0.weight",
 * nn/state.go:28-55).
 */
#ifndef GT_HOST_H
#define GT_HOST_H

#include "gt_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct gth_model gth_model;

/* Layer kinds: nn.NewLinear, nn.NewConv2d, nn.NewMaxPool2d, nn.NewReLU,
 * nn.NewTanh, nn.NewSigmoid, nn.NewFlatten, nn.NewDropout. */
enum {
  GTH_LINEAR = 0, GTH_CONV2D, GTH_MAXPOOL2D, GTH_RELU, GTH_TANH, GTH_SIGMOID, GTH_FLATTEN, GTH_DROPOUT
};

/* One layer. Linear: in, out. Conv2d: in, out, kernel, stride, padding
 * (nn/conv.go:19-28). MaxPool2d: kernel, stride (0 = kernel, nn/conv.go:41-48).
 * Dropout: p (only p = 0, the identity, is supported on this path). */
typedef struct {
  int32_t kind;
  int32_t _pad;
  int64_t in, out, kernel, stride, padding;
  double p;
} gth_layer;

/* Builds the plan for a fixed input shape (batch first) and allocates
 * parameters, gradients and activations on ctx's device. Parameters start
 * at zero: load them with gth_set_params. */
GT_API char* gth_model_new(gt_ctx* ctx, int dtype, const gth_layer* layers, int nlayers, const int64_t* input_shape,
                           int ndim, gth_model** out);
GT_API void gth_model_free(gth_model* m);

/* Parameter tensors in Parameters() order. */
GT_API int gth_num_tensors(const gth_model* m);
GT_API int64_t gth_num_params(const gth_model* m);
/* name (NUL-terminated, truncated to name_cap), shape (up to 4 dims), ndim,
 * offset in elements within the flat buffer. */
GT_API char* gth_param_info(const gth_model* m, int i, char* name, int name_cap, int64_t* shape, int* ndim,
                            int64_t* offset);
/* Flat copies of all parameters / gradients, host side, in the model dtype. */
GT_API char* gth_set_params(gth_model* m, const void* host);
GT_API char* gth_get_params(gth_model* m, void* host);
GT_API char* gth_get_grads(gth_model* m, void* host);
/* Device pointers of the flat buffers (for bulk device-side access). */
GT_API void* gth_params_device(gth_model* m);
GT_API void* gth_grads_device(gth_model* m);

/* Optimizer: optim.NewSGD / optim.NewAdam (optim/optim.go:22-106). Resets the
 * optimizer state. */
GT_API char* gth_set_sgd(gth_model* m, const gt_sgd_cfg* cfg);
GT_API char* gth_set_adam(gth_model* m, const gt_adam_cfg* cfg);

/* Device buffers the next step reads: the input batch (input_shape, model
 * dtype) and the labels (batch int32). The model has two such pairs; a step
 * moves on to the other pair only when a batch has been staged into it
 * (gth_stage_batch), so without staging these pointers never change and a
 * batch written once serves every following step. */
GT_API void* gth_input_device(gth_model* m);
GT_API int32_t* gth_labels_device(gth_model* m);
/* Queues the upload of a host batch (x: input_shape in the model dtype,
 * labels: batch int32) on the context's copy stream, into the pair that the
 * first step without a staged batch will read (at most two batches staged).
 * The copy waits for the last step that read that pair and overlaps the step
 * in flight; the step that reads it waits for the copy. Asynchronous for
 * pinned host memory (gt_host_alloc), which must stay unchanged until that
 * step has run. The data loader's host-to-device hop (data/data.go:60-84). */
GT_API char* gth_stage_batch(gth_model* m, const void* x, const int32_t* labels);
/* Device scalar (model dtype) holding the last loss. */
GT_API void* gth_loss_device(gth_model* m);

/* Loss and gradients for the batch in the input buffers (gradients are
 * overwritten, i.e. ZeroGrad + Backward), averaged over ranks when data
 * parallel. Asynchronous. */
GT_API char* gth_forward_backward(gth_model* m);
/* One optimizer update from the current gradients. Asynchronous. */
GT_API char* gth_optimizer_step(gth_model* m);
/* forward_backward + optimizer_step. With graphs enabled, the step is
 * captured once (after its first eager run) and replayed. Asynchronous. */
GT_API char* gth_train_step(gth_model* m);
GT_API char* gth_enable_graph(gth_model* m, int on);
/* Reads the last loss (synchronizes). */
GT_API char* gth_loss(gth_model* m, double* out);
/* Evaluation forward pass (no gradients): logits (batch, classes) to host. */
GT_API char* gth_forward(gth_model* m, void* logits_host);
/* Evaluation of the batch in the input buffers (no gradients), reduced on
 * the device: the model.Forward(x).Argmax() of every row as int32 (batch
 * values to host), or the number of rows whose Argmax equals the label
 * (NoGrad accuracy loop, examples/mnist/main.go:120-133). */
GT_API char* gth_predict(gth_model* m, int32_t* predictions_host);
GT_API char* gth_count_correct(gth_model* m, int64_t* correct);
/* ---- checkpoints ------------------------------------------------------------
 * The parameters come from (and go to) the device in one copy of the flat
 * buffer, in the model's dtype; the reference goes through float64 host
 * copies of every tensor (Tensor.Float64s).
 *
 * safetensors.Save(path, nn.StateDict(m), dtype, metadata)
 * (weights/safetensors/safetensors.go:116-175): the same bytes; dtype is "F32"
 * or "F64"; n_meta key/value strings (or none). */
GT_API char* gth_save_safetensors(gth_model* m, const char* path, const char* dtype, const char* const* meta_keys,
                                  const char* const* meta_values, int n_meta);
/* safetensors.Load(path) + nn.LoadStateDict(m, sd, strict)
 * (safetensors.go:55-100, nn/state.go:84-126): every dtype of the format, the
 * reference's checks and error messages; all or nothing. */
GT_API char* gth_load_safetensors(gth_model* m, const char* path, int strict);
/* nn.SaveFile / nn.LoadFile (nn/serialize.go:11-89): GOTN v1, parameters by
 * position as float64. Loading applies nothing unless the whole file is
 * read (the reference copies parameter by parameter as it reads). */
GT_API char* gth_save_gotn(gth_model* m, const char* path);
GT_API char* gth_load_gotn(gth_model* m, const char* path);
/* One tensor of a safetensors file as float64 (safetensors.Load for one
 * name): *numel values into out (cap of them; NULL to query), its shape into
 * shape (up to shape_cap dims) and *ndim. A scalar (shape []) holds one value.
 * Host only. */
GT_API char* gth_safetensors_read(const char* path, const char* name, double* out, int64_t cap, int64_t* shape,
                                  int shape_cap, int* ndim, int64_t* numel);
/* The "__metadata__" value for key (NUL-terminated, truncated to cap - 1
 * bytes; *len = its full length). Host only. */
GT_API char* gth_safetensors_metadata(const char* path, const char* key, char* value, int cap, int* len);

/* Number of GPU kernel launches one training step issues (the plan's size). */
GT_API int gth_step_launches(const gth_model* m);

/* Data parallelism: joins a communicator of `world` ranks (one GPU each) and
 * splits the gradient buffer into buckets of about bucket_bytes, averaged as
 * soon as the backward pass has finished them. */
GT_API char* gth_dp_init(gth_model* m, int rank, int world, const unsigned char id[128], int timeout_ms,
                         int64_t bucket_bytes);

/* The bucket plan for parameter tensors of the given sizes (elements, in
 * Parameters() order): buckets are contiguous element ranges of the flat
 * buffer filled from its end (the order in which backward produces
 * gradients), closing once they hold at least bucket_elems elements and only
 * at tensor boundaries. Writes (lo, hi) pairs, last bucket of the buffer
 * first; returns the bucket count, or -1 if cap is too small. Host only. */
GT_API int gth_bucket_plan(const int64_t* sizes, int n, int64_t bucket_elems, int64_t* bounds, int cap);

/* The row-chunk split of the bucket that starts at the first Linear's weight
 * (element offset w_off, N rows of K elements), for a data-parallel step that
 * computes that weight gradient in row chunks and averages each chunk while
 * the next is computed (GT_DP_LAST_CHUNKS). bounds: nb (lo, hi) pairs from
 * gth_bucket_plan. Writes the chunk row boundaries (0, ..., N; chunks of a
 * multiple of 256 rows, or of 32 for small layers) to rows and the new bucket
 * list to out_bounds (*out_nb pairs): the chunk buckets replace that bucket,
 * highest rows first, and the first of them also holds the rest of the
 * original bucket after the weight (the bias). Returns the number of row
 * boundaries, or 0 when nothing is split (no such bucket, one chunk, or a
 * capacity too small). No counterpart in the reference. Host only. */
GT_API int gth_row_chunk_plan(const int64_t* bounds, int nb, int64_t w_off, int64_t N, int64_t K, int chunks,
                              int64_t* rows, int rows_cap, int64_t* out_bounds, int out_cap, int* out_nb);

#ifdef __cplusplus
}
#endif

#endif /* GT_HOST_H */
