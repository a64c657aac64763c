// Native training-step runtime for go-tensor Sequential models on B200.
//
// A Model turns the layer list of an nn.Sequential into a fixed plan of
// fused kernel calls on libgotensor_cuda's C interface and owns every device
// buffer the step touches. The only allocations inside a step are kernel
// scratch from the stream-ordered pool, which stream capture records as
// graph memory nodes, so a step can be captured into one CUDA graph.
#pragma once

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "gt_cuda.h"
#include "gt_host.h"

namespace gotensor {

class Error : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

// Throws the message of a failed gt_* call (and frees it).
inline void check(char* err) {
  if (err) {
    std::string msg(err);
    gt_free_error(err);
    throw Error(msg);
  }
}

// A device allocation from the context's pool, released on destruction.
class DevBuf {
 public:
  DevBuf() = default;
  DevBuf(gt_ctx* ctx, size_t bytes) : ctx_(ctx), bytes_(bytes) { check(gt_alloc(ctx, bytes, &ptr_)); }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept { *this = std::move(o); }
  DevBuf& operator=(DevBuf&& o) noexcept {
    reset();
    ctx_ = o.ctx_, ptr_ = o.ptr_, bytes_ = o.bytes_;
    o.ptr_ = nullptr;
    return *this;
  }
  ~DevBuf() { reset(); }
  void reset() {
    if (ptr_) gt_free_error(gt_release(ctx_, ptr_));
    ptr_ = nullptr;
  }
  void* get() const { return ptr_; }
  size_t bytes() const { return bytes_; }

 private:
  gt_ctx* ctx_ = nullptr;
  void* ptr_ = nullptr;
  size_t bytes_ = 0;
};

struct ParamInfo {
  std::string name;
  std::vector<int64_t> shape;
  int64_t numel = 0;
  int64_t dense_offset = 0;  // in the host (Parameters()-order, packed) layout
  int64_t dev_offset = 0;    // in the device layout (each tensor 256-byte aligned)
};

struct Op {
  enum Kind { LINEAR, CONV, POOL, ACT, IDENTITY } kind = IDENTITY;
  int layer = -1;               // index in the Sequential of the layer owning the params
  int act = GT_ACT_NONE;        // LINEAR/CONV: fused activation; ACT: the activation
  bool relu_in = false;         // POOL: the input is a ReLU output (mask fused into backward)
  std::vector<int64_t> in_shape, out_shape;
  int64_t M = 0, K = 0, N = 0;  // LINEAR: x (M, K) @ W (N, K)^T
  gt_geom g{};                  // CONV / POOL geometry
  int64_t O = 0;                // CONV output channels
  int64_t w_off = -1, b_off = -1;  // device offsets (elements) of weight and bias
  const void* in = nullptr;     // input activation
  void* out = nullptr;          // output activation
  uint8_t* idx = nullptr;       // POOL: first-max window offsets
  bool needs_dx = true;         // false for the first op with parameters
  bool produces_act = false;    // output is an activation's output (derivative can be fused upstream)
  int src = -1;                 // op that produced this op's input, identities skipped (-1: the batch)
  uint32_t* bits = nullptr;     // LINEAR + ReLU, float32: bit mask of the output for the next Linear's dX
  void* cols = nullptr;         // CONV: the forward's im2col columns, reused by the backward
  // LINEAR: the bias gradient is written by the op that writes this op's
  // output gradient (the loss for the last layer, the next Linear's dX
  // otherwise), as the column sums of that gradient.
  bool db_upstream = false;
  // CONV: index of the MaxPool2d after it whose pooled gradient gives this
  // conv's weight gradient directly (gt_conv_bwd_weight_pool); POOL: its
  // backward is left to that conv.
  int fused_pool = -1;
  bool wgrad_fused = false;
  // CONV: index of the MaxPool2d after it whose output and indices this
  // conv's forward writes (gt_conv_fwd_pool); POOL: its forward is left to
  // that conv.
  int pool_fwd = -1;
  bool fwd_fused = false;
};

class Model {
 public:
  Model(gt_ctx* ctx, int dtype, const std::vector<gth_layer>& layers, const std::vector<int64_t>& input_shape);
  ~Model();

  const std::vector<ParamInfo>& params() const { return params_; }
  int64_t num_params() const { return dense_params_; }
  void set_params(const void* host);
  void get_params(void* host);
  void get_grads(void* host);
  void* params_device() const { return params_.empty() ? nullptr : pbuf_.get(); }
  void* grads_device() const { return params_.empty() ? nullptr : gbuf_.get(); }

  void set_sgd(const gt_sgd_cfg& cfg);
  void set_adam(const gt_adam_cfg& cfg);

  // The input and label buffers the next step reads.
  void* input_device() const { return input_[cur_].get(); }
  int32_t* labels_device() const { return (int32_t*)labels_[cur_].get(); }
  void* loss_device() const { return loss_.get(); }
  // Queues the upload of a batch on the copy stream into the buffer pair
  // that the first step without a staged batch will read.
  void stage_batch(const void* x, const int32_t* labels);

  void forward_backward();
  void optimizer_step();
  void train_step();
  void enable_graph(bool on);
  double loss();
  void forward_eval(void* logits_host);
  // Evaluation reduced on the device: per-row Argmax to host (if preds) and
  // the number of rows whose Argmax equals the label (if correct).
  void predict(int32_t* preds, int64_t* correct);
  // Checkpoints (checkpoint.cpp): safetensors by name, GOTN v1 by position.
  void save_safetensors(const std::string& path, const std::string& dtype,
                        const std::vector<std::pair<std::string, std::string>>& metadata);
  void load_safetensors(const std::string& path, bool strict);
  void save_gotn(const std::string& path);
  void load_gotn(const std::string& path);
  int step_launches() const { return launches_; }

  void dp_init(int rank, int world, const unsigned char id[128], int timeout_ms, int64_t bucket_bytes);

 private:
  void plan(const std::vector<gth_layer>& layers, const std::vector<int64_t>& input_shape);
  void forward();
  // join: the compute stream waits for the gradient all-reduce before
  // returning (else the optimizer waits bucket by bucket).
  void backward(bool join = true);
  void issue_ready_buckets(int64_t boundary);
  void drop_graph();
  void bind_input(int p);  // points the plan at input/label buffer pair p
  void begin_read();       // before a step reads pair cur_: wait for its staged upload
  void end_read();         // after it: the pair is free once the step is done; move to a staged pair

  gt_ctx* ctx_;
  int dtype_;
  size_t es_;
  int64_t batch_ = 0, classes_ = 0;
  std::vector<Op> ops_;
  int first_param_op_ = -1;  // backward stops here: nothing before it needs gradients
  std::vector<ParamInfo> params_;
  int64_t dense_params_ = 0, dev_params_ = 0;
  std::vector<DevBuf> acts_;  // activation buffers owned by ops
  std::vector<DevBuf> bits_;  // ReLU bit masks (Op::bits)
  std::vector<DevBuf> cols_;  // conv columns (Op::cols)
  // Data parallel: row boundaries of the first layer's weight gradient,
  // computed chunk by chunk so each chunk's bucket is averaged while the
  // next chunk is computed (empty: one GEMM).
  std::vector<int64_t> first_rows_;
  DevBuf pbuf_, gbuf_, opt_a_, opt_b_, step_dev_;
  // Two input/label buffer pairs: while a step reads one, the next batch can
  // be uploaded into the other on the copy stream.
  DevBuf input_[2], labels_[2];
  int cur_ = 0;                      // pair the next step reads
  bool staged_[2] = {false, false};  // an upload into the pair is queued and not yet waited for
  gt_event* ready_[2] = {};          // copy stream: the pair's upload is done
  gt_event* free_[2] = {};           // compute stream: the last step reading the pair is done
  std::vector<std::pair<int, int>> input_refs_;  // (op, 0 = in / 1 = out) that point at the input
  int64_t input_bytes_ = 0;
  DevBuf loss_, grad_a_, grad_b_;
  DevBuf pred_, count_;  // evaluation outputs (allocated on first use)
  // Pinned host copy of the flat parameter buffer in the device layout, for
  // checkpoints (allocated on first use, kept for the next).
  void* staging_ = nullptr;
  char* param_staging();
  int64_t grad_elems_ = 0;

  enum { OPT_NONE, OPT_SGD, OPT_ADAM } opt_ = OPT_NONE;
  gt_sgd_cfg sgd_{};
  gt_adam_cfg adam_{};
  int64_t opt_steps_ = 0;

  int rank_ = 0, world_ = 1;
  int sm_reserve_ = 0;  // SMs left to the all-reduce while it overlaps backward GEMMs
  std::vector<std::pair<int64_t, int64_t>> buckets_;  // device element ranges, last first
  std::vector<gt_event*> bucket_done_;                 // comm stream: bucket i's all-reduce is done
  size_t next_bucket_ = 0;
  void free_bucket_events();

  bool use_graph_ = false;
  gt_graph* graph_[2] = {};  // the captured step for each input pair
  int launches_ = 0;
};

}  // namespace gotensor
