// Plan construction and execution of the fused training step.
//
// Forward, for the layer patterns of go-tensor's Sequential models:
//   Linear [+ ReLU|Tanh|Sigmoid]        -> gt_linear_fwd (bias + act in the epilogue)
//   Conv2d [+ ReLU]                     -> gt_conv_fwd (bias + act fused)
//   MaxPool2d                           -> gt_maxpool_fwd_idx (value + first-max index)
//   standalone activation               -> gt_unary
//   Flatten, Dropout(p = 0)             -> no kernel (a view of the same buffer)
// then gt_xent_fwd_bwd for CrossEntropyLoss.
//
// Backward walks the plan in reverse. A Linear's input-gradient GEMM applies
// the derivative of the activation that produced its input in its epilogue
// (tensor/ops.go:110-123 folded into the GEMM), and a pool whose input came
// from a ReLU routes the gradient and applies the ReLU mask in one pass.
// Weight gradients land in one flat buffer laid out in Parameters() order; with
// data parallelism each bucket of it is averaged across ranks as soon as the
// backward pass has written it, overlapping the remaining backward GEMMs.
#include "model.hpp"

#include <algorithm>
#include <cstdlib>
#include <cstring>

namespace gotensor {

namespace {

int64_t numel(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (auto d : s) n *= d;
  return n;
}

int act_of(int32_t kind) {
  switch (kind) {
    case GTH_RELU: return GT_ACT_RELU;
    case GTH_TANH: return GT_ACT_TANH;
    case GTH_SIGMOID: return GT_ACT_SIGMOID;
    default: return GT_ACT_NONE;
  }
}

int unary_of(int act) {
  switch (act) {
    case GT_ACT_RELU: return GT_RELU;
    case GT_ACT_TANH: return GT_TANH;
    default: return GT_SIGMOID;
  }
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::string out = "[";
  for (size_t i = 0; i < s.size(); i++) out += (i ? " " : "") + std::to_string(s[i]);
  return out + "]";
}

constexpr int64_t kAlignElems = 64;  // every parameter tensor starts on a 256-byte boundary

}  // namespace

Model::Model(gt_ctx* ctx, int dtype, const std::vector<gth_layer>& layers, const std::vector<int64_t>& input_shape)
    : ctx_(ctx), dtype_(dtype), es_(dtype == GT_FLOAT64 ? 8 : 4) {
  if (dtype != GT_FLOAT32 && dtype != GT_FLOAT64) throw Error("gth_model_new: unknown dtype");
  if (input_shape.empty() || input_shape[0] <= 0) throw Error("gth_model_new: input shape needs a batch dimension");
  plan(layers, input_shape);
  for (int p = 0; p < 2; p++) {
    check(gt_event_new(ctx_, &ready_[p]));
    check(gt_event_new(ctx_, &free_[p]));
  }
}

Model::~Model() {
  drop_graph();
  gt_host_free(staging_);
  free_bucket_events();
  for (int p = 0; p < 2; p++) {
    gt_event_free(ready_[p]);
    gt_event_free(free_[p]);
  }
}

void Model::drop_graph() {
  for (auto& g : graph_) {
    if (g) gt_graph_free(g);
    g = nullptr;
  }
}

void Model::bind_input(int p) {
  void* x = input_[p].get();
  for (auto& r : input_refs_) {
    if (r.second == 0)
      ops_[r.first].in = x;
    else
      ops_[r.first].out = x;
  }
}

void Model::begin_read() {
  if (staged_[cur_]) {
    check(gt_stream_wait_event(ctx_, GT_STREAM_COMPUTE, ready_[cur_]));
    staged_[cur_] = false;
  }
  bind_input(cur_);
}

// Records that the step reading pair cur_ has been queued and moves on to the
// other pair if a batch has been staged there; otherwise the next step reads
// the same buffers again (a batch written once serves any number of steps).
void Model::end_read() {
  check(gt_event_record(ctx_, free_[cur_], GT_STREAM_COMPUTE));
  if (staged_[cur_ ^ 1]) cur_ ^= 1;
}

void Model::stage_batch(const void* x, const int32_t* labels) {
  if (!x || !labels) throw Error("gth_stage_batch: null batch");
  const int s = !staged_[cur_] ? cur_ : !staged_[cur_ ^ 1] ? (cur_ ^ 1) : -1;
  if (s < 0) throw Error("gth_stage_batch: two batches are already staged; run a step first");
  check(gt_stream_wait_event(ctx_, GT_STREAM_COPY, free_[s]));
  check(gt_upload_on(ctx_, GT_STREAM_COPY, input_[s].get(), x, input_bytes_));
  check(gt_upload_on(ctx_, GT_STREAM_COPY, labels_[s].get(), labels, batch_ * sizeof(int32_t)));
  check(gt_event_record(ctx_, ready_[s], GT_STREAM_COPY));
  staged_[s] = true;
}

void Model::plan(const std::vector<gth_layer>& layers, const std::vector<int64_t>& input_shape) {
  batch_ = input_shape[0];
  input_bytes_ = numel(input_shape) * es_;
  for (int p = 0; p < 2; p++) {
    input_[p] = DevBuf(ctx_, input_bytes_);
    labels_[p] = DevBuf(ctx_, batch_ * sizeof(int32_t));
  }
  loss_ = DevBuf(ctx_, 64);

  std::vector<int64_t> shape = input_shape;
  const void* cur = input_[0].get();
  bool cur_is_act = false;  // cur holds an activation output
  int cur_act = GT_ACT_NONE;
  bool seen_params = false;
  int cur_src = -1;  // op that produced `cur` (identities skipped); -1 = the batch
  int64_t dev_off = 0, dense_off = 0, max_elems = numel(input_shape);

  auto add_param = [&](int layer, const char* what, std::vector<int64_t> pshape) {
    ParamInfo p;
    p.name = std::to_string(layer) + "." + what;
    p.shape = pshape;
    p.numel = numel(pshape);
    p.dense_offset = dense_off;
    p.dev_offset = dev_off;
    dense_off += p.numel;
    dev_off += (p.numel + kAlignElems - 1) / kAlignElems * kAlignElems;
    params_.push_back(p);
    return p.dev_offset;
  };

  for (size_t i = 0; i < layers.size(); i++) {
    const gth_layer& L = layers[i];
    Op op;
    op.layer = (int)i;
    op.in_shape = shape;
    op.in = cur;
    switch (L.kind) {
      case GTH_LINEAR: {
        if (shape.size() != 2 || shape[1] != L.in)
          throw Error("Linear(" + std::to_string(L.in) + ", " + std::to_string(L.out) + ") got input " +
                      shape_str(shape) + "; flatten first");
        op.kind = Op::LINEAR;
        op.M = shape[0], op.K = L.in, op.N = L.out;
        op.w_off = add_param((int)i, "weight", {L.out, L.in});
        op.b_off = add_param((int)i, "bias", {L.out});
        if (i + 1 < layers.size() && act_of(layers[i + 1].kind) != GT_ACT_NONE) op.act = act_of(layers[++i].kind);
        op.out_shape = {shape[0], L.out};
        break;
      }
      case GTH_CONV2D: {
        if (shape.size() != 4 || shape[1] != L.in)
          throw Error("Conv2d expects (N, " + std::to_string(L.in) + ", H, W), got " + shape_str(shape));
        if (L.stride < 1 || L.padding < 0 || L.kernel < 1) throw Error("Conv2d: bad kernel/stride/padding");
        op.kind = Op::CONV;
        gt_geom& g = op.g;
        g.N = shape[0], g.C = shape[1], g.H = shape[2], g.W = shape[3];
        g.KH = g.KW = L.kernel, g.stride = L.stride, g.pad = L.padding;
        g.OH = (g.H + 2 * g.pad - g.KH) / g.stride + 1;
        g.OW = (g.W + 2 * g.pad - g.KW) / g.stride + 1;
        if (g.OH <= 0 || g.OW <= 0) throw Error("Conv2d: kernel larger than padded input");
        op.O = L.out;
        op.w_off = add_param((int)i, "weight", {L.out, L.in, L.kernel, L.kernel});
        op.b_off = add_param((int)i, "bias", {L.out});
        if (i + 1 < layers.size() && layers[i + 1].kind == GTH_RELU) {
          op.act = GT_ACT_RELU;
          i++;
        }
        op.out_shape = {g.N, L.out, g.OH, g.OW};
        break;
      }
      case GTH_MAXPOOL2D: {
        if (shape.size() != 4) throw Error("MaxPool2d expects (N, C, H, W), got " + shape_str(shape));
        op.kind = Op::POOL;
        int64_t k = L.kernel, s = L.stride ? L.stride : L.kernel;
        gt_geom& g = op.g;
        g.N = shape[0], g.C = shape[1], g.H = shape[2], g.W = shape[3];
        g.KH = g.KW = k, g.stride = s, g.pad = 0;
        g.OH = (g.H - k) / s + 1;
        g.OW = (g.W - k) / s + 1;
        if (g.OH <= 0 || g.OW <= 0 || k > 16) throw Error("MaxPool2d: window larger than input (or than 16)");
        op.relu_in = cur_is_act && cur_act == GT_ACT_RELU;
        op.out_shape = {g.N, g.C, g.OH, g.OW};
        break;
      }
      case GTH_RELU:
      case GTH_TANH:
      case GTH_SIGMOID:
        op.kind = Op::ACT;
        op.act = act_of(L.kind);
        op.out_shape = shape;
        break;
      case GTH_FLATTEN:
        op.kind = Op::IDENTITY;
        op.out_shape = {shape[0], numel(shape) / shape[0]};
        break;
      case GTH_DROPOUT:
        if (L.p != 0) throw Error("Dropout with p > 0 is not on the fused training path");
        op.kind = Op::IDENTITY;
        op.out_shape = shape;
        break;
      default:
        throw Error("unknown layer kind " + std::to_string(L.kind));
    }
    if (op.kind == Op::LINEAR || op.kind == Op::CONV) {
      op.needs_dx = seen_params;
      seen_params = true;
    }
    if (op.kind == Op::IDENTITY) {
      op.out = const_cast<void*>(cur);  // same buffer, new shape
      op.produces_act = cur_is_act;
      op.act = cur_act;
    } else {
      int64_t n = numel(op.out_shape);
      acts_.emplace_back(ctx_, std::max<int64_t>(n, 1) * es_);
      op.out = acts_.back().get();
      if (op.kind == Op::POOL) {
        acts_.emplace_back(ctx_, std::max<int64_t>(n, 1));
        op.idx = (uint8_t*)acts_.back().get();
        // A pool of ReLU outputs outputs ReLU outputs (max of non-negatives).
        op.produces_act = op.relu_in;
        if (op.relu_in) op.act = GT_ACT_RELU;
      } else {
        op.produces_act = op.act != GT_ACT_NONE;
      }
      max_elems = std::max(max_elems, n);
    }
    max_elems = std::max(max_elems, numel(op.in_shape));
    op.src = cur_src;
    if (op.kind != Op::IDENTITY) cur_src = (int)ops_.size();
    if ((op.kind == Op::LINEAR || op.kind == Op::CONV) && first_param_op_ < 0) first_param_op_ = (int)ops_.size();
    cur = op.out;
    cur_is_act = op.produces_act;
    cur_act = op.produces_act ? op.act : GT_ACT_NONE;
    shape = op.out_shape;
    ops_.push_back(op);
  }
  for (size_t i = 0; i < ops_.size(); i++) {  // the ops that read (or alias) the batch
    if (ops_[i].in == input_[0].get()) input_refs_.emplace_back((int)i, 0);
    if (ops_[i].out == input_[0].get()) input_refs_.emplace_back((int)i, 1);
  }
  // A float32 Linear + ReLU whose output feeds a Linear that needs dX also
  // writes the output's sign bits; that dX reads them instead of the output.
  if (dtype_ == GT_FLOAT32)
    for (auto& op : ops_) {
      if (op.kind != Op::LINEAR || !op.needs_dx || op.src < 0) continue;
      Op& src = ops_[op.src];
      if (src.kind != Op::LINEAR || src.act != GT_ACT_RELU || src.bits) continue;
      bits_.emplace_back(ctx_, (size_t)((src.M + 31) / 32) * (size_t)src.N * sizeof(uint32_t));
      src.bits = (uint32_t*)bits_.back().get();
    }
  // Bias gradients computed where the output gradient is written: the last
  // Linear's by the loss (its logits' gradient), a Linear whose output feeds
  // another Linear's dX by that dX GEMM (its output gradient, with the
  // activation's derivative already applied).
  if (!ops_.empty() && ops_.back().kind == Op::LINEAR && ops_.back().act == GT_ACT_NONE)
    ops_.back().db_upstream = true;
  for (auto& op : ops_)
    if (op.kind == Op::LINEAR && op.needs_dx && op.src >= 0 && ops_[op.src].kind == Op::LINEAR)
      ops_[op.src].db_upstream = true;
  // The first conv [+ ReLU] followed by a MaxPool2d with non-overlapping
  // windows: its weight gradient comes straight from the pooled gradient
  // (gt_conv_bwd_weight_pool), and the pool's own backward is skipped.
  for (size_t i = 0; i < ops_.size(); i++) {
    Op& pool = ops_[i];
    if (pool.kind != Op::POOL || pool.src < 0 || pool.g.stride < pool.g.KH || pool.g.stride < pool.g.KW) continue;
    Op& conv = ops_[pool.src];
    if (conv.kind != Op::CONV || conv.needs_dx) continue;
    if (conv.act != GT_ACT_NONE && !(conv.act == GT_ACT_RELU && pool.relu_in)) continue;
    conv.fused_pool = (int)i;
    pool.wgrad_fused = true;
  }
  // A float32 conv [+ ReLU] followed by a 2 x 2 / stride-2 MaxPool2d writes
  // only the pooled output and its indices (gt_conv_fwd_pool): nothing reads
  // the conv's own output, because the pool's backward takes the ReLU mask
  // from the pooled values.
  if (dtype_ == GT_FLOAT32)
    for (size_t i = 0; i < ops_.size(); i++) {
      Op& pool = ops_[i];
      if (pool.kind != Op::POOL || pool.src < 0 || pool.g.KH != 2 || pool.g.KW != 2 || pool.g.stride != 2) continue;
      Op& conv = ops_[pool.src];
      if (conv.kind != Op::CONV || (conv.act != GT_ACT_NONE && !(conv.act == GT_ACT_RELU && pool.relu_in))) continue;
      conv.pool_fwd = (int)i;
      pool.fwd_fused = true;
    }
  // A float64 conv keeps its forward's im2col columns for its backward; the
  // float32 convs are implicit GEMMs and keep none, nor does a conv whose
  // weight gradient comes from the pooled gradient.
  for (auto& op : ops_) {
    if (op.kind != Op::CONV || dtype_ != GT_FLOAT64 || op.fused_pool >= 0) continue;
    const int64_t rows = op.g.N * op.g.OH * op.g.OW, ckk = op.g.C * op.g.KH * op.g.KW;
    if (rows * ckk == 0) continue;
    cols_.emplace_back(ctx_, (size_t)(rows * ckk) * es_);
    op.cols = cols_.back().get();
  }
  if (shape.size() != 2) throw Error("the model must end in (batch, classes) logits, got " + shape_str(shape));
  if (!seen_params) throw Error("the model has no parameters");
  classes_ = shape[1];
  dense_params_ = dense_off;
  dev_params_ = dev_off;
  pbuf_ = DevBuf(ctx_, dev_params_ * es_);
  gbuf_ = DevBuf(ctx_, dev_params_ * es_);
  check(gt_zero(ctx_, pbuf_.get(), dev_params_ * es_));
  check(gt_zero(ctx_, gbuf_.get(), dev_params_ * es_));
  grad_elems_ = max_elems;
  grad_a_ = DevBuf(ctx_, max_elems * es_);
  grad_b_ = DevBuf(ctx_, max_elems * es_);
  step_dev_ = DevBuf(ctx_, 64);
  check(gt_zero(ctx_, step_dev_.get(), 64));
}

// ---- parameters -------------------------------------------------------------

void Model::set_params(const void* host) {
  drop_graph();
  const char* h = (const char*)host;
  for (auto& p : params_)
    check(gt_upload(ctx_, (char*)pbuf_.get() + p.dev_offset * es_, h + p.dense_offset * es_, p.numel * es_));
}

void Model::get_params(void* host) {
  std::vector<char> tmp(dev_params_ * es_);
  check(gt_download(ctx_, tmp.data(), pbuf_.get(), tmp.size()));
  for (auto& p : params_)
    memcpy((char*)host + p.dense_offset * es_, tmp.data() + p.dev_offset * es_, p.numel * es_);
}

void Model::get_grads(void* host) {
  std::vector<char> tmp(dev_params_ * es_);
  check(gt_download(ctx_, tmp.data(), gbuf_.get(), tmp.size()));
  for (auto& p : params_)
    memcpy((char*)host + p.dense_offset * es_, tmp.data() + p.dev_offset * es_, p.numel * es_);
}

void Model::set_sgd(const gt_sgd_cfg& cfg) {
  drop_graph();
  opt_ = OPT_SGD;
  sgd_ = cfg;
  opt_steps_ = 0;
  opt_b_.reset();
  opt_a_ = DevBuf(ctx_, dev_params_ * es_);  // velocity
  check(gt_zero(ctx_, opt_a_.get(), dev_params_ * es_));
}

void Model::set_adam(const gt_adam_cfg& cfg) {
  drop_graph();
  opt_ = OPT_ADAM;
  adam_ = cfg;
  opt_steps_ = 0;
  opt_a_ = DevBuf(ctx_, dev_params_ * es_);  // m
  opt_b_ = DevBuf(ctx_, dev_params_ * es_);  // v
  check(gt_zero(ctx_, opt_a_.get(), dev_params_ * es_));
  check(gt_zero(ctx_, opt_b_.get(), dev_params_ * es_));
  check(gt_zero(ctx_, step_dev_.get(), 64));
}

// ---- step -------------------------------------------------------------------

void Model::forward() {
  char* p = (char*)pbuf_.get();
  for (auto& op : ops_) {
    switch (op.kind) {
      case Op::LINEAR:
        if (op.bits)
          check(gt_linear_fwd_bits(ctx_, dtype_, op.in, p + op.w_off * es_, p + op.b_off * es_, op.out, op.bits,
                                   op.M, op.K, op.N));
        else
          check(gt_linear_fwd(ctx_, dtype_, op.in, p + op.w_off * es_, p + op.b_off * es_, op.out, op.M, op.K,
                              op.N, op.act));
        break;
      case Op::CONV:
        if (op.pool_fwd >= 0) {  // the pooled output and indices only
          Op& pool = ops_[op.pool_fwd];
          check(gt_conv_fwd_pool(ctx_, dtype_, op.in, p + op.w_off * es_, p + op.b_off * es_, pool.out, pool.idx, &op.g,
                                 &pool.g, op.O, op.act));
        } else if (op.cols)
          check(gt_conv_fwd_cols(ctx_, dtype_, op.in, p + op.w_off * es_, p + op.b_off * es_, op.out, op.cols, &op.g,
                                 op.O, op.act));
        else
          check(gt_conv_fwd(ctx_, dtype_, op.in, p + op.w_off * es_, p + op.b_off * es_, op.out, &op.g, op.O,
                            op.act));
        break;
      case Op::POOL:
        if (!op.fwd_fused) check(gt_maxpool_fwd_idx(ctx_, dtype_, op.in, op.out, op.idx, &op.g));
        break;
      case Op::ACT:
        check(gt_unary(ctx_, dtype_, unary_of(op.act), 0.0, op.in, op.out, numel(op.out_shape)));
        break;
      case Op::IDENTITY:
        break;
    }
  }
}

void Model::issue_ready_buckets(int64_t boundary) {
  if (next_bucket_ == 0 && next_bucket_ < buckets_.size() && buckets_[0].first >= boundary && sm_reserve_ > 0)
    check(gt_set_gemm_sm_reserve(ctx_, sm_reserve_));  // the all-reduce kernels run beside the GEMMs from here
  while (next_bucket_ < buckets_.size() && buckets_[next_bucket_].first >= boundary) {
    auto b = buckets_[next_bucket_];
    check(gt_allreduce_avg_async(ctx_, dtype_, (char*)gbuf_.get() + b.first * es_, b.second - b.first));
    check(gt_event_record(ctx_, bucket_done_[next_bucket_], GT_STREAM_COMM));
    next_bucket_++;
  }
}

void Model::free_bucket_events() {
  for (auto* e : bucket_done_) gt_event_free(e);
  bucket_done_.clear();
}

void Model::backward(bool join) {
  char* p = (char*)pbuf_.get();
  char* gr = (char*)gbuf_.get();
  // Invariant: g is the gradient w.r.t. the output of op i; g_pre says the
  // derivative of the activation that produced that output is already in it.
  void* g = grad_a_.get();
  void* spare = grad_b_.get();
  if (ops_.back().db_upstream)  // the last Linear's bias gradient in the same pass
    check(gt_xent_fwd_bwd_db(ctx_, dtype_, ops_.back().out, labels_device(), batch_, classes_, loss_.get(), g,
                             gr + ops_.back().b_off * es_, nullptr));
  else
    check(gt_xent_fwd_bwd(ctx_, dtype_, ops_.back().out, labels_device(), batch_, classes_, loss_.get(), g, nullptr));
  bool g_pre = false;
  next_bucket_ = 0;
  for (int i = (int)ops_.size() - 1; i >= first_param_op_; i--) {
    Op& op = ops_[i];
    const bool has_act = (op.kind == Op::LINEAR || op.kind == Op::CONV || op.kind == Op::ACT) && op.act != GT_ACT_NONE;
    if (has_act && !g_pre) check(gt_act_bwd(ctx_, dtype_, op.act, g, op.out, g, numel(op.out_shape)));
    if (op.kind != Op::IDENTITY) g_pre = false;  // g is now w.r.t. the op's pre-activation / input
    switch (op.kind) {
      case Op::LINEAR: {
        if (world_ > 1 && i == first_param_op_ && !first_rows_.empty()) {
          // db first: it sits in the bucket of the first chunk issued
          if (!op.db_upstream) check(gt_reduce(ctx_, dtype_, GT_SUM, g, gr + op.b_off * es_, 1, op.M, op.N));
          for (size_t j = first_rows_.size() - 1; j-- > 0;) {
            check(gt_linear_bwd_weight_rows(ctx_, dtype_, op.in, g, gr + op.w_off * es_, op.M, op.K, op.N,
                                            first_rows_[j], first_rows_[j + 1]));
            issue_ready_buckets(op.w_off + first_rows_[j] * op.K);
          }
        } else {
          check(gt_linear_bwd_weight(ctx_, dtype_, op.in, g, gr + op.w_off * es_,
                                     op.db_upstream ? nullptr : gr + op.b_off * es_, op.M, op.K, op.N));
          if (world_ > 1) issue_ready_buckets(op.w_off);
        }
        if (op.needs_dx) {
          // Fold the derivative of the activation that produced this input
          // into the GEMM epilogue when the producer is a Linear/Conv/act.
          const Op* src = op.src >= 0 ? &ops_[op.src] : nullptr;
          bool fuse = src && src->kind != Op::POOL && src->act != GT_ACT_NONE;
          // the producer's bias gradient from this dX (its output gradient)
          void* db_prev = src && src->kind == Op::LINEAR && src->db_upstream ? gr + src->b_off * es_ : nullptr;
          if (fuse && src->bits && db_prev)
            check(gt_linear_bwd_data_bits_db(ctx_, dtype_, g, p + op.w_off * es_, src->bits, spare, db_prev, op.M,
                                             op.K, op.N));
          else if (fuse && src->bits)
            check(gt_linear_bwd_data_bits(ctx_, dtype_, g, p + op.w_off * es_, src->bits, spare, op.M, op.K, op.N));
          else if (db_prev)
            check(gt_linear_bwd_data_db(ctx_, dtype_, g, p + op.w_off * es_, fuse ? op.in : nullptr,
                                        fuse ? src->act : GT_ACT_NONE, spare, db_prev, op.M, op.K, op.N));
          else
            check(gt_linear_bwd_data(ctx_, dtype_, g, p + op.w_off * es_, fuse ? op.in : nullptr,
                                     fuse ? src->act : GT_ACT_NONE, spare, op.M, op.K, op.N));
          std::swap(g, spare);
          g_pre = fuse;
        }
        break;
      }
      case Op::CONV:
        if (op.fused_pool >= 0) {  // g is the pooled gradient; no dx (first conv)
          const Op& pool = ops_[op.fused_pool];
          check(gt_conv_bwd_weight_pool(ctx_, dtype_, op.in, g, pool.idx, pool.out, pool.relu_in ? 1 : 0,
                                        gr + op.w_off * es_, gr + op.b_off * es_, &op.g, &pool.g, op.O));
          if (world_ > 1) issue_ready_buckets(op.w_off);
          break;
        }
        if (!op.cols) {  // float32 (implicit GEMMs from x and dy), or no output positions
          check(gt_conv_bwd_weight(ctx_, dtype_, op.in, g, gr + op.w_off * es_, gr + op.b_off * es_, &op.g, op.O));
          if (world_ > 1) issue_ready_buckets(op.w_off);
          if (op.needs_dx) {
            check(gt_conv_bwd_data(ctx_, dtype_, g, p + op.w_off * es_, spare, &op.g, op.O));
            std::swap(g, spare);
          }
          break;
        }
        if (world_ == 1) {  // one call: dy rearranged once for dW and dX
          check(gt_conv_bwd(ctx_, dtype_, op.cols, g, p + op.w_off * es_, op.needs_dx ? spare : nullptr,
                            gr + op.w_off * es_, gr + op.b_off * es_, &op.g, op.O));
        } else {  // the bucket goes out before dX is computed
          check(gt_conv_bwd(ctx_, dtype_, op.cols, g, p + op.w_off * es_, nullptr, gr + op.w_off * es_,
                            gr + op.b_off * es_, &op.g, op.O));
          issue_ready_buckets(op.w_off);
          if (op.needs_dx) check(gt_conv_bwd_data(ctx_, dtype_, g, p + op.w_off * es_, spare, &op.g, op.O));
        }
        if (op.needs_dx) std::swap(g, spare);
        break;
      case Op::POOL:
        if (op.wgrad_fused) {  // the conv before takes g as it is (ReLU mask included)
          g_pre = op.relu_in;
          break;
        }
        if (op.g.stride >= op.g.KH && op.g.stride >= op.g.KW) {
          // Routes g to each window's first maximum; with relu_in the ReLU
          // mask of the producer is applied in the same pass.
          check(gt_maxpool_bwd_idx(ctx_, dtype_, g, op.idx, op.out, op.relu_in ? 1 : 0, spare, &op.g));
          g_pre = op.relu_in;
        } else {
          check(gt_maxpool_bwd(ctx_, dtype_, op.in, g, spare, &op.g));
        }
        std::swap(g, spare);
        break;
      case Op::ACT:      // derivative applied above
      case Op::IDENTITY:  // same buffer, g_pre carried through
        break;
    }
  }
  if (world_ > 1) {
    issue_ready_buckets(0);
    if (sm_reserve_ > 0) check(gt_set_gemm_sm_reserve(ctx_, 0));
    check(gt_allreduce_avg_async(ctx_, dtype_, loss_.get(), 1));
    if (join) check(gt_comm_wait(ctx_));
  }
}

void Model::forward_backward() {
  begin_read();
  forward();
  backward();
  end_read();
}

void Model::optimizer_step() {
  if (opt_ == OPT_NONE) throw Error("no optimizer: call gth_set_sgd or gth_set_adam");
  if (opt_ == OPT_SGD && world_ > 1 && !bucket_done_.empty()) {
    // Bucket by bucket, each as soon as its all-reduce is done: the updates of
    // the buckets averaged first overlap the all-reduce of the last ones.
    // (The update is elementwise, so the ranges give the same result as one
    // launch over the whole buffer.)
    char* p = (char*)pbuf_.get();
    char* g = (char*)gbuf_.get();
    char* v = (char*)opt_a_.get();
    for (size_t i = 0; i < buckets_.size(); i++) {
      const int64_t lo = buckets_[i].first, n = buckets_[i].second - buckets_[i].first;
      check(gt_stream_wait_event(ctx_, GT_STREAM_COMPUTE, bucket_done_[i]));
      check(gt_sgd_step(ctx_, dtype_, p + lo * es_, g + lo * es_, v + lo * es_, n, &sgd_, opt_steps_ == 0));
    }
    check(gt_comm_wait(ctx_));  // the loss average, and every stream joined
  } else if (opt_ == OPT_SGD) {
    if (world_ > 1) check(gt_comm_wait(ctx_));
    check(gt_sgd_step(ctx_, dtype_, pbuf_.get(), gbuf_.get(), opt_a_.get(), dev_params_, &sgd_, opt_steps_ == 0));
  } else {
    if (world_ > 1) check(gt_comm_wait(ctx_));
    check(gt_adam_step_dev(ctx_, dtype_, pbuf_.get(), gbuf_.get(), opt_a_.get(), opt_b_.get(), dev_params_, &adam_,
                           (int64_t*)step_dev_.get()));
  }
  opt_steps_++;
}

void Model::train_step() {
  if (opt_ == OPT_NONE) throw Error("no optimizer: call gth_set_sgd or gth_set_adam");
  const int p = cur_;
  begin_read();  // outside any capture: the wait for a staged upload is per step
  if (use_graph_ && graph_[p]) {
    check(gt_graph_launch(ctx_, graph_[p]));
    opt_steps_++;
  } else {
    // The first SGD step initialises the velocity, so capture from the second
    // (a graph per input pair, each reading its own buffers).
    bool capture = use_graph_ && opt_steps_ >= 1;
    int64_t before = gt_launch_count();
    if (capture) check(gt_capture_begin(ctx_));
    try {
      forward();
      backward(false);  // the optimizer waits for the gradient buckets itself
      optimizer_step();
    } catch (...) {
      if (capture) {
        gt_graph* g = nullptr;
        gt_free_error(gt_capture_end(ctx_, &g));
        gt_graph_free(g);
      }
      throw;
    }
    launches_ = (int)(gt_launch_count() - before);
    if (capture) {
      check(gt_capture_end(ctx_, &graph_[p]));
      opt_steps_--;  // the captured step has not run yet
      check(gt_graph_launch(ctx_, graph_[p]));
      opt_steps_++;
    }
  }
  end_read();
}

void Model::enable_graph(bool on) {
  use_graph_ = on;
  if (!on) drop_graph();
}

double Model::loss() {
  double out = 0;
  if (dtype_ == GT_FLOAT64) {
    check(gt_download(ctx_, &out, loss_.get(), 8));
  } else {
    float f = 0;
    check(gt_download(ctx_, &f, loss_.get(), 4));
    out = f;
  }
  return out;
}

void Model::predict(int32_t* preds, int64_t* correct) {
  if (!pred_.get()) {
    pred_ = DevBuf(ctx_, batch_ * sizeof(int32_t));
    count_ = DevBuf(ctx_, sizeof(int64_t));
  }
  begin_read();
  const int32_t* labels = labels_device();  // the pair this evaluation reads
  forward();
  check(gt_argmax_rows(ctx_, dtype_, ops_.back().out, batch_, classes_, (int32_t*)pred_.get()));
  if (correct) check(gt_count_equal(ctx_, (const int32_t*)pred_.get(), labels, batch_, (int64_t*)count_.get()));
  end_read();
  if (preds) check(gt_download(ctx_, preds, pred_.get(), batch_ * sizeof(int32_t)));
  if (correct) check(gt_download(ctx_, correct, count_.get(), sizeof(int64_t)));
}

void Model::forward_eval(void* logits_host) {
  begin_read();
  forward();
  end_read();
  check(gt_download(ctx_, logits_host, ops_.back().out, batch_ * classes_ * es_));
}

// ---- data parallelism -------------------------------------------------------

void Model::dp_init(int rank, int world, const unsigned char id[128], int timeout_ms, int64_t bucket_bytes) {
  drop_graph();
  // SMs the backward GEMMs leave to the all-reduce kernels running beside
  // them (GT_DP_SM_RESERVE; 0 = none).
  if (const char* r = getenv("GT_DP_SM_RESERVE")) sm_reserve_ = std::max(0, atoi(r));
  if (world > 1) check(gt_comm_init(ctx_, rank, world, id, timeout_ms));
  rank_ = rank;
  world_ = world;
  std::vector<int64_t> sizes;
  for (size_t i = 0; i < params_.size(); i++) {
    int64_t end = i + 1 < params_.size() ? params_[i + 1].dev_offset : dev_params_;
    sizes.push_back(end - params_[i].dev_offset);
  }
  std::vector<int64_t> bounds(2 * sizes.size() + 2);
  int nb = gth_bucket_plan(sizes.data(), (int)sizes.size(), std::max<int64_t>(1, bucket_bytes / (int64_t)es_),
                           bounds.data(), (int)sizes.size());
  buckets_.clear();
  for (int b = 0; b < nb; b++) buckets_.emplace_back(bounds[2 * b], bounds[2 * b + 1]);
  // The first layer's weight gradient is the backward's last GEMM, so its
  // bucket's all-reduce and update cannot overlap anything. When it is a
  // Linear whose weight starts a bucket, that bucket is split at row chunks
  // (multiples of 256 rows, or of 32 for small layers; GT_DP_LAST_CHUNKS
  // chunks, default 1 = off: it gained 2 % per step at 2 GPUs and lost 9 %
  // at 8, where each chunk is a one-wave GEMM that competes with NCCL for
  // SMs), and the
  // backward computes the chunks from the last rows down, each bucket
  // issued as soon as its rows are done: only the last chunk stays exposed.
  first_rows_.clear();
  int chunks = 1;
  if (const char* c = getenv("GT_DP_LAST_CHUNKS")) chunks = std::max(1, atoi(c));
  if (world > 1 && chunks > 1 && first_param_op_ >= 0 && ops_[first_param_op_].kind == Op::LINEAR) {
    const Op& op = ops_[first_param_op_];
    const int64_t cap = op.N / 32 + 3;  // chunks are at least 32 rows
    std::vector<int64_t> flat, rows(cap), out(2 * (nb + cap));
    for (auto& b : buckets_) flat.push_back(b.first), flat.push_back(b.second);
    int out_nb = 0;
    const int nr = gth_row_chunk_plan(flat.data(), nb, op.w_off, op.N, op.K, chunks, rows.data(), (int)rows.size(),
                                      out.data(), (int)out.size() / 2, &out_nb);
    if (nr > 0) {
      first_rows_.assign(rows.begin(), rows.begin() + nr);
      buckets_.clear();
      for (int b = 0; b < out_nb; b++) buckets_.emplace_back(out[2 * b], out[2 * b + 1]);
    }
  }
  nb = (int)buckets_.size();
  free_bucket_events();
  for (int b = 0; b < nb; b++) {
    gt_event* e = nullptr;
    check(gt_event_new(ctx_, &e));
    bucket_done_.push_back(e);
  }
}

}  // namespace gotensor

extern "C" int gth_bucket_plan(const int64_t* sizes, int n, int64_t bucket_elems, int64_t* bounds, int cap) {
  int count = 0;
  int64_t total = 0;
  for (int i = 0; i < n; i++) total += sizes[i];
  int64_t hi = total, acc = 0, pos = total;
  for (int i = n - 1; i >= 0; i--) {
    pos -= sizes[i];
    acc += sizes[i];
    if (acc >= bucket_elems || i == 0) {
      if (count >= cap) return -1;
      bounds[2 * count] = pos;
      bounds[2 * count + 1] = hi;
      count++;
      hi = pos;
      acc = 0;
    }
  }
  return count;
}

// The first layer's weight gradient is the backward's last GEMM, so the
// all-reduce of its bucket cannot overlap anything. The bucket that starts at
// that weight (w_off, N rows of K) is split at row chunks: rows per chunk a
// multiple of 256 (whole GEMM tiles) or, for small layers, of 32. Sub-buckets
// are listed highest offsets first, the order the backward computes the
// chunks; the last one keeps the rest of the original bucket (the bias and
// anything after it).
extern "C" int gth_row_chunk_plan(const int64_t* bounds, int nb, int64_t w_off, int64_t N, int64_t K, int chunks,
                                  int64_t* rows, int rows_cap, int64_t* out_bounds, int out_cap, int* out_nb) {
  if (out_nb) *out_nb = 0;
  if (!bounds || !rows || !out_bounds || !out_nb || nb < 0 || N <= 0 || K <= 0 || chunks < 2) return 0;
  int64_t per = (N + chunks - 1) / chunks;
  per = per >= 256 ? per / 256 * 256 : per / 32 * 32;
  if (per <= 0) return 0;
  int b = 0;
  while (b < nb && bounds[2 * b] != w_off) b++;
  if (b == nb) return 0;
  int nr = 0;
  for (int64_t r = 0; r < N; r += per) {
    if (nr >= rows_cap) return 0;
    rows[nr++] = r;
  }
  if (nr >= rows_cap) return 0;
  rows[nr++] = N;
  if (nr < 3) return 0;  // one chunk: nothing to split
  const int total = nb - 1 + (nr - 1);
  if (total > out_cap) return 0;
  int k = 0;
  for (int i = 0; i < b; i++, k++) out_bounds[2 * k] = bounds[2 * i], out_bounds[2 * k + 1] = bounds[2 * i + 1];
  const int64_t end = bounds[2 * b + 1];
  for (int j = nr - 2; j >= 0; j--, k++) {
    out_bounds[2 * k] = w_off + rows[j] * K;
    out_bounds[2 * k + 1] = j == nr - 2 ? end : w_off + rows[j + 1] * K;
  }
  for (int i = b + 1; i < nb; i++, k++) out_bounds[2 * k] = bounds[2 * i], out_bounds[2 * k + 1] = bounds[2 * i + 1];
  *out_nb = k;
  return nr;
}
