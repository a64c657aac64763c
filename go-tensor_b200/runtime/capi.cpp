// C interface of the training-step runtime (include/gt_host.h): every entry
// point converts C++ exceptions into the char* error convention of gt_cuda.h.
#include <cstring>

#include "model.hpp"

using gotensor::Error;
using gotensor::Model;

struct gth_model {
  Model* m;
};

namespace {

char* dup(const std::string& s) {
  char* out = (char*)malloc(s.size() + 1);
  if (out) memcpy(out, s.c_str(), s.size() + 1);
  return out;
}

template <typename F>
char* guard(F&& f) {
  try {
    f();
    return nullptr;
  } catch (const std::exception& e) {
    return dup(e.what());
  } catch (...) {
    return dup("gth: unknown error");
  }
}

}  // namespace

extern "C" {

GT_API char* gth_model_new(gt_ctx* ctx, int dtype, const gth_layer* layers, int nlayers, const int64_t* input_shape,
                           int ndim, gth_model** out) {
  return guard([&] {
    if (!ctx || !out || !layers || nlayers <= 0 || !input_shape || ndim <= 0) throw Error("gth_model_new: bad arguments");
    *out = nullptr;
    std::vector<gth_layer> ls(layers, layers + nlayers);
    std::vector<int64_t> shape(input_shape, input_shape + ndim);
    *out = new gth_model{new Model(ctx, dtype, ls, shape)};
  });
}

GT_API void gth_model_free(gth_model* m) {
  if (!m) return;
  delete m->m;
  delete m;
}

GT_API int gth_num_tensors(const gth_model* m) { return (int)m->m->params().size(); }
GT_API int64_t gth_num_params(const gth_model* m) { return m->m->num_params(); }

GT_API char* gth_param_info(const gth_model* m, int i, char* name, int name_cap, int64_t* shape, int* ndim,
                            int64_t* offset) {
  return guard([&] {
    const auto& ps = m->m->params();
    if (i < 0 || i >= (int)ps.size()) throw Error("gth_param_info: index out of range");
    const auto& p = ps[i];
    if (name && name_cap > 0) {
      strncpy(name, p.name.c_str(), name_cap - 1);
      name[name_cap - 1] = 0;
    }
    if (ndim) *ndim = (int)p.shape.size();
    if (shape)
      for (size_t d = 0; d < p.shape.size() && d < 4; d++) shape[d] = p.shape[d];
    if (offset) *offset = p.dense_offset;
  });
}

GT_API char* gth_set_params(gth_model* m, const void* host) { return guard([&] { m->m->set_params(host); }); }
GT_API char* gth_get_params(gth_model* m, void* host) { return guard([&] { m->m->get_params(host); }); }
GT_API char* gth_get_grads(gth_model* m, void* host) { return guard([&] { m->m->get_grads(host); }); }
GT_API void* gth_params_device(gth_model* m) { return m->m->params_device(); }
GT_API void* gth_grads_device(gth_model* m) { return m->m->grads_device(); }

GT_API char* gth_set_sgd(gth_model* m, const gt_sgd_cfg* cfg) {
  return guard([&] {
    if (!cfg) throw Error("gth_set_sgd: null config");
    m->m->set_sgd(*cfg);
  });
}

GT_API char* gth_set_adam(gth_model* m, const gt_adam_cfg* cfg) {
  return guard([&] {
    if (!cfg) throw Error("gth_set_adam: null config");
    m->m->set_adam(*cfg);
  });
}

GT_API void* gth_input_device(gth_model* m) { return m->m->input_device(); }
GT_API int32_t* gth_labels_device(gth_model* m) { return m->m->labels_device(); }
GT_API void* gth_loss_device(gth_model* m) { return m->m->loss_device(); }
GT_API char* gth_stage_batch(gth_model* m, const void* x, const int32_t* labels) {
  return guard([&] { m->m->stage_batch(x, labels); });
}

GT_API char* gth_forward_backward(gth_model* m) { return guard([&] { m->m->forward_backward(); }); }
GT_API char* gth_optimizer_step(gth_model* m) { return guard([&] { m->m->optimizer_step(); }); }
GT_API char* gth_train_step(gth_model* m) { return guard([&] { m->m->train_step(); }); }
GT_API char* gth_enable_graph(gth_model* m, int on) { return guard([&] { m->m->enable_graph(on != 0); }); }
GT_API char* gth_loss(gth_model* m, double* out) {
  return guard([&] {
    if (!out) throw Error("gth_loss: null output");
    *out = m->m->loss();
  });
}
GT_API char* gth_forward(gth_model* m, void* logits_host) { return guard([&] { m->m->forward_eval(logits_host); }); }
GT_API int gth_step_launches(const gth_model* m) { return m->m->step_launches(); }
GT_API char* gth_predict(gth_model* m, int32_t* predictions_host) {
  return guard([&] {
    if (!predictions_host) throw Error("gth_predict: null output");
    m->m->predict(predictions_host, nullptr);
  });
}
GT_API char* gth_save_safetensors(gth_model* m, const char* path, const char* dtype, const char* const* meta_keys,
                                  const char* const* meta_values, int n_meta) {
  return guard([&] {
    if (!path || !dtype || n_meta < 0 || (n_meta > 0 && (!meta_keys || !meta_values)))
      throw Error("gth_save_safetensors: bad arguments");
    std::vector<std::pair<std::string, std::string>> meta;
    for (int i = 0; i < n_meta; i++) meta.emplace_back(meta_keys[i], meta_values[i]);
    m->m->save_safetensors(path, dtype, meta);
  });
}
GT_API char* gth_load_safetensors(gth_model* m, const char* path, int strict) {
  return guard([&] {
    if (!path) throw Error("gth_load_safetensors: null path");
    m->m->load_safetensors(path, strict != 0);
  });
}
GT_API char* gth_save_gotn(gth_model* m, const char* path) {
  return guard([&] {
    if (!path) throw Error("gth_save_gotn: null path");
    m->m->save_gotn(path);
  });
}
GT_API char* gth_load_gotn(gth_model* m, const char* path) {
  return guard([&] {
    if (!path) throw Error("gth_load_gotn: null path");
    m->m->load_gotn(path);
  });
}
GT_API char* gth_count_correct(gth_model* m, int64_t* correct) {
  return guard([&] {
    if (!correct) throw Error("gth_count_correct: null output");
    m->m->predict(nullptr, correct);
  });
}

GT_API char* gth_dp_init(gth_model* m, int rank, int world, const unsigned char id[128], int timeout_ms,
                         int64_t bucket_bytes) {
  return guard([&] { m->m->dp_init(rank, world, id, timeout_ms, bucket_bytes); });
}

}  // extern "C"
