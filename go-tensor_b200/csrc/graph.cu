// CUDA graph capture of the context's stream, stream timing points, and the
// events and copy stream that let a host overlap the next batch's upload with
// the step in flight.
#include "gt_common.cuh"

struct gt_graph {
  cudaGraphExec_t exec = nullptr;
  cudaGraph_t graph = nullptr;
};

extern "C" {

char* gt_capture_begin(gt_ctx* ctx) {
  GT_ENTER(ctx);
  GT_CUDA(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  return nullptr;
}

char* gt_capture_end(gt_ctx* ctx, gt_graph** out) {
  GT_ENTER(ctx);
  if (!out) return gt::errorf("gt_capture_end: null output");
  *out = nullptr;
  cudaGraph_t g = nullptr;
  GT_CUDA(cudaStreamEndCapture(ctx->stream, &g));
  gt_graph* gr = new gt_graph();
  gr->graph = g;
  cudaError_t e = cudaGraphInstantiate(&gr->exec, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    delete gr;
    return gt::cuda_error(e, "cudaGraphInstantiate", __FILE__, __LINE__);
  }
  *out = gr;
  return nullptr;
}

char* gt_graph_launch(gt_ctx* ctx, gt_graph* graph) {
  GT_ENTER(ctx);
  if (!graph) return gt::errorf("gt_graph_launch: null graph");
  GT_CUDA(cudaGraphLaunch(graph->exec, ctx->stream));
  return nullptr;
}

void gt_graph_free(gt_graph* graph) {
  if (!graph) return;
  if (graph->exec) cudaGraphExecDestroy(graph->exec);
  if (graph->graph) cudaGraphDestroy(graph->graph);
  delete graph;
}

char* gt_mark(gt_ctx* ctx, int slot) {
  GT_ENTER(ctx);
  if (slot < 0 || slot >= 8) return gt::errorf("gt_mark: slot %d out of range", slot);
  GT_CUDA(cudaEventRecord(ctx->marks[slot], ctx->stream));
  return nullptr;
}

char* gt_elapsed_ms(gt_ctx* ctx, int from, int to, float* ms) {
  GT_ENTER(ctx);
  if (from < 0 || from >= 8 || to < 0 || to >= 8 || !ms) return gt::errorf("gt_elapsed_ms: bad arguments");
  GT_CUDA(cudaEventSynchronize(ctx->marks[to]));
  GT_CUDA(cudaEventElapsedTime(ms, ctx->marks[from], ctx->marks[to]));
  return nullptr;
}

// ---- events and the copy stream ---------------------------------------------

struct gt_event {
  cudaEvent_t ev = nullptr;
};

static cudaStream_t stream_of(gt_ctx* ctx, int which) {
  switch (which) {
    case GT_STREAM_COMPUTE: return ctx->stream;
    case GT_STREAM_COPY: return ctx->copy_stream;
    case GT_STREAM_COMM: return ctx->comm_stream;
    default: return nullptr;
  }
}

char* gt_event_new(gt_ctx* ctx, gt_event** out) {
  GT_ENTER(ctx);
  if (!out) return gt::errorf("gt_event_new: null output");
  auto* e = new gt_event();
  cudaError_t r = cudaEventCreateWithFlags(&e->ev, cudaEventDisableTiming);
  if (r != cudaSuccess) {
    delete e;
    return gt::cuda_error(r, "cudaEventCreateWithFlags", __FILE__, __LINE__);
  }
  *out = e;
  return nullptr;
}

void gt_event_free(gt_event* e) {
  if (!e) return;
  if (e->ev) cudaEventDestroy(e->ev);
  delete e;
}

char* gt_event_record(gt_ctx* ctx, gt_event* e, int stream) {
  GT_ENTER(ctx);
  cudaStream_t st = stream_of(ctx, stream);
  if (!e || !st) return gt::errorf("gt_event_record: bad event or stream %d", stream);
  GT_CUDA(cudaEventRecord(e->ev, st));
  return nullptr;
}

char* gt_stream_wait_event(gt_ctx* ctx, int stream, gt_event* e) {
  GT_ENTER(ctx);
  cudaStream_t st = stream_of(ctx, stream);
  if (!e || !st) return gt::errorf("gt_stream_wait_event: bad event or stream %d", stream);
  GT_CUDA(cudaStreamWaitEvent(st, e->ev, 0));
  return nullptr;
}

char* gt_upload_on(gt_ctx* ctx, int stream, void* dst, const void* src, size_t bytes) {
  GT_ENTER(ctx);
  cudaStream_t st = stream_of(ctx, stream);
  if (!st) return gt::errorf("gt_upload_on: bad stream %d", stream);
  if (bytes == 0) return nullptr;
  if (!dst || !src) return gt::errorf("gt_upload_on: null pointer");
  GT_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st));
  return nullptr;
}

char* gt_host_alloc(size_t bytes, void** out) {
  if (!out) return gt::errorf("gt_host_alloc: null output");
  *out = nullptr;
  GT_CUDA(cudaHostAlloc(out, bytes ? bytes : 1, cudaHostAllocPortable));
  return nullptr;
}

void gt_host_free(void* p) {
  if (p) cudaFreeHost(p);
}

}  // extern "C"
