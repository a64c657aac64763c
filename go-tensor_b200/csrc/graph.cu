// CUDA graph capture of the context's stream, and stream timing points.
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

}  // extern "C"
