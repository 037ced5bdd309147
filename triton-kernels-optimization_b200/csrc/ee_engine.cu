// ee_engine.cu - the C++ launcher of the gated layer loop: a fixed description of L
// gated layers (each: routing logits + P projections, all at fixed device addresses)
// enqueued eagerly or recorded once into a CUDA graph and replayed.  This replaces the
// reference's Python per-layer loop with its host synchronisation per layer
// (EE/python/dispatch.py:192, :199-203, quality_eval.py:133-141) and its single-kernel
// cubin launcher (EE/csrc/engine.cpp:64-200).
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/ee_b200.h"
#include "ee_internal.h"

struct ee_engine {
  int64_t rows = 0;
  double tau_low = 0.0, tau_high = 0.0;
  std::vector<ee_gated_layer> layers;
  std::vector<std::vector<ee_projection>> projs;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int device = -1;
  std::mutex mu;  // one launch or capture at a time per engine
};

namespace {

int engine_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  ee::set_last_error(buf);  // what ee_last_error() returns on this thread
  return code;
}

int64_t max_k(const ee_engine& e) {
  int64_t k = 16;
  for (const auto& ps : e.projs)
    for (const auto& p : ps) k = p.K > k ? p.K : k;
  return k;
}

int run_layers(ee_engine& e, void* stream) {
  for (size_t l = 0; l < e.layers.size(); ++l) {
    const ee_gated_layer& L = e.layers[l];
    // the header was zeroed at creation and every kernel leaves it zero: no memset node
    int st = ee::gate_rows_impl(L.logits, e.rows, L.n_logits, L.ld_logits, e.tau_low, e.tau_high, nullptr, nullptr,
                                nullptr, e.workspace, e.workspace_bytes, stream, false);
    if (st != EE_OK) return st;
    for (const ee_projection& p : e.projs[l]) {
      st = ee_gated_gemm(p.A, p.lda, e.rows, p.K, p.w_i8_nk, p.w_e4m3_nk, p.w_f16_nk, p.w_scale, p.N, p.Y, p.ldy,
                         e.workspace, e.workspace_bytes, stream);
      if (st != EE_OK) return st;
    }
  }
  return EE_OK;
}

}  // namespace

extern "C" {

size_t ee_engine_workspace_bytes(int64_t rows, int32_t n_layers, const ee_gated_layer* layers) {
  if (rows < 0 || n_layers < 0 || (n_layers > 0 && layers == nullptr)) return 0;
  int64_t k = 16;
  for (int32_t l = 0; l < n_layers; ++l) {
    if (layers[l].n_proj < 0 || (layers[l].n_proj > 0 && layers[l].proj == nullptr)) return 0;
    for (int32_t p = 0; p < layers[l].n_proj; ++p) k = layers[l].proj[p].K > k ? layers[l].proj[p].K : k;
  }
  return ee_gated_workspace_bytes(rows, k);
}

int ee_engine_create(int64_t rows, double tau_low, double tau_high, int32_t n_layers, const ee_gated_layer* layers,
                     void* workspace, size_t workspace_bytes, ee_engine** out) {
  if (out == nullptr) return engine_fail(EE_ERR_INVALID, "ee_engine_create: out is NULL");
  *out = nullptr;
  if (rows < 0 || n_layers <= 0 || layers == nullptr)
    return engine_fail(EE_ERR_INVALID, "ee_engine_create: need rows >= 0 and at least one layer");
  ee_engine* e = new (std::nothrow) ee_engine();
  if (e == nullptr) return engine_fail(EE_ERR_INVALID, "ee_engine_create: out of host memory");
  e->rows = rows;
  e->tau_low = tau_low;
  e->tau_high = tau_high;
  for (int32_t l = 0; l < n_layers; ++l) {
    const ee_gated_layer& L = layers[l];
    if (L.logits == nullptr || L.n_logits <= 0 || L.ld_logits < L.n_logits || L.n_proj < 0 ||
        (L.n_proj > 0 && L.proj == nullptr)) {
      delete e;
      return engine_fail(EE_ERR_INVALID, "ee_engine_create: layer %d is malformed", l);
    }
    e->layers.push_back(L);
    e->projs.emplace_back(L.proj, L.proj + L.n_proj);
    e->layers.back().proj = nullptr;  // the copy in projs is the one used
  }
  const size_t need = ee_gated_workspace_bytes(rows, max_k(*e));
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u)) {
    delete e;
    return engine_fail(EE_ERR_INVALID, "ee_engine_create: workspace must be 256-byte aligned and >= %zu bytes", need);
  }
  e->workspace = workspace;
  e->workspace_bytes = workspace_bytes;
  if (cudaGetDevice(&e->device) != cudaSuccess || ee::prepare_device() != 0 ||
      cudaMemset(workspace, 0, ee::gated_ws_head_bytes()) != cudaSuccess) {  // ticket, counts, tile
                                                                             // counter, look-back epoch
    delete e;
    return engine_fail(EE_ERR_CUDA, "ee_engine_create: CUDA device not usable");
  }
  *out = e;
  return EE_OK;
}

int ee_engine_run(ee_engine* e, void* stream) {
  if (e == nullptr) return engine_fail(EE_ERR_INVALID, "ee_engine_run: engine is NULL");
  std::lock_guard<std::mutex> lock(e->mu);
  return run_layers(*e, stream);
}

int ee_engine_capture(ee_engine* e, void* stream) {
  if (e == nullptr) return engine_fail(EE_ERR_INVALID, "ee_engine_capture: engine is NULL");
  if (stream == nullptr) return engine_fail(EE_ERR_INVALID, "ee_engine_capture: needs a non-default stream");
  std::lock_guard<std::mutex> lock(e->mu);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
  if (err != cudaSuccess) return engine_fail(EE_ERR_CUDA, "cudaStreamBeginCapture: %s", cudaGetErrorString(err));
  const int st = run_layers(*e, stream);
  cudaGraph_t graph = nullptr;
  err = cudaStreamEndCapture(s, &graph);
  if (st != EE_OK) {
    if (graph) cudaGraphDestroy(graph);
    return st;
  }
  if (err != cudaSuccess) return engine_fail(EE_ERR_CUDA, "cudaStreamEndCapture: %s", cudaGetErrorString(err));
  cudaGraphExec_t exec = nullptr;
  err = cudaGraphInstantiate(&exec, graph, 0);
  if (err != cudaSuccess) {
    cudaGraphDestroy(graph);
    return engine_fail(EE_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(err));
  }
  if (e->exec) cudaGraphExecDestroy(e->exec);
  if (e->graph) cudaGraphDestroy(e->graph);
  e->graph = graph;
  e->exec = exec;
  return EE_OK;
}

int ee_engine_launch(ee_engine* e, void* stream) {
  if (e == nullptr) return engine_fail(EE_ERR_INVALID, "ee_engine_launch: engine is NULL");
  if (e->exec == nullptr) {
    int st = ee_engine_capture(e, stream);
    if (st != EE_OK) return st;
  }
  std::lock_guard<std::mutex> lock(e->mu);
  cudaError_t err = cudaGraphLaunch(e->exec, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return engine_fail(EE_ERR_CUDA, "cudaGraphLaunch: %s", cudaGetErrorString(err));
  return EE_OK;
}

int ee_engine_destroy(ee_engine* e) {
  if (e == nullptr) return EE_OK;
  if (e->exec) cudaGraphExecDestroy(e->exec);
  if (e->graph) cudaGraphDestroy(e->graph);
  delete e;
  return EE_OK;
}

}  // extern "C"
