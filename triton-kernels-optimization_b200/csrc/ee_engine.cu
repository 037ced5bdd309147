// ee_engine.cu - the C++ launcher of the gated layer loop: a fixed description of L
// gated layers (each: routing logits + P projections, all at fixed device addresses)
// enqueued eagerly or recorded once into a CUDA graph and replayed.  This replaces the
// reference's Python per-layer loop with its host synchronisation per layer
// (EE/python/dispatch.py:192, :199-203, quality_eval.py:133-141) and its single-kernel
// cubin launcher (EE/csrc/engine.cpp:64-200).
#include <cuda_fp16.h>
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

// ===================================================================================
// Decoder-stack engine: the whole Llama decoder stack for one batch shape, every step
// an entry point of this library on one stream (see ee_decoder_* in ee_b200.h).
// ===================================================================================
struct ee_decoder {
  ee_decoder_config cfg{};
  std::vector<ee_decoder_layer> layers;
  const void* final_norm = nullptr;
  const void* cos = nullptr;
  const void* sin = nullptr;
  int32_t* layer_counts = nullptr;
  // workspace regions (see dec_layout)
  __half* hbuf = nullptr;   // h_l: the block input (residual of the attention)
  __half* sbuf = nullptr;   // s_l = h_l + attention output (residual of the MLP)
  __half* x = nullptr;      // normalised rows
  __half* qkv = nullptr;    // [M, (heads + 2 kv_heads) head_dim]
  __half* att = nullptr;    // attention output [M, heads head_dim]
  float* rows = nullptr;    // row entropies [batch, heads, seq]
  float* ht[2] = {nullptr, nullptr};  // per-token entropies, this layer / the previous one
  float* hb = nullptr;      // per-batch mean entropies [batch]
  float* hall[2] = {nullptr, nullptr};  // batch-max router input [M], this layer / the previous one
  float* hinf = nullptr;    // +inf [M]: routes every row to FP16 (first layer's projections)
  __half* o = nullptr;      // o projection [M, hidden]
  __half* hmid = nullptr;   // SwiGLU output [M, intermediate]
  __half* mlp = nullptr;    // down projection [M, hidden]
  void* att_ws = nullptr;
  size_t att_ws_bytes = 0;
  void* gws = nullptr;      // gated workspace (routing, packed rows, K-split partials)
  size_t gws_bytes = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int device = -1;
  std::mutex mu;
};

namespace {

struct DecLayout {
  size_t hbuf, sbuf, x, qkv, att, rows, ht0, ht1, hb, hall0, hall1, hinf, o, hmid, mlp, att_ws, gws, total;
  size_t att_ws_bytes, gws_bytes;
};

inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

bool dec_config_ok(const ee_decoder_config& c) {
  return c.batch > 0 && c.seq > 0 && c.hidden > 0 && c.heads > 0 && c.kv_heads > 0 && c.heads % c.kv_heads == 0 &&
         (c.head_dim == 64 || c.head_dim == 128) && c.intermediate > 0 && c.intermediate % 128 == 0 &&
         c.hidden % 16 == 0 && (c.routing == EE_ROUTE_TOKEN || c.routing == EE_ROUTE_BATCH) &&
         (c.route_all == 0 || c.route_all == 1) && (c.exact_entropy == 0 || c.exact_entropy == 1) &&
         c.batch * c.seq < (int64_t(1) << 31);
}

DecLayout dec_layout(const ee_decoder_config& c) {
  DecLayout L{};
  const size_t M = size_t(c.batch) * size_t(c.seq), d = size_t(c.hidden), I = size_t(c.intermediate);
  const size_t nq = size_t(c.heads) * c.head_dim, nqkv = size_t(c.heads + 2 * c.kv_heads) * c.head_dim;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += al256(bytes);
    return at;
  };
  L.hbuf = take(2 * M * d);
  L.sbuf = take(2 * M * d);
  L.x = take(2 * M * d);
  L.qkv = take(2 * M * nqkv);
  L.att = take(2 * M * nq);
  L.rows = take(4 * size_t(c.batch) * c.heads * c.seq);
  L.ht0 = take(4 * M);
  L.ht1 = take(4 * M);
  L.hb = take(4 * size_t(c.batch));
  L.hall0 = take(4 * M);
  L.hall1 = take(4 * M);
  L.hinf = take(4 * M);
  L.o = take(2 * M * d);
  L.hmid = take(2 * M * I);
  L.mlp = take(2 * M * d);
  L.att_ws_bytes = c.exact_entropy
                       ? ee_attention_exact_workspace_bytes(c.batch, c.heads, c.kv_heads, c.seq, c.head_dim)
                       : ee_attention_rope_workspace_bytes(c.batch, c.heads, c.kv_heads, c.seq, c.head_dim);
  L.att_ws = take(L.att_ws_bytes);
  int64_t kmax = c.hidden > int64_t(nq) ? c.hidden : int64_t(nq);
  kmax = kmax > c.intermediate ? kmax : c.intermediate;
  L.gws_bytes = ee_gated_workspace_split_bytes(int64_t(M), kmax);
  L.gws = take(L.gws_bytes);
  L.total = off;
  return L;
}

bool pack_ok(const ee_weight_pack& p) { return p.w_i8 && p.w_e4m3 && p.w_f16 && p.scale; }

// One routed projection: route M rows by H, place A's rows in the buckets, gated GEMM.
int routed_linear(ee_decoder& D, const float* H, const void* A, int64_t K, const ee_weight_pack& w, int64_t N, void* Y,
                  int32_t* counts, cudaStream_t s) {
  const int64_t M = D.cfg.batch * D.cfg.seq;
  int st = ee_gate_entropies(H, M, D.cfg.tau_low, D.cfg.tau_high, nullptr, counts, D.gws, D.gws_bytes, s);
  if (st != EE_OK) return st;
  if ((st = ee_gated_pack(A, K, M, K, D.gws, D.gws_bytes, s)) != EE_OK) return st;
  return ee_gated_gemm_packed(M, K, w.w_i8, w.w_e4m3, w.w_f16, w.scale, N, Y, N, D.gws, D.gws_bytes, s);
}

int dec_check(int st, const char* what) {
  if (st == EE_OK) return st;
  // keep the failing step's own message, prefixed with where in the stack it happened
  const std::string inner = ee_last_error();
  ee::set_last_error((std::string("decoder ") + what + ": " + inner).c_str());
  return st;
}

int run_decoder(ee_decoder& D, const void* hin, void* hout, void* rout, cudaStream_t s) {
  const ee_decoder_config& c = D.cfg;
  const int64_t M = c.batch * c.seq, d = c.hidden, I = c.intermediate;
  const int64_t nq = c.heads * c.head_dim, nkv = c.kv_heads * c.head_dim, nqkv = nq + 2 * nkv;
  const bool batch = c.routing == EE_ROUTE_BATCH;
  int st;
  if (c.route_all && (st = dec_check(ee::launch_fill_value(D.hinf, M, __builtin_huge_valf(), s) == 0 ? EE_OK : EE_ERR_CUDA,
                                     "fill")) != EE_OK)
    return st;
  for (size_t l = 0; l < D.layers.size(); ++l) {
    const ee_decoder_layer& L = D.layers[l];
    const int cur = static_cast<int>(l & 1), prev = cur ^ 1;
    // x = RMSNorm(h_l); for l > 0, h_l = s_{l-1} + mlp_{l-1} is formed in the same pass
    if (l == 0)
      st = ee_add_rmsnorm(hin, d, nullptr, 0, nullptr, 0, L.input_norm, c.rms_eps, D.x, d, M, d, s);
    else
      st = ee_add_rmsnorm(D.mlp, d, D.sbuf, d, D.hbuf, d, L.input_norm, c.rms_eps, D.x, d, M, d, s);
    if ((st = dec_check(st, "input norm")) != EE_OK) return st;
    const void* h_l = l == 0 ? hin : D.hbuf;
    // q / k / v
    if (c.route_all) {
      const float* hr = l == 0 ? D.hinf : (batch ? D.hall[prev] : D.ht[prev]);
      st = routed_linear(D, hr, D.x, d, L.qkv, nqkv, D.qkv, nullptr, s);
    } else {
      st = ee_gemm_fp16(D.x, L.qkv_f16, D.qkv, M, nqkv, d, nqkv, s);
    }
    if ((st = dec_check(st, "qkv projection")) != EE_OK) return st;
    // rotary embedding + causal flash attention with the entropy of every query row
    st = (c.exact_entropy ? ee_flash_attention_rope_entropy_exact : ee_flash_attention_rope_entropy)(
        D.qkv, nqkv, D.qkv + nq, nqkv, D.qkv + nq + nkv, nqkv, D.cos, D.sin, c.head_dim, c.batch, c.heads, c.kv_heads,
        c.seq, c.head_dim, 1, c.attn_scale, D.att, D.rows, D.att_ws, D.att_ws_bytes, s);
    if ((st = dec_check(st, "attention")) != EE_OK) return st;
    st = ee_head_mean_entropy(D.rows, c.batch, c.heads, c.seq, D.ht[cur], batch ? D.hb : nullptr, s);
    if ((st = dec_check(st, "head mean")) != EE_OK) return st;
    if (batch && (st = dec_check(ee::launch_batch_max_fill(D.hb, c.batch, D.hall[cur], M, s) == 0 ? EE_OK : EE_ERR_CUDA,
                                 "batch max")) != EE_OK)
      return st;
    const float* hcur = batch ? D.hall[cur] : D.ht[cur];
    // o projection
    if (c.route_all)
      st = routed_linear(D, hcur, D.att, nq, L.o, d, D.o, nullptr, s);
    else
      st = ee_gemm_fp16(D.att, L.o_f16, D.o, M, d, nq, d, s);
    if ((st = dec_check(st, "o projection")) != EE_OK) return st;
    // s_l = h_l + o, x = RMSNorm(s_l)
    st = ee_add_rmsnorm(D.o, d, h_l, d, D.sbuf, d, L.post_norm, c.rms_eps, D.x, d, M, d, s);
    if ((st = dec_check(st, "post-attention norm")) != EE_OK) return st;
    // routed SwiGLU MLP: gate / up in one GEMM, then down, on the same routing
    int32_t* counts = D.layer_counts ? D.layer_counts + 3 * l : nullptr;
    st = ee_gate_entropies(hcur, M, c.tau_low, c.tau_high, nullptr, counts, D.gws, D.gws_bytes, s);
    if (st == EE_OK) st = ee_gated_pack(D.x, d, M, d, D.gws, D.gws_bytes, s);
    if (st == EE_OK)
      st = ee_gated_swiglu_packed(M, d, L.gate_up.w_i8, L.gate_up.w_e4m3, L.gate_up.w_f16, L.gate_up.scale, I, D.hmid,
                                  I, D.gws, D.gws_bytes, s);
    if (st == EE_OK) st = ee_gated_pack(D.hmid, I, M, I, D.gws, D.gws_bytes, s);
    if (st == EE_OK)
      st = ee_gated_gemm_packed(M, I, L.down.w_i8, L.down.w_e4m3, L.down.w_f16, L.down.scale, d, D.mlp, d, D.gws,
                                D.gws_bytes, s);
    if ((st = dec_check(st, "MLP")) != EE_OK) return st;
  }
  // h_L = s + mlp (returned as residual_out), hidden_out = RMSNorm_final(h_L)
  st = ee_add_rmsnorm(D.mlp, d, D.sbuf, d, rout, d, D.final_norm, c.rms_eps, hout, d, M, d, s);
  return dec_check(st, "final norm");
}

}  // namespace

extern "C" {

size_t ee_decoder_workspace_bytes(const ee_decoder_config* cfg) {
  if (cfg == nullptr || !dec_config_ok(*cfg)) return 0;
  return dec_layout(*cfg).total;
}

int ee_decoder_create(const ee_decoder_config* cfg, int32_t n_layers, const ee_decoder_layer* layers,
                      const void* final_norm, const void* cos, const void* sin, int32_t* layer_counts, void* workspace,
                      size_t workspace_bytes, ee_decoder** out) {
  if (out == nullptr) return engine_fail(EE_ERR_INVALID, "ee_decoder_create: out is NULL");
  *out = nullptr;
  if (cfg == nullptr || !dec_config_ok(*cfg))
    return engine_fail(EE_ERR_INVALID,
                       "ee_decoder_create: bad config (head_dim 64 / 128, heads %% kv_heads == 0, intermediate %% 128 "
                       "== 0, hidden %% 16 == 0, routing 0 / 1, route_all 0 / 1, exact_entropy 0 / 1)");
  if (n_layers <= 0 || layers == nullptr || final_norm == nullptr || cos == nullptr || sin == nullptr)
    return engine_fail(EE_ERR_INVALID, "ee_decoder_create: layers, final_norm, cos and sin are required");
  for (int32_t l = 0; l < n_layers; ++l) {
    const ee_decoder_layer& L = layers[l];
    const bool attn_ok = cfg->route_all ? (pack_ok(L.qkv) && pack_ok(L.o)) : (L.qkv_f16 != nullptr && L.o_f16 != nullptr);
    if (!L.input_norm || !L.post_norm || !attn_ok || !pack_ok(L.gate_up) || !pack_ok(L.down))
      return engine_fail(EE_ERR_INVALID, "ee_decoder_create: layer %d is missing a weight", l);
  }
  const DecLayout lay = dec_layout(*cfg);
  if (workspace == nullptr || workspace_bytes < lay.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return engine_fail(EE_ERR_INVALID, "ee_decoder_create: workspace must be 256-byte aligned and >= %zu bytes",
                       lay.total);
  ee_decoder* D = new (std::nothrow) ee_decoder();
  if (D == nullptr) return engine_fail(EE_ERR_INVALID, "ee_decoder_create: out of host memory");
  D->cfg = *cfg;
  D->layers.assign(layers, layers + n_layers);
  D->final_norm = final_norm;
  D->cos = cos;
  D->sin = sin;
  D->layer_counts = layer_counts;
  uint8_t* base = static_cast<uint8_t*>(workspace);
  D->hbuf = reinterpret_cast<__half*>(base + lay.hbuf);
  D->sbuf = reinterpret_cast<__half*>(base + lay.sbuf);
  D->x = reinterpret_cast<__half*>(base + lay.x);
  D->qkv = reinterpret_cast<__half*>(base + lay.qkv);
  D->att = reinterpret_cast<__half*>(base + lay.att);
  D->rows = reinterpret_cast<float*>(base + lay.rows);
  D->ht[0] = reinterpret_cast<float*>(base + lay.ht0);
  D->ht[1] = reinterpret_cast<float*>(base + lay.ht1);
  D->hb = reinterpret_cast<float*>(base + lay.hb);
  D->hall[0] = reinterpret_cast<float*>(base + lay.hall0);
  D->hall[1] = reinterpret_cast<float*>(base + lay.hall1);
  D->hinf = reinterpret_cast<float*>(base + lay.hinf);
  D->o = reinterpret_cast<__half*>(base + lay.o);
  D->hmid = reinterpret_cast<__half*>(base + lay.hmid);
  D->mlp = reinterpret_cast<__half*>(base + lay.mlp);
  D->att_ws = base + lay.att_ws;
  D->att_ws_bytes = lay.att_ws_bytes;
  D->gws = base + lay.gws;
  D->gws_bytes = lay.gws_bytes;
  // the gated workspace's header starts at zero (ee_gate_entropies re-zeroes it per call)
  if (cudaGetDevice(&D->device) != cudaSuccess || ee::prepare_device() != 0 ||
      cudaMemset(D->gws, 0, ee::gated_ws_head_bytes()) != cudaSuccess) {
    delete D;
    return engine_fail(EE_ERR_CUDA, "ee_decoder_create: CUDA device not usable");
  }
  *out = D;
  return EE_OK;
}

int ee_decoder_run(ee_decoder* dec, const void* hidden_in, void* hidden_out, void* residual_out, void* stream) {
  if (dec == nullptr || hidden_in == nullptr || hidden_out == nullptr)
    return engine_fail(EE_ERR_INVALID, "ee_decoder_run: decoder, hidden_in and hidden_out are required");
  std::lock_guard<std::mutex> lock(dec->mu);
  return run_decoder(*dec, hidden_in, hidden_out, residual_out, static_cast<cudaStream_t>(stream));
}

int ee_decoder_capture(ee_decoder* dec, const void* hidden_in, void* hidden_out, void* residual_out, void* stream) {
  if (dec == nullptr || hidden_in == nullptr || hidden_out == nullptr)
    return engine_fail(EE_ERR_INVALID, "ee_decoder_capture: decoder, hidden_in and hidden_out are required");
  if (stream == nullptr) return engine_fail(EE_ERR_INVALID, "ee_decoder_capture: needs a non-default stream");
  std::lock_guard<std::mutex> lock(dec->mu);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
  if (err != cudaSuccess) return engine_fail(EE_ERR_CUDA, "cudaStreamBeginCapture: %s", cudaGetErrorString(err));
  const int st = run_decoder(*dec, hidden_in, hidden_out, residual_out, s);
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
  if (dec->exec) cudaGraphExecDestroy(dec->exec);
  if (dec->graph) cudaGraphDestroy(dec->graph);
  dec->graph = graph;
  dec->exec = exec;
  return EE_OK;
}

int ee_decoder_launch(ee_decoder* dec, void* stream) {
  if (dec == nullptr) return engine_fail(EE_ERR_INVALID, "ee_decoder_launch: decoder is NULL");
  std::lock_guard<std::mutex> lock(dec->mu);
  if (dec->exec == nullptr) return engine_fail(EE_ERR_INVALID, "ee_decoder_launch: nothing captured yet");
  cudaError_t err = cudaGraphLaunch(dec->exec, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return engine_fail(EE_ERR_CUDA, "cudaGraphLaunch: %s", cudaGetErrorString(err));
  return EE_OK;
}

int ee_decoder_destroy(ee_decoder* dec) {
  if (dec == nullptr) return EE_OK;
  if (dec->exec) cudaGraphExecDestroy(dec->exec);
  if (dec->graph) cudaGraphDestroy(dec->graph);
  delete dec;
  return EE_OK;
}

}  // extern "C"
