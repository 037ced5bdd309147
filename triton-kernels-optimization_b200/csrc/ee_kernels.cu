// ee_kernels.cu - the single device translation unit: every kernel of the engine and
// the C++ launchers the C-ABI layer (ee_capi.cu) calls.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <utility>

#include "ee_attention.cuh"
#include "ee_block.cuh"
#include "ee_gemm.cuh"
#include "ee_gemm_skinny.cuh"
#include "ee_internal.h"
#include "ee_kvcache.cuh"
#include "ee_rows.cuh"

namespace ee {

namespace {
inline int status_of(cudaError_t e) { return e == cudaSuccess ? 0 : -4; }

// Launch with programmatic stream serialization: the kernel may be scheduled while the
// previous kernel in the stream finishes (it waits in griddep_wait before reading
// anything), which hides launch latency between the kernels of a step.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return status_of(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// launch_pdl for a kernel whose CTAs form clusters of cluster_x along x (runtime size)
template <typename... KArgs, typename... Args>
int launch_cluster_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, unsigned cluster_x, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[3];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  // let a cluster's CTAs share SMs (two per SM where shared memory allows) instead of
  // spreading them one per SM
  attr[2].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
  attr[2].val.clusterSchedulingPolicyPreference = cudaClusterSchedulingPolicyLoadBalancing;
  cfg.attrs = attr;
  cfg.numAttrs = 3;
  return status_of(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

inline unsigned grid_of(int64_t rows, int per_block) {
  return static_cast<unsigned>((rows + per_block - 1) / per_block);
}

template <int TPR, int NV, int MINB = 1>
int run_softmax_vec(const SoftmaxArgs& a, cudaStream_t s) {
  const unsigned grid = grid_of(a.rows, kRowThreads / TPR);
  if (a.causal || a.probs != nullptr)
    return launch_pdl(softmax_entropy_vec_kernel<TPR, NV, true, 1>, dim3(grid), dim3(kRowThreads), 0, s, a);
  return launch_pdl(softmax_entropy_vec_kernel<TPR, NV, false, MINB>, dim3(grid), dim3(kRowThreads), 0, s, a);
}

template <int TPR, int NV, int MINB = 1>
int run_pack_vec(const PackArgs& a, cudaStream_t s) {
  return launch_pdl(pack_rows_vec_kernel<TPR, NV, MINB>, dim3(grid_of(a.M, kRowThreads / TPR)), dim3(kRowThreads), 0,
                    s, a);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

// Router fast path: two blocks per SM (the ring's shared memory), never more blocks than
// rows; the bucket scan follows as a one-block launch that starts while the router drains.
template <int NV>
int run_route_tma(const SoftmaxArgs& a, cudaStream_t s) {
  constexpr size_t kSmem = 128 + size_t(kRouteSlots) * NV * 32 * 16 + 2 * kRouteSlots * 8 + 16;
  static std::once_flag once[64];
  static cudaError_t err[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -4;
  std::call_once(once[dev], [dev] {
    err[dev] = cudaFuncSetAttribute(route_rows_tma_kernel<NV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kSmem));
  });
  if (err[dev] != cudaSuccess) return -4;
  const int64_t fill = int64_t(sm_count()) * 2;
  const unsigned grid = static_cast<unsigned>(a.rows < fill ? a.rows : fill);
  int st = launch_pdl(route_rows_tma_kernel<NV>, dim3(grid), dim3(kRouteThreads), kSmem, s, a);
  if (st != 0 || a.chunk_tab == nullptr) return st;
  return launch_pdl(route_chunk_scan_kernel, dim3(1), dim3(kScanThreads), 0, s, static_cast<const int8_t*>(a.route),
                    a.rows, a.chunk_tab, a.counts);
}

int launch_softmax_entropy(const SoftmaxArgs& a, cudaStream_t s) {
  if (a.rows <= 0) return 0;
  const bool vec = (a.n % 8 == 0) && (a.ldx % 8 == 0) && aligned16(a.x) &&
                   (a.probs == nullptr || ((a.ldp % 8 == 0) && aligned16(a.probs)));
  if (vec && !a.causal && a.probs == nullptr && a.n <= 4096) {
    // entropy + route only (the gating step): rows staged by TMA bulk copies, one
    // consumer warp per row (route_rows_tma_kernel)
    if (a.n <= 1024) return run_route_tma<4>(a, s);
    if (a.n <= 2048) return run_route_tma<8>(a, s);
    return run_route_tma<16>(a, s);
  }
  if (vec) {
    // one warp per row up to 1024 columns (no block-level synchronisation), then 2 / 4 / 8
    // warps per row so every thread keeps at most 8 vectors (64 fp16) in registers.  A
    // sweep on B200 at 4096 columns (4096 and 16384 rows, L2 cold): 2 warps x 8 vectors
    // with registers capped for 4 resident blocks per SM was fastest (12.7 us / 36.4 us
    // against 14.7 / 39.4 uncapped).
    const int n = a.n;
    if (n <= 256) return run_softmax_vec<32, 1>(a, s);
    if (n <= 512) return run_softmax_vec<32, 2>(a, s);
    if (n <= 1024) return run_softmax_vec<32, 4>(a, s);
    if (n <= 2048) return run_softmax_vec<64, 4, 4>(a, s);
    if (n <= 4096) return run_softmax_vec<64, 8, 4>(a, s);
    if (n <= 8192) return run_softmax_vec<128, 8>(a, s);
    if (n <= 16384) return run_softmax_vec<256, 8>(a, s);
  }
  return launch_pdl(softmax_entropy_loop_kernel, dim3(static_cast<unsigned>(a.rows)), dim3(256), 0, s, a);
}

int launch_pack_rows(const PackArgs& a, cudaStream_t s) {
  if (a.M <= 0) return 0;
  const int K = a.K;

  // The same sweep for the packing (K = 4096: 4 warps x 4 vectors, 12.7 us against 14.9
  // for 2 x 8; K = 14336: 8 warps x 7 vectors, which covers the row exactly).
  if (K <= 512) return run_pack_vec<32, 2>(a, s);
  if (K <= 1024) return run_pack_vec<32, 4>(a, s);
  if (K <= 2048) return run_pack_vec<64, 4, 4>(a, s);
  if (K <= 4096) return run_pack_vec<128, 4, 4>(a, s);
  if (K <= 8192) return run_pack_vec<128, 8>(a, s);
  if (K <= 14336) return run_pack_vec<256, 7, 2>(a, s);
  if (K <= 16384) return run_pack_vec<256, 8, 2>(a, s);
  return launch_pdl(pack_rows_loop_kernel, dim3(static_cast<unsigned>(a.M)), dim3(256), 0, s, a);
}

int launch_quantize_weights(const void* W, int64_t ldw, int64_t N, int64_t K, int8_t* w_kn, int8_t* w_nk,
                            float* scale, int div_mode, cudaStream_t s) {
  if (N <= 0) return 0;
  quantize_weights_kernel<<<static_cast<unsigned>(N), 256, 0, s>>>(static_cast<const __half*>(W), ldw, N, K, w_kn,
                                                                   w_nk, scale, div_mode);
  return status_of(cudaGetLastError());
}

int launch_pack_weights(const int8_t* w_kn, const float* scale, int64_t K, int64_t N, int8_t* w_i8,
                        uint8_t* w_e4m3, void* w_f16, cudaStream_t s) {
  if (K <= 0 || N <= 0) return 0;
  dim3 grid(static_cast<unsigned>((K + 31) / 32), static_cast<unsigned>((N + 31) / 32));
  pack_weights_kernel<<<grid, 256, 0, s>>>(w_kn, scale, K, N, w_i8, w_e4m3, static_cast<__half*>(w_f16));
  return status_of(cudaGetLastError());
}

int launch_attention_entropy(const void* P, bool f32, int64_t rows, int64_t n, int64_t ld, float* H, cudaStream_t s) {
  if (rows <= 0) return 0;
  const int64_t want = (rows + 7) / 8;  // 8 rows (warps) per block; a few waves of 148 SMs at most
  const unsigned grid = static_cast<unsigned>(want < int64_t(sm_count()) * 16 ? want : int64_t(sm_count()) * 16);
  const int width = f32 ? 4 : 8;  // elements per 16-byte vector
  const bool vec = aligned16(P) && n % width == 0 && ld % width == 0;
  if (f32) {
    if (vec) attention_entropy_kernel<true, true><<<grid, 256, 0, s>>>(P, rows, n, ld, H);
    else attention_entropy_kernel<true, false><<<grid, 256, 0, s>>>(P, rows, n, ld, H);
  } else {
    if (vec) attention_entropy_kernel<false, true><<<grid, 256, 0, s>>>(P, rows, n, ld, H);
    else attention_entropy_kernel<false, false><<<grid, 256, 0, s>>>(P, rows, n, ld, H);
  }
  return status_of(cudaGetLastError());
}

int launch_batch_mean(const float* H, int64_t B, int64_t per_batch, float* out, cudaStream_t s) {
  if (B <= 0) return 0;
  batch_mean_kernel<<<static_cast<unsigned>(B), 256, 0, s>>>(H, per_batch, out);
  return status_of(cudaGetLastError());
}

int launch_head_mean(const float* H, int64_t B, int64_t Hq, int64_t S, float* out, cudaStream_t s) {
  if (B * S <= 0) return 0;
  return launch_pdl(head_mean_kernel, dim3(static_cast<unsigned>((B * S + 255) / 256)), dim3(256), 0, s, H, B, Hq, S,
                    out);
}

int launch_batch_max_fill(const float* Hb, int64_t B, float* out, int64_t M, cudaStream_t s) {
  if (B <= 0 || M <= 0) return 0;
  const int64_t blocks = std::min<int64_t>((M + 255) / 256, 1024);
  return launch_pdl(batch_max_fill_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, Hb, B, out, M);
}

int launch_fill_value(float* out, int64_t M, float v, cudaStream_t s) {
  if (M <= 0) return 0;
  const int64_t blocks = std::min<int64_t>((M + 255) / 256, 1024);
  return launch_pdl(fill_value_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, out, M, v);
}

int launch_batch_max_route(const float* H, int64_t n, double tl, double th, float* max_out, int8_t* tier_out,
                           cudaStream_t s) {
  batch_max_route_kernel<<<1, 256, 0, s>>>(H, n, tl, th, max_out, tier_out);
  return status_of(cudaGetLastError());
}

int launch_route_entropies(const float* H, int64_t rows, double tl, double th, float* Hws, int8_t* route, int4* tab,
                           int32_t* counts, uint32_t* ticket, cudaStream_t s) {
  if (rows <= 0) return 0;
  route_entropies_kernel<<<grid_of(rows, 256), 256, 0, s>>>(H, rows, tl, th, Hws, route, tab, counts, ticket);
  return status_of(cudaGetLastError());
}

int launch_route(const float* H, int64_t rows, double tl, double th, int8_t* route, cudaStream_t s) {
  if (rows <= 0) return 0;
  route_kernel<<<grid_of(rows, 256), 256, 0, s>>>(H, rows, tl, th, route);
  return status_of(cudaGetLastError());
}

int prepare_device() {
  static std::once_flag attr_once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -4;
  std::call_once(attr_once[dev], [dev] {
    attr_err[dev] = cudaFuncSetAttribute(gated_gemm_kernel<kBN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(SingleCfg<kBN>::kSmem));
    if (attr_err[dev] == cudaSuccess)
      attr_err[dev] = cudaFuncSetAttribute(gated_gemm_kernel<kBNNarrow>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(SingleCfg<kBNNarrow>::kSmem));
    if (attr_err[dev] == cudaSuccess)
      attr_err[dev] = cudaFuncSetAttribute(gated_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(kGemmSmemPair));
    if (attr_err[dev] == cudaSuccess)
      attr_err[dev] = cudaFuncSetAttribute(gated_gemm_skinny_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(SkinnyCfg<16>::kSmem));
    if (attr_err[dev] == cudaSuccess)
      attr_err[dev] = cudaFuncSetAttribute(gated_gemm_skinny_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(SkinnyCfg<32>::kSmem));
    if (attr_err[dev] == cudaSuccess)
      attr_err[dev] = cudaFuncSetAttribute(gated_gemm_skinny_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(SkinnyCfg<64>::kSmem));
    if (attr_err[dev] == cudaSuccess)
      attr_err[dev] = cudaFuncSetAttribute(gated_gemm_skinny_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(SkinnyCfg<128>::kSmem));
  });
  return attr_err[dev] == cudaSuccess ? 0 : -4;
}

int launch_gated_gemm_pair(const GemmMaps& m, const GemmArgs& args, int pairs, cudaStream_t s) {
  if (prepare_device() != 0) return -4;
  if (pairs <= 0) return 0;
  return launch_pdl(gated_gemm_pair_kernel, dim3(2 * pairs), dim3(kGemmThreads), kGemmSmemPair, s, m.a8, m.a16, m.w[0],
                    m.w[1], m.w[2], m.a8h, m.a16h, args);
}

int launch_gated_gemm(const GemmMaps& m, const GemmArgs& args, int grid, int bn, cudaStream_t s) {
  if (prepare_device() != 0) return -4;
  if (grid <= 0) return 0;
  if (bn == kBNNarrow)
    return launch_pdl(gated_gemm_kernel<kBNNarrow>, dim3(grid), dim3(kGemmThreads), SingleCfg<kBNNarrow>::kSmem, s,
                      m.a8, m.a16, m.w[0], m.w[1], m.w[2], args);
  return launch_pdl(gated_gemm_kernel<kBN>, dim3(grid), dim3(kGemmThreads), SingleCfg<kBN>::kSmem, s, m.a8, m.a16,
                    m.w[0], m.w[1], m.w[2], args);
}

int launch_reduce_partials(const GemmArgs& args, bool pair, int64_t tiles, cudaStream_t s) {
  if (args.part == nullptr || tiles <= 0) return 0;
  const int ranks = pair ? 2 : 1;
  const dim3 grid(static_cast<unsigned>(tiles * ranks * 4));
  return launch_pdl(reduce_partials_kernel, grid, dim3(kReduceThreads), 0, s, args, pair ? kPairRows : kBM, ranks,
                    (pair && args.out_mode != 2) ? 1 : 0);
}

int launch_gated_gemm_skinny(const GemmMaps& m, const GemmArgs& args, int nb, int splits, cudaStream_t s) {
  if (prepare_device() != 0) return -4;
  if (splits < 1 || splits > kSkinnyMaxSplits) return -1;
  const unsigned ntn = static_cast<unsigned>((args.N + kSkinnyRows - 1) / kSkinnyRows);
  if (ntn == 0) return 0;
  const dim3 grid(ntn * static_cast<unsigned>(splits), 3);
  const dim3 block(kSkinnyThreads);
  const unsigned cx = static_cast<unsigned>(splits);
  switch (nb) {
    case 16:
      return launch_cluster_pdl(gated_gemm_skinny_kernel<16>, grid, block, SkinnyCfg<16>::kSmem, cx, s, m.a8, m.a16,
                                m.w[0], m.w[1], m.w[2], args);
    case 32:
      return launch_cluster_pdl(gated_gemm_skinny_kernel<32>, grid, block, SkinnyCfg<32>::kSmem, cx, s, m.a8, m.a16,
                                m.w[0], m.w[1], m.w[2], args);
    case 64:
      return launch_cluster_pdl(gated_gemm_skinny_kernel<64>, grid, block, SkinnyCfg<64>::kSmem, cx, s, m.a8, m.a16,
                                m.w[0], m.w[1], m.w[2], args);
    case 128:
      return launch_cluster_pdl(gated_gemm_skinny_kernel<128>, grid, block, SkinnyCfg<128>::kSmem, cx, s, m.a8,
                                m.a16, m.w[0], m.w[1], m.w[2], args);
    default:
      return -1;
  }
}

int launch_transpose_v(const void* V, int64_t B, int64_t Hkv, int64_t S, int64_t S_pad, int64_t D, int64_t sb,
                       int64_t sh, int64_t ss, void* VT, cudaStream_t s) {
  if (B * Hkv <= 0 || S_pad <= 0) return 0;
  const dim3 grid(static_cast<unsigned>((S_pad + 31) / 32), static_cast<unsigned>(B * Hkv));
  if (D == 64)
    return launch_pdl(transpose_v_kernel<64>, grid, dim3(256), 0, s, static_cast<const __half*>(V), Hkv, S, S_pad, sb,
                      sh, ss, static_cast<__half*>(VT));
  return launch_pdl(transpose_v_kernel<128>, grid, dim3(256), 0, s, static_cast<const __half*>(V), Hkv, S, S_pad, sb,
                    sh, ss, static_cast<__half*>(VT));
}

int launch_add_rmsnorm(const AddNormArgs& a, cudaStream_t s) {
  if (a.M <= 0) return 0;
  // TPR threads per row, NV 16-byte vectors per thread (rows up to TPR * NV * 8)
  if (a.d <= 1024)
    return launch_pdl(add_rmsnorm_kernel<32, 4>, dim3(grid_of(a.M, kNormThreads / 32)), dim3(kNormThreads), 0, s, a);
  if (a.d <= 2048)
    return launch_pdl(add_rmsnorm_kernel<64, 4>, dim3(grid_of(a.M, kNormThreads / 64)), dim3(kNormThreads), 0, s, a);
  if (a.d <= 4096)
    return launch_pdl(add_rmsnorm_kernel<128, 4>, dim3(grid_of(a.M, kNormThreads / 128)), dim3(kNormThreads), 0, s, a);
  if (a.d <= 8192)
    return launch_pdl(add_rmsnorm_kernel<256, 4>, dim3(grid_of(a.M, 1)), dim3(kNormThreads), 0, s, a);
  return -1;
}

int launch_rope_layout(const RopeArgs& a, int D, cudaStream_t s) {
  if (a.B * a.S <= 0) return 0;
  const dim3 grid(static_cast<unsigned>(a.B * a.S));
  if (D == 64) return launch_pdl(rope_layout_kernel<64>, grid, dim3(256), 0, s, a);
  return launch_pdl(rope_layout_kernel<128>, grid, dim3(256), 0, s, a);
}

int launch_flash_attention(const AttnLaunch& a, cudaStream_t s) {
  static std::once_flag once[64];
  static cudaError_t err[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -4;
  std::call_once(once[dev], [dev] {
    err[dev] = cudaFuncSetAttribute(flash_attention_entropy_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(AttnCfg<64>::kSmem));
    if (err[dev] == cudaSuccess)
      err[dev] = cudaFuncSetAttribute(flash_attention_entropy_kernel<128>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(AttnCfg<128>::kSmem));
  });
  if (err[dev] != cudaSuccess) return -4;
  AttnArgs args;
  args.B = a.B;
  args.Hq = a.Hq;
  args.Hkv = a.Hkv;
  args.S = a.S;
  args.S_pad = a.S_pad;
  args.scale = a.scale;
  args.causal = a.causal;
  args.O = static_cast<__half*>(a.O);
  args.H = a.H;
  args.ml = static_cast<float2*>(a.ml);
  // persistent: one CTA per SM (its shared memory), each taking units of 256 query rows
  const int64_t nqc = (a.S + 2 * kAttnTile - 1) / (2 * kAttnTile);
  const int64_t units = a.B * a.Hq * nqc;
  const int64_t sms = sm_count();
  const dim3 grid(static_cast<unsigned>(units < sms ? units : sms));
  if (a.D == 64)
    return launch_pdl(flash_attention_entropy_kernel<64>, grid, dim3(kAttnThreads), AttnCfg<64>::kSmem, s, a.q, a.k,
                      a.vt, args);
  return launch_pdl(flash_attention_entropy_kernel<128>, grid, dim3(kAttnThreads), AttnCfg<128>::kSmem, s, a.q, a.k,
                    a.vt, args);
}

int launch_attention_entropy_exact(const AttnLaunch& a, cudaStream_t s) {
  static std::once_flag once[64];
  static cudaError_t err[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || a.ml == nullptr) return -4;
  std::call_once(once[dev], [dev] {
    err[dev] = cudaFuncSetAttribute(attention_entropy_exact_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(ExactCfg<64>::kSmem));
    if (err[dev] == cudaSuccess)
      err[dev] = cudaFuncSetAttribute(attention_entropy_exact_kernel<128>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(ExactCfg<128>::kSmem));
  });
  if (err[dev] != cudaSuccess) return -4;
  AttnArgs args;
  args.B = a.B;
  args.Hq = a.Hq;
  args.Hkv = a.Hkv;
  args.S = a.S;
  args.S_pad = a.S_pad;
  args.scale = a.scale;
  args.causal = a.causal;
  args.O = nullptr;
  args.H = a.H;
  args.ml = static_cast<float2*>(a.ml);
  // persistent like the flash kernel: one CTA per SM taking the same units in the same order
  const int64_t nqc = (a.S + 2 * kAttnTile - 1) / (2 * kAttnTile);
  const int64_t units = a.B * a.Hq * nqc;
  const int64_t sms = sm_count();
  const dim3 grid(static_cast<unsigned>(units < sms ? units : sms));
  if (a.D == 64)
    return launch_pdl(attention_entropy_exact_kernel<64>, grid, dim3(kAttnThreads), ExactCfg<64>::kSmem, s, a.q,
                      a.k, args);
  return launch_pdl(attention_entropy_exact_kernel<128>, grid, dim3(kAttnThreads), ExactCfg<128>::kSmem, s, a.q,
                    a.k, args);
}

int launch_kv_append(const KvCacheArgs& c, const void* k_rows, int64_t ldk, const void* v_rows, int64_t ldv,
                     const int8_t* tier, int64_t t_new, cudaStream_t s) {
  if (c.batch <= 0 || t_new <= 0) return 0;
  const dim3 grid(static_cast<unsigned>(c.batch * t_new));
  const auto* kr = static_cast<const __half*>(k_rows);
  const auto* vr = static_cast<const __half*>(v_rows);
  int st = c.head_dim == 64
               ? launch_pdl(kv_append_kernel<64>, grid, dim3(kKvThreads), 0, s, c, kr, ldk, vr, ldv, tier, t_new)
               : launch_pdl(kv_append_kernel<128>, grid, dim3(kKvThreads), 0, s, c, kr, ldk, vr, ldv, tier, t_new);
  if (st != 0) return st;
  return launch_pdl(kv_commit_kernel, dim3(static_cast<unsigned>((c.batch + 127) / 128)), dim3(128), 0, s, c, t_new);
}

namespace {
template <int D, int G>
int run_kv_decode(const KvCacheArgs& c, const void* q, int64_t ldq, const void* k_new, const void* v_new,
                  int64_t ld_new, float scale, int splits, float* part, cudaStream_t s) {
  constexpr int GC = G;  // every query head of the KV head in one CTA (rows of the M = 16 MMA)
  static std::once_flag once[64];
  static cudaError_t err[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -4;
  std::call_once(once[dev], [dev] {
    err[dev] = cudaFuncSetAttribute(kv_decode_attention_kernel<D, G, GC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(KvPipe<D>::kSmem));
  });
  if (err[dev] != cudaSuccess) return -4;
  const dim3 grid(static_cast<unsigned>(c.batch * c.kv_heads), static_cast<unsigned>(splits), G / GC);
  return launch_pdl(kv_decode_attention_kernel<D, G, GC>, grid, dim3(kKvPipeThreads), KvPipe<D>::kSmem, s, c,
                    static_cast<const __half*>(q), ldq, static_cast<const __half*>(k_new),
                    static_cast<const __half*>(v_new), ld_new, scale, splits, part);
}
template <int D>
int run_kv_decode_g(const KvCacheArgs& c, int64_t G, const void* q, int64_t ldq, const void* k_new,
                    const void* v_new, int64_t ld_new, float scale, int splits, float* part, cudaStream_t s) {
  switch (G) {
    case 1: return run_kv_decode<D, 1>(c, q, ldq, k_new, v_new, ld_new, scale, splits, part, s);
    case 2: return run_kv_decode<D, 2>(c, q, ldq, k_new, v_new, ld_new, scale, splits, part, s);
    case 4: return run_kv_decode<D, 4>(c, q, ldq, k_new, v_new, ld_new, scale, splits, part, s);
    case 8: return run_kv_decode<D, 8>(c, q, ldq, k_new, v_new, ld_new, scale, splits, part, s);
    default: return -3;
  }
}
}  // namespace

int launch_kv_decode_attention(const KvCacheArgs& c, const void* q, int64_t ldq, int64_t Hq, const void* k_new,
                               const void* v_new, int64_t ld_new, float scale, int splits, float* part, void* out,
                               int64_t ldo, float* H, cudaStream_t s) {
  if (c.batch <= 0) return 0;
  const int64_t G = Hq / c.kv_heads;
  int st = c.head_dim == 64 ? run_kv_decode_g<64>(c, G, q, ldq, k_new, v_new, ld_new, scale, splits, part, s)
                            : run_kv_decode_g<128>(c, G, q, ldq, k_new, v_new, ld_new, scale, splits, part, s);
  if (st != 0) return st;
  const dim3 grid(static_cast<unsigned>(c.batch * Hq));
  if (c.head_dim == 64)
    return launch_pdl(kv_decode_combine_kernel<64>, grid, dim3(kKvThreads), 0, s, part, splits,
                      static_cast<__half*>(out), ldo, H, static_cast<int>(Hq));
  return launch_pdl(kv_decode_combine_kernel<128>, grid, dim3(kKvThreads), 0, s, part, splits,
                    static_cast<__half*>(out), ldo, H, static_cast<int>(Hq));
}

int read_and_clear_device_error(int* value) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) return -4;
  if (v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return -4;
  }
  *value = v;
  return 0;
}

}  // namespace ee
