// ee_internal.h - declarations shared by the device translation unit (ee_kernels.cu)
// and the C-ABI translation unit (ee_capi.cu).  Not part of the public interface.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace ee {

// Precision buckets (route ids); the numbering is the reference's PrecisionTier.
enum Bucket : int { kINT8 = 0, kFP8 = 1, kFP16 = 2 };

// Device error word bits (read back by ee_device_check).
enum DeviceError : int {
  kErrWaitTimeout = 1,  // an mbarrier wait in the GEMM gave up
  kErrTmem = 2,         // tensor-memory allocation returned an unusable address
  kErrShape = 4,        // a bucket holds more rows than the kernel's tile was launched for
  kErrCapacity = 8,     // a KV-cache pool or sequence was full: the token was not stored
};

// ----------------------------------------------------------------- row kernels
struct SoftmaxArgs {
  const void* x;      // fp16 [rows, n] with row stride ldx (elements)
  int64_t ldx;
  int64_t rows;
  int n;
  int causal;         // mask column j of row r when j > r % S
  int64_t S;
  void* probs;        // fp16 [rows, n] with row stride ldp, nullable
  int64_t ldp;
  float* H;           // fp32 [rows], required
  int8_t* route;      // int8 [rows], nullable
  double tau_low, tau_high;  // compared in double, like the reference's Python floats
  // bucket scan (all nullable together; needs route): the last block to finish counts
  // the routes per 16-row chunk and writes, per chunk, the rows of each bucket in all
  // earlier chunks (int4: INT8, FP8, FP16, 0) plus the bucket totals.  A row's
  // position in the stable bucket order then follows from its own chunk alone.
  int4* chunk_tab;    // [ceil(rows / 16)]
  int32_t* counts;    // [4] rows per bucket (INT8, FP8, FP16) + spare
  uint32_t* ticket;   // zero-initialised counter; left at zero by the kernel
};
int launch_softmax_entropy(const SoftmaxArgs& a, cudaStream_t s);

struct PackArgs {
  const void* A;      // fp16 [M, K], row stride lda (elements)
  int64_t lda;
  int64_t M;
  int K;
  const int8_t* route;  // nullable: every row goes to fixed_bucket
  int fixed_bucket;
  // bucket placement (nullable together, needs route; else position = row): the scan
  // of SoftmaxArgs.  Each row's position = bucket offset + rows of its bucket in earlier
  // chunks + rows of its bucket before it in its chunk; perm[position] = row and
  // slot[row] = position are written on the way.
  const int4* chunk_tab;
  const int32_t* counts;
  int32_t* perm;
  int32_t* slot;
  float* sa;            // [positions] per-row activation scale (8-bit buckets)
  uint8_t* buf8;        // [positions, K] int8 / e4m3 rows, row stride ld8 bytes
  int64_t ld8;
  void* buf16;          // [positions, K] fp16 rows, row stride ld16 elements, nullable if unused
  int64_t ld16;
};
int launch_pack_rows(const PackArgs& a, cudaStream_t s);

// per-output-channel INT8 weight quantisation of W fp16 [N, K]
// div_mode 0: scale = amax * fp32(1/127) (torch on CUDA); 1: scale = amax / 127 (torch on CPU)
int launch_quantize_weights(const void* W, int64_t ldw, int64_t N, int64_t K, int8_t* w_kn, int8_t* w_nk,
                            float* scale, int div_mode, cudaStream_t s);
// [K, N] int8 + scale[N] -> K-major packs for the three buckets
int launch_pack_weights(const int8_t* w_kn, const float* scale, int64_t K, int64_t N, int8_t* w_i8,
                        uint8_t* w_e4m3, void* w_f16, cudaStream_t s);
int launch_batch_mean(const float* H, int64_t B, int64_t per_batch, float* out, cudaStream_t s);
// per query position the mean over the heads of H [B, Hq, S] -> out [B * S]
int launch_head_mean(const float* H, int64_t B, int64_t Hq, int64_t S, float* out, cudaStream_t s);
// out[0 .. M) = max of Hb[0 .. B)
int launch_batch_max_fill(const float* Hb, int64_t B, float* out, int64_t M, cudaStream_t s);
// out[0 .. M) = v
int launch_fill_value(float* out, int64_t M, float v, cudaStream_t s);
// per-row attention entropy of probabilities fp16 (f32 = false) or fp32 [rows, n], row stride ld
int launch_attention_entropy(const void* P, bool f32, int64_t rows, int64_t n, int64_t ld, float* H, cudaStream_t s);
int launch_batch_max_route(const float* H, int64_t n, double tl, double th, float* max_out, int8_t* tier_out,
                           cudaStream_t s);
int launch_route(const float* H, int64_t rows, double tl, double th, int8_t* route, cudaStream_t s);
// route ids of given entropies + the bucket scan (SoftmaxArgs' chunk_tab / counts / ticket)
int launch_route_entropies(const float* H, int64_t rows, double tl, double th, float* Hws, int8_t* route, int4* tab,
                           int32_t* counts, uint32_t* ticket, cudaStream_t s);

// ----------------------------------------------------------------- gated GEMM
constexpr int kBM = 128;          // rows per tile (UMMA M)
constexpr int kBN = 256;          // columns per tile (UMMA N)
constexpr int kBNNarrow = 64;     // columns per tile of the single-CTA kernel for few-row (weight-streaming) calls
constexpr int kBKBytes = 128;     // bytes of K per pipeline stage (one 128B swizzle row)

struct GemmArgs {
  int M_cap;               // positions covered by the A tensor maps
  int N, K;
  const int32_t* dyn_counts;  // device [3] rows per bucket, or null to use counts[]
  int counts[3];
  const int32_t* perm;     // position -> output row, nullable (identity)
  const float* sa;         // [M_cap] activation scale per position (INT8 / FP8 buckets)
  const float* sb;         // [N] weight scale per output channel (INT8 / FP8 buckets)
  void* Y;                 // fp16 [rows, N] (out_mode 0) or 32-bit [rows, N] (out_mode 1)
  int64_t ldy;             // elements
  int out_mode;            // 0: dequantised fp16, 1: raw accumulators (int32 / fp32),
                           // 2: SwiGLU of gate / up rows interleaved by 128 (fp16 [rows, N/2])
  uint32_t* sched;         // nullable: [0] next tile, [1] CTAs done -- zero at launch, left zero;
                           // null = static round-robin tile order
  // K-split of the tiles (part == null: every tile whole).  The kernel splits the K loop
  // of a tile into up to kMaxKSplits ranges (the same choice in every CTA, from the
  // bucket counts, K and split_slots), each range's raw accumulator goes to one partial
  // block, and reduce_partials_kernel adds a split tile's blocks in range order and runs
  // its epilogue.
  uint32_t* part;          // part_blocks blocks of kPartBlockBytes (int32 / fp32 partials)
  int part_blocks;
  int split_slots;         // CTAs (single-CTA kernel) or CTA pairs of the launch
  int32_t* split_plan;     // [3] ranges per tile of each bucket, written by the GEMM's first
                           // CTA for the reduction kernel (with part)
  int drop_load_cta;       // failure-detection test hook of the single-CTA kernel: 0 none, else
                           // c + 1 -- CTA c issues neither the copies nor the arrival of its
                           // first K stage, so its MMA warp's bounded wait on that stage gives up
};
constexpr int kPartBlockBytes = 128 * 256 * 4;  // one CTA's 128 x 256 accumulator
constexpr int kMaxKSplits = 16;
constexpr int kSplitMinKBlocks = 8;             // fewest K stages of one split range
struct GemmMaps {
  CUtensorMap a8;          // uint8 [M_cap, K], box {128, 128}
  CUtensorMap a16;         // fp16  [M_cap, K], box {64, 128}
  CUtensorMap w[3];        // bucket weights [N, K] K-major, box {128 B, 256}
  CUtensorMap a8h, a16h;   // the same A tensors with 64-row boxes (CTA-pair half tiles)
};
// single-CTA kernel, 128 x bn tiles (bn = kBN, or kBNNarrow for weight-streaming calls)
int launch_gated_gemm(const GemmMaps& maps, const GemmArgs& args, int grid, int bn, cudaStream_t s);
// CTA-pair kernel: 256-row tiles; grid = 2 x pairs; the A / W maps use 128-row boxes
int launch_gated_gemm_pair(const GemmMaps& maps, const GemmArgs& args, int pairs, cudaStream_t s);
// the K-split tiles' reduction and epilogue after either kernel (args.part != null):
// one 256-thread block per (tile, CTA of the tile, 32-row quarter); tiles = an upper
// bound of the call's tiles
int launch_reduce_partials(const GemmArgs& args, bool pair, int64_t tiles, cudaStream_t s);
constexpr int kPairTileRows = 256;
// weight-streaming kernel for at most 128 rows (ee_gemm_skinny.cuh): 128-channel tiles,
// nb = activation rows per tile (16, 32, 64 or 128, >= the rows of every bucket), K split
// over clusters of `splits` CTAs; the A maps use nb-row boxes, the W maps 128-row boxes
int launch_gated_gemm_skinny(const GemmMaps& maps, const GemmArgs& args, int nb, int splits, cudaStream_t s);
constexpr int kSkinnyMaxRows = 128;
constexpr int kSkinnyAutoRows = 64;
constexpr int kSkinnyMaxSplits = 8;

// device error word
int read_and_clear_device_error(int* value);

// entropy-tied KV cache (ee_kvcache.cuh); the fields of ee_kv_cache (include/ee_b200.h)
struct KvCacheArgs {
  int64_t batch, kv_heads, head_dim, max_tokens, slots8, slots16;
  uint8_t* k8;
  uint8_t* v8;
  void* k16;
  void* v16;
  float* k_scale;
  float* v_scale;
  int32_t* slot;
  int32_t* length;
  uint32_t* pool_used;
};
// append t_new tokens to every sequence (rows b * t_new + t of k_rows / v_rows), each at
// the tier tier[b * t_new + t]; then the lengths grow by t_new
int launch_kv_append(const KvCacheArgs& c, const void* k_rows, int64_t ldk, const void* v_rows, int64_t ldv,
                     const int8_t* tier, int64_t t_new, cudaStream_t s);
// attention of one new query row per sequence (q rows [batch, Hq * D], row stride ldq)
// over its cached tokens and its own new K / V rows (k_new / v_new [batch, kv_heads * D],
// row stride ld_new); part: batch * Hq * splits * (3 + D) floats
int launch_kv_decode_attention(const KvCacheArgs& c, const void* q, int64_t ldq, int64_t Hq, const void* k_new,
                               const void* v_new, int64_t ld_new, float scale, int splits, float* part, void* out,
                               int64_t ldo, float* H, cudaStream_t s);
// flash attention with row entropy (ee_attention.cuh): Q [B*Hq*S, D], K [B*Hkv*S, D],
// V^T [B*Hkv*D, S_pad] maps (box 64 x 128 / 64 x D), outputs O [B, S, Hq, D], H [B, Hq, S]
constexpr int kAttnTile = 128;  // queries per attention CTA and keys per KV tile
struct AttnLaunch {
  CUtensorMap q, k, vt;
  int64_t B, Hq, Hkv, S, S_pad, D;
  float scale;
  int causal;
  void* O;
  float* H;
  void* ml;  // nullable float2 [B, Hq, S]: each row's (m, l), for the exact-entropy pass
};
int launch_flash_attention(const AttnLaunch& a, cudaStream_t s);
// second pass: H [B, Hq, S] from the fp16-rounded probabilities the reference's eager
// path takes its entropy of (needs a.ml from launch_flash_attention; a.vt unused)
int launch_attention_entropy_exact(const AttnLaunch& a, cudaStream_t s);
// V element (b, h, s, c) at V + b * sb + h * sh + s * ss + c  ->  V^T [B*Hkv, D, S_pad]
int launch_transpose_v(const void* V, int64_t B, int64_t Hkv, int64_t S, int64_t S_pad, int64_t D, int64_t sb,
                       int64_t sh, int64_t ss, void* VT, cudaStream_t s);

// the Llama block's elementwise passes (ee_block.cuh)
struct AddNormArgs {
  const __half* x;      // [M, d], row stride ldx
  int64_t ldx;
  const __half* res;    // nullable: residual [M, d], row stride ldr (s = fp16(res + x))
  int64_t ldr;
  __half* sum_out;      // nullable (needs res): s, row stride lds
  int64_t lds;
  const __half* w;      // [d] RMSNorm weight
  __half* y;            // [M, d], row stride ldy
  int64_t ldy;
  int64_t M;
  int d;
  float eps;
};
int launch_add_rmsnorm(const AddNormArgs& a, cudaStream_t s);
struct RopeArgs {
  const __half* q;      // [B*S, Hq*D] rows of the q projection, row stride ldq
  int64_t ldq;
  const __half* k;      // [B*S, Hkv*D], row stride ldk
  int64_t ldk;
  const __half* cos;    // [B*S, D], row stride ld_cs
  const __half* sin;
  int64_t ld_cs;
  int64_t B, S;
  int Hq, Hkv;
  __half* q_out;        // [B, Hq, S, D]
  __half* k_out;        // [B, Hkv, S, D]
};
int launch_rope_layout(const RopeArgs& a, int D, cudaStream_t s);
// ee_gate_rows with the workspace-header memset optional (see ee_capi.cu)
// bytes at the start of a gated workspace that a caller zeroes once (header + look-back)
size_t gated_ws_head_bytes();
int gate_rows_impl(const void* logits, int64_t M, int64_t n, int64_t ld, double tau_low, double tau_high, float* H,
                   int8_t* route, int32_t* bucket_counts, void* workspace, size_t workspace_bytes, void* stream,
                   bool clear_header);

// one-time per-device set-up of kernel attributes (safe to call repeatedly); lets a
// caller finish it before a stream capture starts
int prepare_device();

// sets the text ee_last_error() returns on the calling thread
void set_last_error(const char* msg);

}  // namespace ee
