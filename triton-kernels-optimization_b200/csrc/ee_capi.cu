// ee_capi.cu - the extern "C" boundary (include/ee_b200.h): argument validation,
// status codes, workspace layout, TMA tensor-map encoding and kernel sequencing.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/ee_b200.h"
#include "ee_internal.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(EE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int check_launch(int st, const char* what) {
  if (st == 0) return EE_OK;
  cudaError_t e = cudaGetLastError();
  return fail(EE_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
constexpr int64_t kMaxDim = (int64_t(1) << 31) - 1;

// ---------------------------------------------------------------- driver entry point
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D K-major operand map: rows x K elements, 128-byte swizzled boxes of
// {128 bytes of K} x box_rows.
int encode_kmajor(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int64_t ld_elems, int elem_bytes,
                  int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(EE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (no CUDA driver?)");
  const CUtensorMapDataType dt = elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_elems) * elem_bytes};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elem_bytes), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(EE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return EE_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cache[dev & 63] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev & 63] = v;
  }
  return cache[dev & 63];
}

// ---------------------------------------------------------------- GEMM plumbing
struct GemmOperands {
  const void* a8 = nullptr;   // uint8 [M_cap, K] (INT8 / FP8 buckets)
  const void* a16 = nullptr;  // fp16  [M_cap, K] (FP16 bucket)
  int64_t ld8 = 0, ld16 = 0;
  const void* w[3] = {nullptr, nullptr, nullptr};  // [N, K] per bucket
};

int check_gemm_shape(int64_t M, int64_t N, int64_t K, int64_t ldy) {
  if (M < 0 || N <= 0 || K <= 0) return fail(EE_ERR_INVALID, "bad GEMM shape M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (M > kMaxDim || N > kMaxDim || K > kMaxDim) return fail(EE_ERR_UNSUPPORTED, "GEMM dimension >= 2^31");
  if (K % 16 != 0) return fail(EE_ERR_UNSUPPORTED, "K=%lld must be a multiple of 16", (long long)K);
  if (N % 8 != 0) return fail(EE_ERR_UNSUPPORTED, "N=%lld must be a multiple of 8", (long long)N);
  if (ldy < N || ldy % 8 != 0) return fail(EE_ERR_MISALIGNED, "ldy=%lld must be >= N and a multiple of 8", (long long)ldy);
  return EE_OK;
}

std::atomic<int> g_gemm_policy{0};  // 0 auto, 1 single-CTA 128x256, 2 CTA-pair 256x256, 3 single-CTA 128x64,
                                    // 4 weight-streaming (skinny) where the call has at most 128 rows
std::atomic<int> g_gemm_splits{0};  // skinny kernel's K splits per tile: 0 = chosen per call
std::atomic<int> g_drop_next_load{0};  // ee_debug_drop_next_gemm_load: armed CTA + 1, or 0

// K splits of the skinny kernel: one per 2048 of K (about 0.5 MB of fp16 weight per
// CTA), but no more than keep the three buckets' 128-channel tiles in one wave of
// resident CTAs (a second, partial wave costs more than the split saves), at most 8 (a
// portable cluster), at least 4 K blocks per split.  Measured on B200 at M = 16 .. 64:
// N = K = 4096 best at 2 splits, K = 14336 at 3-4, N = 14336 unsplit.
int skinny_splits(const ee::GemmArgs& args, int nb) {
  const int forced = g_gemm_splits.load(std::memory_order_relaxed);
  const int nkb = (args.K + ee::kBKBytes - 1) / ee::kBKBytes;  // 8-bit buckets: the fewest K blocks
  int s = forced;
  if (s <= 0) {
    const int64_t ntn = (args.N + 127) / 128;
    const int64_t slots = int64_t(num_sms()) * (nb <= 64 ? 2 : 1);
    s = static_cast<int>(std::min<int64_t>(slots / (3 * ntn), (args.K + 2047) / 2048));
    s = std::min(s, std::max(1, nkb / 4));
  }
  return std::max(1, std::min(s, ee::kSkinnyMaxSplits));
}

// Row tiles a call may produce: with routing on the device the bucket sizes are unknown
// here, and each bucket boundary can add one partial tile.
int64_t row_tiles(const ee::GemmArgs& args, bool dynamic_counts, int64_t bm) {
  if (dynamic_counts) return (args.M_cap + bm - 1) / bm + 2;
  int64_t t = 0;
  for (int b = 0; b < 3; ++b) t += (args.counts[b] + bm - 1) / bm;
  return t;
}

// K split allowed for a call whose whole 256-column tiles number `tiles` on `slots`
// CTAs (pairs): long K loops, tiles for at most 3/4 of the slots (measured on B200:
// splitting pays for K >= 8192; at K = 4096 the unsplit tiles are as fast, and where the
// device plans no split the reduction launch alone costs ~5 us)
bool split_eligible(const ee::GemmArgs& args, int64_t tiles, int64_t slots) {
  return args.part != nullptr && args.K >= 8192 && 4 * tiles <= 3 * slots;
}

// The CTA-pair kernel (forced; the automatic policy takes single-CTA tiles there when they
// may split) between 513 and 768 rows may also split with up to two tiles per pair: there
// the FP16 tiles (twice the 8-bit tiles' K loop) set the makespan while the 8-bit tiles
// fit in one round, and the device's plan splits the FP16 tiles, alone or with the 8-bit
// ones (measured on B200, K 14336 x N 4096, the bench's routing law, back-to-back calls:
// 768 rows 95.1 -> 87.9 us).  At 1024 rows the 8-bit tiles alone can fill the pairs (80
// tiles on 74), the plan then keeps every tile whole, and the reduction launch alone cost
// 6.5 us (100.6 -> 107.1 us), so the gate stops at 768.
bool pair_split_eligible(const ee::GemmArgs& args, int64_t tiles, int64_t pairs) {
  return args.part != nullptr && args.K >= 8192 && args.M_cap > 512 && args.M_cap <= 768 && tiles <= 2 * pairs;
}

// Between 513 and 768 rows with K >= 8192 the automatic policy takes single-CTA 128 x 256
// tiles, which may split with up to two tiles per SM: with 128-row tiles the 8-bit
// buckets' tiles fit in one round of the 148 CTAs, so the plan can level the makespan by
// splitting the FP16 tiles (measured on B200, K 14336 x N 4096, the bench's routing law,
// back-to-back calls: 768 rows 95.1 us with whole pair tiles, 87.9 with the pairs' split,
// 79.7 here).  Above 768 rows the single-CTA tiles' larger operand traffic per flop costs
// more than the levelling saves (1024 rows 106.9 us against 100.5 for whole pair tiles,
// 1280 rows 113.5 against 104.6), so the pairs keep those.
bool single_split_eligible(const ee::GemmArgs& args, int64_t tiles, int64_t sms) {
  return args.part != nullptr && args.K >= 8192 && args.M_cap > 512 && args.M_cap <= 768 && tiles <= 2 * sms;
}

// Automatic policy between 129 and 512 rows: single-CTA 128 x 256 tiles instead of CTA
// pairs when they need fewer rounds of the persistent grid, or when only they qualify
// for the K split (measured on B200 with 20/60/20 routing, back-to-back calls: 256 rows
// x N 14336 49 us against 58, 512 rows x K 14336 69 us against 82; pairs stay ahead or
// equal on the other Llama-3-8B shapes).  Between 513 and 768 rows: single-CTA tiles
// when they may split (single_split_eligible); above 768 rows always pairs.
bool single_beats_pairs(const ee::GemmArgs& args, bool dynamic_counts) {
  if (args.M_cap > 768) return false;
  const int64_t ntn = (args.N + ee::kBN - 1) / ee::kBN;
  const int64_t st = row_tiles(args, dynamic_counts, ee::kBM) * ntn;
  if (args.M_cap > 512) return single_split_eligible(args, st, num_sms());
  const int64_t pt = row_tiles(args, dynamic_counts, ee::kPairTileRows) * ntn;
  const int64_t sms = num_sms(), pairs = num_sms() / 2;
  const int64_t s_rounds = (st + sms - 1) / sms, p_rounds = (pt + pairs - 1) / pairs;
  return s_rounds < p_rounds || (split_eligible(args, st, sms) && !split_eligible(args, pt, pairs));
}

// Encodes the maps for the operands present and launches the persistent kernel.  Auto
// policy: more than 128 rows -> the CTA-pair kernel (256 x 256 tiles); at most 128 rows
// the call streams its weights -> single-CTA tiles, 128 x 256 when their count already
// covers the SMs, else 128 x 64 so that the weight spreads over every SM (measured on
// B200: M = 16..128 at N = 4096 36 us instead of 42, at N = 14336 the wide tiles stay
// faster, 58 us against 95).  Unused map slots get a copy of a valid map (never
// dereferenced).
int run_gemm(const GemmOperands& op, ee::GemmArgs args, bool dynamic_counts, cudaStream_t s) {
  const int policy = g_gemm_policy.load(std::memory_order_relaxed);
  // weight-streaming kernel: forced (policy 4) up to 128 rows, automatic up to 64 (at 128
  // rows the 128 x 64 tiles of the persistent kernel measured faster on B200)
  if (args.out_mode != 2 &&
      ((policy == 4 && args.M_cap <= ee::kSkinnyMaxRows) || (policy == 0 && args.M_cap <= ee::kSkinnyAutoRows))) {
    const int nb = args.M_cap <= 16 ? 16 : args.M_cap <= 32 ? 32 : args.M_cap <= 64 ? 64 : 128;
    ee::GemmMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    const CUtensorMap* any = nullptr;
    int st;
    if (op.a8) {
      if ((st = encode_kmajor(&maps.a8, op.a8, args.M_cap, args.K, op.ld8, 1, nb)) != EE_OK) return st;
      any = &maps.a8;
    }
    if (op.a16) {
      if ((st = encode_kmajor(&maps.a16, op.a16, args.M_cap, args.K, op.ld16, 2, nb)) != EE_OK) return st;
      any = any ? any : &maps.a16;
    }
    for (int b = 0; b < 3; ++b) {
      if (op.w[b]) {
        const int eb = (b == ee::kFP16) ? 2 : 1;
        if ((st = encode_kmajor(&maps.w[b], op.w[b], args.N, args.K, args.K, eb, 128)) != EE_OK) return st;
      }
    }
    if (any == nullptr) return fail(EE_ERR_INVALID, "GEMM without an A operand");
    if (!op.a8) maps.a8 = *any;
    if (!op.a16) maps.a16 = *any;
    for (int b = 0; b < 3; ++b)
      if (!op.w[b]) maps.w[b] = op.w[0] ? maps.w[0] : (op.w[1] ? maps.w[1] : maps.w[2]);
    return check_launch(ee::launch_gated_gemm_skinny(maps, args, nb, skinny_splits(args, nb), s),
                        "gated_gemm_skinny_kernel");
  }
  const int64_t wide_tiles = row_tiles(args, dynamic_counts, ee::kBM) * ((args.N + ee::kBN - 1) / ee::kBN);
  const bool pair = policy == 2 || (policy == 0 && args.M_cap > ee::kBM && !single_beats_pairs(args, dynamic_counts));
  // K split (split_eligible): 256-column tiles, the device then plans the ranges from the
  // bucket counts
  const int64_t slots = pair ? num_sms() / 2 : num_sms();
  const int64_t split_tiles = pair ? row_tiles(args, dynamic_counts, ee::kPairTileRows) * ((args.N + ee::kBN - 1) / ee::kBN)
                                   : wide_tiles;
  const bool split = policy != 3 && (split_eligible(args, split_tiles, slots) ||
                                     (pair ? pair_split_eligible(args, split_tiles, slots)
                                           : single_split_eligible(args, split_tiles, slots)));
  if (!split) {
    args.part = nullptr;
    args.part_blocks = 0;
    args.split_plan = nullptr;
  }
  // the SwiGLU epilogue pairs 128-column groups inside a 256-column tile
  const bool narrow = !split && args.out_mode != 2 &&
                      (policy == 3 || (policy == 0 && !pair && args.M_cap <= ee::kBM && wide_tiles < num_sms()));
  const int bn = narrow ? ee::kBNNarrow : ee::kBN;
  const int wbox = pair ? ee::kBN / 2 : bn;
  ee::GemmMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  const CUtensorMap* any = nullptr;
  int st;
  if (op.a8) {
    if ((st = encode_kmajor(&maps.a8, op.a8, args.M_cap, args.K, op.ld8, 1, ee::kBM)) != EE_OK) return st;
    if (pair && (st = encode_kmajor(&maps.a8h, op.a8, args.M_cap, args.K, op.ld8, 1, ee::kBM / 2)) != EE_OK) return st;
    any = &maps.a8;
  }
  if (op.a16) {
    if ((st = encode_kmajor(&maps.a16, op.a16, args.M_cap, args.K, op.ld16, 2, ee::kBM)) != EE_OK) return st;
    if (pair && (st = encode_kmajor(&maps.a16h, op.a16, args.M_cap, args.K, op.ld16, 2, ee::kBM / 2)) != EE_OK)
      return st;
    any = any ? any : &maps.a16;
  }
  for (int b = 0; b < 3; ++b) {
    if (op.w[b]) {
      const int eb = (b == ee::kFP16) ? 2 : 1;
      if ((st = encode_kmajor(&maps.w[b], op.w[b], args.N, args.K, args.K, eb, wbox)) != EE_OK) return st;
    }
  }
  if (any == nullptr) return fail(EE_ERR_INVALID, "GEMM without an A operand");
  if (!op.a8) maps.a8 = *any;
  if (!op.a16) maps.a16 = *any;
  if (!pair || !op.a8) maps.a8h = maps.a8;  // never dereferenced then
  if (!pair || !op.a16) maps.a16h = maps.a16;
  for (int b = 0; b < 3; ++b)
    if (!op.w[b]) maps.w[b] = op.w[0] ? maps.w[0] : (op.w[1] ? maps.w[1] : maps.w[2]);

  const int64_t ntn = (args.N + bn - 1) / bn;
  const int64_t bm = pair ? ee::kPairTileRows : ee::kBM;
  const int64_t tiles = row_tiles(args, dynamic_counts, bm) * ntn;
  // a split call runs one CTA (pair) per slot: its units outnumber its tiles
  const int grid = static_cast<int>(split ? slots : (tiles < slots ? tiles : slots));
  args.split_slots = split ? grid : 0;
  if (!pair) args.drop_load_cta = g_drop_next_load.exchange(0, std::memory_order_relaxed);
  int st2 = pair ? check_launch(ee::launch_gated_gemm_pair(maps, args, grid, s), "gated_gemm_pair_kernel")
                 : check_launch(ee::launch_gated_gemm(maps, args, grid, bn, s), "gated_gemm_kernel");
  if (st2 != EE_OK || !split) return st2;
  return check_launch(ee::launch_reduce_partials(args, pair, tiles, s), "reduce_partials_kernel");
}

// The part of a gated workspace past this call's own layout (M rows, K) holds the K-split
// partial blocks of its GEMM; a workspace without that room runs every tile whole.
void attach_split_area(ee::GemmArgs& args, void* ws, size_t ws_bytes, int64_t M, int64_t K);

ee::GemmArgs base_args(int64_t M_cap, int64_t N, int64_t K, void* Y, int64_t ldy, int out_mode) {
  ee::GemmArgs a;
  std::memset(&a, 0, sizeof(a));
  a.M_cap = static_cast<int>(M_cap);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.Y = Y;
  a.ldy = ldy;
  a.out_mode = out_mode;
  return a;
}

// ---------------------------------------------------------------- workspaces
struct LinearWs {
  float* sa;
  uint8_t* q;
};
size_t linear_ws_bytes(int64_t M, int64_t K) { return align256(sizeof(float) * M) + align256(size_t(M) * K); }
LinearWs linear_ws(void* ws, int64_t M) {
  uint8_t* p = static_cast<uint8_t*>(ws);
  LinearWs w;
  w.sa = reinterpret_cast<float*>(p);
  w.q = p + align256(sizeof(float) * M);
  return w;
}

struct GatedWs {
  uint32_t* ticket;
  int32_t* counts;
  uint32_t* sched;  // GEMM tile scheduler words (zeroed by ee_gate_rows, left zero by the GEMM)
  int32_t* perm;
  int32_t* slot;
  int8_t* route;
  float* H;
  float* sa;
  int4* chunk_tab;  // per 16-row chunk: rows of each bucket in earlier chunks
  uint8_t* buf8;
  void* buf16;
};
size_t chunk_tab_bytes(int64_t M) { return align256(sizeof(int4) * size_t((M + 15) / 16)); }
// the header (bucket counters, ticket, GEMM tile counters): the part a caller zeroes
// once (ee_gate_rows zeroes it on every call)
constexpr size_t kWsHeadBytes = 256;
}  // namespace
size_t ee::gated_ws_head_bytes() { return kWsHeadBytes; }
namespace {
size_t gated_ws_bytes(int64_t M, int64_t K) {
  return kWsHeadBytes + 2 * align256(sizeof(int32_t) * M) + align256(M) + 2 * align256(sizeof(float) * M) +
         chunk_tab_bytes(M) + align256(size_t(M) * K) + align256(size_t(M) * K * 2);
}
GatedWs gated_ws(void* ws, int64_t M, int64_t K) {
  uint8_t* p = static_cast<uint8_t*>(ws);
  GatedWs w;
  w.ticket = reinterpret_cast<uint32_t*>(p);
  w.counts = reinterpret_cast<int32_t*>(p + 16);
  w.sched = reinterpret_cast<uint32_t*>(p + 64);
  p += kWsHeadBytes;
  w.perm = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * M);
  w.slot = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * M);
  w.route = reinterpret_cast<int8_t*>(p);
  p += align256(M);
  w.H = reinterpret_cast<float*>(p);
  p += align256(sizeof(float) * M);
  w.sa = reinterpret_cast<float*>(p);
  p += align256(sizeof(float) * M);
  w.chunk_tab = reinterpret_cast<int4*>(p);
  p += chunk_tab_bytes(M);
  w.buf8 = p;
  p += align256(size_t(M) * K);
  w.buf16 = p;
  return w;
}

void attach_split_area(ee::GemmArgs& args, void* ws, size_t ws_bytes, int64_t M, int64_t K) {
  const size_t base = gated_ws_bytes(M, K);  // a multiple of 256
  if (ws == nullptr || ws_bytes < base + 256 + 2 * size_t(ee::kPartBlockBytes)) return;
  const size_t blocks = (ws_bytes - base - 256) / ee::kPartBlockBytes;
  uint8_t* p = static_cast<uint8_t*>(ws) + base;
  args.split_plan = reinterpret_cast<int32_t*>(p);  // 256 bytes: the plan, then the blocks
  args.part = reinterpret_cast<uint32_t*>(p + 256);
  args.part_blocks = static_cast<int>(blocks < size_t(1) << 30 ? blocks : size_t(1) << 30);
}

// recommended room for the K-split partials: four blocks per SM (a split plan can run up
// to four ranges per CTA of the launch); none for calls the weight-streaming kernel takes
// and none above 4096 rows, where the tiles of any projection of useful width already
// fill the SMs (the host never splits there)
size_t split_area_bytes(int64_t M) {
  if (M <= ee::kSkinnyAutoRows || M > 4096) return 0;
  return 256 + size_t(4) * size_t(num_sms()) * size_t(ee::kPartBlockBytes);
}

int check_ws(const void* ws, size_t have, size_t need) {
  if (ws == nullptr) return fail(EE_ERR_INVALID, "workspace is NULL");
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return fail(EE_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  if (have < need) return fail(EE_ERR_INVALID, "workspace too small: %zu < %zu bytes", have, need);
  return EE_OK;
}

// gw != nullptr: the rows go to the bucket order of a gated workspace (positions from
// its chunk table, perm / slot written); else every row keeps its index as position
int pack_rows(const void* A, int64_t lda, int64_t M, int64_t K, const int8_t* route, int fixed_bucket,
              const GatedWs* gw, float* sa, uint8_t* buf8, int64_t ld8, void* buf16, int64_t ld16, cudaStream_t s) {
  ee::PackArgs p;
  p.A = A;
  p.lda = lda;
  p.M = M;
  p.K = static_cast<int>(K);
  p.route = route;
  p.fixed_bucket = fixed_bucket;
  p.chunk_tab = gw ? gw->chunk_tab : nullptr;
  p.counts = gw ? gw->counts : nullptr;
  p.perm = gw ? gw->perm : nullptr;
  p.slot = gw ? gw->slot : nullptr;
  p.sa = sa;
  p.buf8 = buf8;
  p.ld8 = ld8;
  p.buf16 = buf16;
  p.ld16 = ld16;
  return check_launch(ee::launch_pack_rows(p, s), "pack_rows");
}

int check_rows_input(const void* A, int64_t M, int64_t K, int64_t lda) {
  if (A == nullptr && M != 0) return fail(EE_ERR_INVALID, "A is NULL");  // M == 0: an empty batch, no pointers needed
  if (M < 0 || K <= 0 || M > kMaxDim || K > kMaxDim) return fail(EE_ERR_INVALID, "bad shape M=%lld K=%lld", (long long)M, (long long)K);
  if (K % 8 != 0 || lda < K || lda % 8 != 0 || !al16(A))
    return fail(EE_ERR_MISALIGNED, "A needs K %% 8 == 0, lda %% 8 == 0 (lda >= K) and a 16-byte aligned base");
  return EE_OK;
}

}  // namespace

namespace ee {
void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }
}  // namespace ee

extern "C" {

int ee_abi_version(void) { return EE_ABI_VERSION; }

int ee_set_gemm_policy(int policy) {
  if (policy < 0 || policy > 4)
    return fail(EE_ERR_INVALID,
                "policy must be 0 (auto), 1 (single-CTA), 2 (CTA pair), 3 (single-CTA narrow) or 4 (weight-streaming)");
  g_gemm_policy.store(policy, std::memory_order_relaxed);
  return EE_OK;
}

int ee_set_gemm_splits(int splits) {
  if (splits < 0 || splits > ee::kSkinnyMaxSplits) return fail(EE_ERR_INVALID, "splits must be 0 (automatic) .. 8");
  g_gemm_splits.store(splits, std::memory_order_relaxed);
  return EE_OK;
}

int ee_debug_drop_next_gemm_load(int cta) {
  if (cta < 0 || cta >= num_sms()) return fail(EE_ERR_INVALID, "cta must be in [0, %d)", num_sms());
  g_drop_next_load.store(cta + 1, std::memory_order_relaxed);
  return EE_OK;
}

const char* ee_last_error(void) { return g_last_error.c_str(); }

int ee_device_check(int* value) {
  int v = 0;
  if (ee::read_and_clear_device_error(&v) != 0) return fail(EE_ERR_CUDA, "reading the device error word failed");
  if (value) *value = v;
  if (v != 0) return fail(EE_ERR_DEVICE, "device error word 0x%x (a bounded wait in a kernel gave up)", v);
  return EE_OK;
}

// ------------------------------------------------------------------ softmax + entropy
int ee_softmax_entropy(const void* x, int64_t rows, int64_t n, int64_t ld, int causal, int64_t S, void* probs,
                       int64_t ldp, float* H, int8_t* route, double tau_low, double tau_high, void* stream) {
  if (rows < 0 || rows > kMaxDim) return fail(EE_ERR_INVALID, "bad rows=%lld", (long long)rows);
  if (rows == 0) return EE_OK;
  if (x == nullptr || H == nullptr) return fail(EE_ERR_INVALID, "x and H are required");
  if (n <= 0 || n > kMaxDim || ld < n) return fail(EE_ERR_INVALID, "bad n=%lld / ld=%lld", (long long)n, (long long)ld);
  if (probs != nullptr && ldp < n) return fail(EE_ERR_INVALID, "ldp=%lld < n", (long long)ldp);
  if (causal && S <= 0) return fail(EE_ERR_INVALID, "causal masking needs S >= 1");
  if ((reinterpret_cast<uintptr_t>(x) & 1u) || (probs && (reinterpret_cast<uintptr_t>(probs) & 1u)) ||
      (reinterpret_cast<uintptr_t>(H) & 3u))
    return fail(EE_ERR_MISALIGNED, "x/probs must be 2-byte and H 4-byte aligned");
  ee::SoftmaxArgs a;
  std::memset(&a, 0, sizeof(a));
  a.x = x;
  a.ldx = ld;
  a.rows = rows;
  a.n = static_cast<int>(n);
  a.causal = causal ? 1 : 0;
  a.S = causal ? S : 1;
  a.probs = probs;
  a.ldp = ldp;
  a.H = H;
  a.route = route;
  a.tau_low = tau_low;
  a.tau_high = tau_high;
  return check_launch(ee::launch_softmax_entropy(a, as_stream(stream)), "softmax_entropy");
}

int ee_fused_softmax_entropy_4d(const void* logits, int64_t B, int64_t Hh, int64_t S, int causal, void* probs,
                                float* row_entropy, float* batch_entropy, void* stream) {
  if (B < 0 || Hh < 0 || S < 0) return fail(EE_ERR_INVALID, "negative shape");
  if (B == 0 || Hh == 0 || S == 0) return EE_OK;
  if (row_entropy == nullptr || batch_entropy == nullptr)
    return fail(EE_ERR_INVALID, "row_entropy and batch_entropy are required");
  const int64_t rows = B * Hh * S;
  int st = ee_softmax_entropy(logits, rows, S, S, causal, S, probs, S, row_entropy, nullptr, 0.f, 0.f, stream);
  if (st != EE_OK) return st;
  return check_launch(ee::launch_batch_mean(row_entropy, B, Hh * S, batch_entropy, as_stream(stream)), "batch_mean");
}

int ee_attention_entropy(const void* probs, int dtype, int64_t rows, int64_t n, int64_t ld, float* row_entropy,
                         int64_t batches, float* batch_entropy, void* stream) {
  if (rows < 0 || n < 0 || batches < 0) return fail(EE_ERR_INVALID, "negative shape");
  if (dtype != EE_DTYPE_F16 && dtype != EE_DTYPE_F32) return fail(EE_ERR_INVALID, "dtype must be EE_DTYPE_F16 or EE_DTYPE_F32");
  if (rows == 0) return EE_OK;
  if (probs == nullptr || row_entropy == nullptr) return fail(EE_ERR_INVALID, "probs and row_entropy are required");
  if (n == 0 || ld < n) return fail(EE_ERR_INVALID, "bad n=%lld / ld=%lld", (long long)n, (long long)ld);
  const size_t esize = dtype == EE_DTYPE_F32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(probs) % esize != 0) return fail(EE_ERR_MISALIGNED, "probs misaligned for its dtype");
  if (batch_entropy != nullptr && (batches <= 0 || rows % batches != 0))
    return fail(EE_ERR_INVALID, "rows=%lld is not a multiple of batches=%lld", (long long)rows, (long long)batches);
  cudaStream_t s = as_stream(stream);
  int st = check_launch(ee::launch_attention_entropy(probs, dtype == EE_DTYPE_F32, rows, n, ld, row_entropy, s),
                        "attention_entropy");
  if (st != EE_OK || batch_entropy == nullptr) return st;
  return check_launch(ee::launch_batch_mean(row_entropy, batches, rows / batches, batch_entropy, s), "batch_mean");
}

size_t ee_attention_workspace_bytes(int64_t B, int64_t Hkv, int64_t S, int64_t head_dim) {
  if (B < 0 || Hkv < 0 || S < 0 || head_dim < 0) return 0;
  const int64_t s_pad = (S + 63) / 64 * 64;
  return align256(sizeof(uint16_t) * size_t(B) * Hkv * head_dim * s_pad);
}

int ee_flash_attention_entropy(const void* Q, const void* K, const void* V, int64_t B, int64_t Hq, int64_t Hkv,
                               int64_t S, int64_t head_dim, int causal, float scale, void* O, float* H,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (B < 0 || Hq <= 0 || Hkv <= 0 || S < 0) return fail(EE_ERR_INVALID, "bad shape");
  if (Hq % Hkv != 0) return fail(EE_ERR_INVALID, "Hq=%lld is not a multiple of Hkv=%lld", (long long)Hq, (long long)Hkv);
  if (head_dim != 64 && head_dim != 128) return fail(EE_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (causal != 0 && causal != 1) return fail(EE_ERR_INVALID, "causal must be 0 or 1");
  if (B == 0 || S == 0) return EE_OK;
  if (B * Hq * S >= (int64_t(1) << 31) || B * Hkv * head_dim >= (int64_t(1) << 31))
    return fail(EE_ERR_UNSUPPORTED, "more than 2^31 rows");
  if (!Q || !K || !V || !O || !H) return fail(EE_ERR_INVALID, "Q, K, V, O and H are required");
  if (!al16(Q) || !al16(K) || !al16(V) || !al16(O) || (reinterpret_cast<uintptr_t>(H) & 3u))
    return fail(EE_ERR_MISALIGNED, "Q, K, V and O must be 16-byte aligned, H 4-byte aligned");
  int st = check_ws(workspace, workspace_bytes, ee_attention_workspace_bytes(B, Hkv, S, head_dim));
  if (st != EE_OK) return st;
  cudaStream_t s = as_stream(stream);
  const int64_t s_pad = (S + 63) / 64 * 64;
  if ((st = check_launch(ee::launch_transpose_v(V, B, Hkv, S, s_pad, head_dim, Hkv * S * head_dim, S * head_dim,
                                                head_dim, workspace, s),
                         "transpose_v")) != EE_OK)
    return st;
  ee::AttnLaunch a;
  std::memset(&a, 0, sizeof(a));
  if ((st = encode_kmajor(&a.q, Q, B * Hq * S, head_dim, head_dim, 2, ee::kAttnTile)) != EE_OK) return st;
  // K tiles of 128 keys for head_dim 64, 64 keys for 128 (the kernel's KT)
  if ((st = encode_kmajor(&a.k, K, B * Hkv * S, head_dim, head_dim, 2, 128)) != EE_OK) return st;
  if ((st = encode_kmajor(&a.vt, workspace, B * Hkv * head_dim, s_pad, s_pad, 2, static_cast<int>(head_dim))) != EE_OK)
    return st;
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.S = S;
  a.S_pad = s_pad;
  a.D = head_dim;
  a.scale = scale;
  a.causal = causal;
  a.O = O;
  a.H = H;
  return check_launch(ee::launch_flash_attention(a, s), "flash_attention_entropy");
}

size_t ee_attention_rope_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t head_dim) {
  if (B < 0 || Hq < 0 || Hkv < 0 || S < 0 || head_dim < 0) return 0;
  return align256(sizeof(uint16_t) * size_t(B) * Hq * S * head_dim) +
         align256(sizeof(uint16_t) * size_t(B) * Hkv * S * head_dim) + ee_attention_workspace_bytes(B, Hkv, S, head_dim);
}

}  // extern "C"

namespace {
// the rotary flash attention of ee_flash_attention_rope_entropy; exact: the row
// entropies come from a second pass over the keys with the reference's fp16 rounding of
// each probability (the workspace then also holds each row's (m, l) of the first pass)
int rope_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                   const void* cos, const void* sin, int64_t ld_cs, int64_t B, int64_t Hq, int64_t Hkv, int64_t S,
                   int64_t head_dim, int causal, float scale, void* O, float* H, void* workspace,
                   size_t workspace_bytes, void* stream, bool exact) {
  if (B < 0 || Hq <= 0 || Hkv <= 0 || S < 0) return fail(EE_ERR_INVALID, "bad shape");
  if (Hq % Hkv != 0) return fail(EE_ERR_INVALID, "Hq=%lld is not a multiple of Hkv=%lld", (long long)Hq, (long long)Hkv);
  if (head_dim != 64 && head_dim != 128) return fail(EE_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (causal != 0 && causal != 1) return fail(EE_ERR_INVALID, "causal must be 0 or 1");
  if (B == 0 || S == 0) return EE_OK;
  if (B * Hq * S >= (int64_t(1) << 31) || B * Hkv * head_dim >= (int64_t(1) << 31))
    return fail(EE_ERR_UNSUPPORTED, "more than 2^31 rows");
  if (!q || !k || !v || !cos || !sin || !O || !H) return fail(EE_ERR_INVALID, "q, k, v, cos, sin, O and H are required");
  if (ldq < Hq * head_dim || ldk < Hkv * head_dim || ldv < Hkv * head_dim || ld_cs < head_dim)
    return fail(EE_ERR_INVALID, "row strides below the rows");
  if (!al16(q) || !al16(k) || !al16(v) || !al16(cos) || !al16(sin) || !al16(O) || (reinterpret_cast<uintptr_t>(H) & 3u) ||
      ldq % 8 || ldk % 8 || ldv % 8 || ld_cs % 8)
    return fail(EE_ERR_MISALIGNED, "q, k, v, cos, sin and O must be 16-byte aligned with row strides of 8 elements");
  const size_t rope_bytes = ee_attention_rope_workspace_bytes(B, Hq, Hkv, S, head_dim);
  int st = check_ws(workspace, workspace_bytes,
                    exact ? ee_attention_exact_workspace_bytes(B, Hq, Hkv, S, head_dim) : rope_bytes);
  if (st != EE_OK) return st;
  cudaStream_t s = as_stream(stream);
  uint8_t* p = static_cast<uint8_t*>(workspace);
  void* ml = exact ? p + rope_bytes : nullptr;
  __half* qr = reinterpret_cast<__half*>(p);
  p += align256(sizeof(uint16_t) * size_t(B) * Hq * S * head_dim);
  __half* kr = reinterpret_cast<__half*>(p);
  p += align256(sizeof(uint16_t) * size_t(B) * Hkv * S * head_dim);
  void* vt = p;
  ee::RopeArgs r;
  r.q = static_cast<const __half*>(q);
  r.ldq = ldq;
  r.k = static_cast<const __half*>(k);
  r.ldk = ldk;
  r.cos = static_cast<const __half*>(cos);
  r.sin = static_cast<const __half*>(sin);
  r.ld_cs = ld_cs;
  r.B = B;
  r.S = S;
  r.Hq = static_cast<int>(Hq);
  r.Hkv = static_cast<int>(Hkv);
  r.q_out = qr;
  r.k_out = kr;
  if ((st = check_launch(ee::launch_rope_layout(r, static_cast<int>(head_dim), s), "rope_layout")) != EE_OK) return st;
  const int64_t s_pad = (S + 63) / 64 * 64;
  if ((st = check_launch(ee::launch_transpose_v(v, B, Hkv, S, s_pad, head_dim, S * ldv, head_dim, ldv, vt, s),
                         "transpose_v")) != EE_OK)
    return st;
  ee::AttnLaunch a;
  std::memset(&a, 0, sizeof(a));
  if ((st = encode_kmajor(&a.q, qr, B * Hq * S, head_dim, head_dim, 2, ee::kAttnTile)) != EE_OK) return st;
  if ((st = encode_kmajor(&a.k, kr, B * Hkv * S, head_dim, head_dim, 2, 128)) != EE_OK)
    return st;
  if ((st = encode_kmajor(&a.vt, vt, B * Hkv * head_dim, s_pad, s_pad, 2, static_cast<int>(head_dim))) != EE_OK)
    return st;
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.S = S;
  a.S_pad = s_pad;
  a.D = head_dim;
  a.scale = scale;
  a.causal = causal;
  a.O = O;
  a.H = H;
  a.ml = ml;
  if ((st = check_launch(ee::launch_flash_attention(a, s), "flash_attention_entropy")) != EE_OK || !exact) return st;
  return check_launch(ee::launch_attention_entropy_exact(a, s), "attention_entropy_exact");
}
}  // namespace

extern "C" {

int ee_flash_attention_rope_entropy(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                                    const void* cos, const void* sin, int64_t ld_cs, int64_t B, int64_t Hq, int64_t Hkv,
                                    int64_t S, int64_t head_dim, int causal, float scale, void* O, float* H,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  return rope_attention(q, ldq, k, ldk, v, ldv, cos, sin, ld_cs, B, Hq, Hkv, S, head_dim, causal, scale, O, H,
                        workspace, workspace_bytes, stream, false);
}

size_t ee_attention_exact_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t head_dim) {
  if (B < 0 || Hq < 0 || Hkv < 0 || S < 0 || head_dim < 0) return 0;
  return ee_attention_rope_workspace_bytes(B, Hq, Hkv, S, head_dim) + align256(sizeof(float) * 2 * size_t(B) * Hq * S);
}

int ee_flash_attention_rope_entropy_exact(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                          int64_t ldv, const void* cos, const void* sin, int64_t ld_cs, int64_t B,
                                          int64_t Hq, int64_t Hkv, int64_t S, int64_t head_dim, int causal,
                                          float scale, void* O, float* H, void* workspace, size_t workspace_bytes,
                                          void* stream) {
  return rope_attention(q, ldq, k, ldk, v, ldv, cos, sin, ld_cs, B, Hq, Hkv, S, head_dim, causal, scale, O, H,
                        workspace, workspace_bytes, stream, true);
}

// ------------------------------------------------------------------ entropy-tied KV cache
}  // extern "C"
namespace {
struct KvLayout {
  size_t k8, v8, k16, v16, ks, vs, slot, length, pool, total;
};
KvLayout kv_layout(int64_t batch, int64_t kv_heads, int64_t head_dim, int64_t max_tokens, int64_t slots8,
                   int64_t slots16) {
  KvLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align256(bytes);
    return at;
  };
  const size_t row = size_t(kv_heads) * head_dim;
  L.k8 = take(size_t(slots8) * row);
  L.v8 = take(size_t(slots8) * row);
  L.k16 = take(2 * size_t(slots16) * row);
  L.v16 = take(2 * size_t(slots16) * row);
  L.ks = take(4 * size_t(slots8) * kv_heads);
  L.vs = take(4 * size_t(slots8) * kv_heads);
  L.slot = take(4 * size_t(batch) * max_tokens);
  L.length = take(4 * size_t(batch));
  L.pool = take(8);
  L.total = off;
  return L;
}
bool kv_shape_ok(int64_t batch, int64_t kv_heads, int64_t head_dim, int64_t max_tokens, int64_t slots8,
                 int64_t slots16) {
  return batch > 0 && kv_heads > 0 && (head_dim == 64 || head_dim == 128) && max_tokens > 0 && slots8 >= 0 &&
         slots16 >= 0 && slots8 < (int64_t(1) << 28) && slots16 < (int64_t(1) << 28) &&
         batch * max_tokens < (int64_t(1) << 31) && max_tokens < (int64_t(1) << 30);
}
ee::KvCacheArgs kv_args(const ee_kv_cache& c) {
  ee::KvCacheArgs a;
  a.batch = c.batch;
  a.kv_heads = c.kv_heads;
  a.head_dim = c.head_dim;
  a.max_tokens = c.max_tokens;
  a.slots8 = c.slots8;
  a.slots16 = c.slots16;
  a.k8 = c.k8;
  a.v8 = c.v8;
  a.k16 = c.k16;
  a.v16 = c.v16;
  a.k_scale = c.k_scale;
  a.v_scale = c.v_scale;
  a.slot = c.slot;
  a.length = c.length;
  a.pool_used = c.pool_used;
  return a;
}
// token splits of the decode attention: about 256 cached tokens per CTA (four warps of
// 64), so that enough warps are in flight to hide the slot-table and row loads, and at
// least two CTAs per SM over the batch's KV heads
int kv_splits(int64_t batch, int64_t kv_heads, int64_t max_tokens) {
  const int64_t ctas = batch * kv_heads;
  // about 1024 tokens per CTA (32 ring stages: the copy pipeline's fill and drain amortised;
  // measured on B200 at 16 x 8192 tokens: 256 tokens 246 us, 512 209, 1024 172, 2048 205)
  int64_t s = (max_tokens + 1 + 1023) / 1024;
  const int64_t fill = (2 * int64_t(num_sms()) + ctas - 1) / ctas;
  s = s > fill ? s : fill;
  return static_cast<int>(s < 1 ? 1 : (s > 1024 ? 1024 : s));
}
}  // namespace
extern "C" {

size_t ee_kv_cache_bytes(int64_t batch, int64_t kv_heads, int64_t head_dim, int64_t max_tokens, int64_t slots8,
                         int64_t slots16) {
  if (!kv_shape_ok(batch, kv_heads, head_dim, max_tokens, slots8, slots16)) return 0;
  return kv_layout(batch, kv_heads, head_dim, max_tokens, slots8, slots16).total;
}

int ee_kv_cache_init(ee_kv_cache* cache, void* memory, size_t bytes, int64_t batch, int64_t kv_heads,
                     int64_t head_dim, int64_t max_tokens, int64_t slots8, int64_t slots16, void* stream) {
  if (cache == nullptr) return fail(EE_ERR_INVALID, "cache is NULL");
  if (!kv_shape_ok(batch, kv_heads, head_dim, max_tokens, slots8, slots16))
    return fail(EE_ERR_INVALID, "bad KV-cache shape (head_dim 64 / 128, positive sizes, pools < 2^28 slots)");
  const KvLayout L = kv_layout(batch, kv_heads, head_dim, max_tokens, slots8, slots16);
  int st = check_ws(memory, bytes, L.total);
  if (st != EE_OK) return st;
  uint8_t* p = static_cast<uint8_t*>(memory);
  cache->batch = batch;
  cache->kv_heads = kv_heads;
  cache->head_dim = head_dim;
  cache->max_tokens = max_tokens;
  cache->slots8 = slots8;
  cache->slots16 = slots16;
  cache->k8 = p + L.k8;
  cache->v8 = p + L.v8;
  cache->k16 = p + L.k16;
  cache->v16 = p + L.v16;
  cache->k_scale = reinterpret_cast<float*>(p + L.ks);
  cache->v_scale = reinterpret_cast<float*>(p + L.vs);
  cache->slot = reinterpret_cast<int32_t*>(p + L.slot);
  cache->length = reinterpret_cast<int32_t*>(p + L.length);
  cache->pool_used = reinterpret_cast<uint32_t*>(p + L.pool);
  cudaError_t e = cudaMemsetAsync(p + L.length, 0, L.total - L.length, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
  return EE_OK;
}

int ee_kv_append(const ee_kv_cache* cache, const void* k_rows, int64_t ldk, const void* v_rows, int64_t ldv,
                 const int8_t* tier, int64_t t_new, void* stream) {
  if (cache == nullptr || cache->length == nullptr) return fail(EE_ERR_INVALID, "cache is not initialised");
  if (t_new < 0) return fail(EE_ERR_INVALID, "t_new must be >= 0");
  if (t_new == 0) return EE_OK;
  if (!k_rows || !v_rows || !tier) return fail(EE_ERR_INVALID, "k_rows, v_rows and tier are required");
  const int64_t row = cache->kv_heads * cache->head_dim;
  if (ldk < row || ldv < row || ldk % 8 || ldv % 8 || !al16(k_rows) || !al16(v_rows))
    return fail(EE_ERR_MISALIGNED, "K / V rows must be 16-byte aligned with strides >= kv_heads * head_dim, % 8");
  if (cache->batch * t_new >= (int64_t(1) << 31)) return fail(EE_ERR_UNSUPPORTED, "too many tokens in one append");
  return check_launch(ee::launch_kv_append(kv_args(*cache), k_rows, ldk, v_rows, ldv, tier, t_new, as_stream(stream)),
                      "kv_append");
}

size_t ee_kv_decode_workspace_bytes(const ee_kv_cache* cache, int64_t heads) {
  if (cache == nullptr || cache->batch <= 0 || cache->kv_heads <= 0 || heads <= 0 || cache->head_dim <= 0) return 0;
  return align256(sizeof(float) * size_t(cache->batch) * heads *
                  kv_splits(cache->batch, cache->kv_heads, cache->max_tokens) * (3 + cache->head_dim));
}

int ee_kv_decode_attention(const ee_kv_cache* cache, const void* q, int64_t ldq, int64_t heads, const void* k_new,
                           const void* v_new, int64_t ld_new, float scale, void* out, int64_t ldo, float* H,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (cache == nullptr || cache->length == nullptr) return fail(EE_ERR_INVALID, "cache is not initialised");
  const int64_t G = heads / (cache->kv_heads > 0 ? cache->kv_heads : 1);
  if (heads <= 0 || heads % cache->kv_heads || (G != 1 && G != 2 && G != 4 && G != 8))
    return fail(EE_ERR_UNSUPPORTED, "heads must be 1, 2, 4 or 8 times kv_heads");
  if (!q || !k_new || !v_new || !out) return fail(EE_ERR_INVALID, "q, k_new, v_new and out are required");
  const int64_t d = cache->head_dim;
  if (ldq < heads * d || ldo < heads * d || ld_new < cache->kv_heads * d || ldq % 8 || ldo % 8 || ld_new % 8 ||
      !al16(q) || !al16(k_new) || !al16(v_new) || !al16(out) || (reinterpret_cast<uintptr_t>(H) & 3u))
    return fail(EE_ERR_MISALIGNED, "q / k_new / v_new / out rows 16-byte aligned with strides % 8, H 4-byte aligned");
  // the decode kernel gathers whole K / V rows with bulk copies: 16-byte aligned pools
  if (!al16(cache->k8) || !al16(cache->v8) || !al16(cache->k16) || !al16(cache->v16))
    return fail(EE_ERR_MISALIGNED, "the cache's K / V pools must be 16-byte aligned");
  int st = check_ws(workspace, workspace_bytes, ee_kv_decode_workspace_bytes(cache, heads));
  if (st != EE_OK) return st;
  return check_launch(ee::launch_kv_decode_attention(kv_args(*cache), q, ldq, heads, k_new, v_new, ld_new, scale,
                                                     kv_splits(cache->batch, cache->kv_heads, cache->max_tokens),
                                                     static_cast<float*>(workspace), out, ldo, H, as_stream(stream)),
                      "kv_decode_attention");
}

int ee_head_mean_entropy(const float* H, int64_t B, int64_t Hq, int64_t S, float* token_entropy,
                         float* batch_entropy, void* stream) {
  if (B < 0 || Hq <= 0 || S < 0 || B * Hq * S >= (int64_t(1) << 40)) return fail(EE_ERR_INVALID, "bad shape");
  if (B == 0 || S == 0) return EE_OK;
  if (H == nullptr || token_entropy == nullptr) return fail(EE_ERR_INVALID, "H and token_entropy are required");
  if ((reinterpret_cast<uintptr_t>(H) | reinterpret_cast<uintptr_t>(token_entropy) |
       reinterpret_cast<uintptr_t>(batch_entropy)) & 3u)
    return fail(EE_ERR_MISALIGNED, "H and the outputs must be 4-byte aligned");
  cudaStream_t s = as_stream(stream);
  int st = check_launch(ee::launch_head_mean(H, B, Hq, S, token_entropy, s), "head_mean");
  if (st != EE_OK || batch_entropy == nullptr) return st;
  return check_launch(ee::launch_batch_mean(H, B, Hq * S, batch_entropy, s), "batch_mean");
}

// ------------------------------------------------------------------ the block's norms
int ee_add_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr, void* sum_out, int64_t lds,
                   const void* weight, float eps, void* y, int64_t ldy, int64_t M, int64_t d, void* stream) {
  if (M < 0 || d <= 0 || d > 8192 || d % 8) return fail(EE_ERR_UNSUPPORTED, "d=%lld: 8 .. 8192, a multiple of 8", (long long)d);
  if (M == 0) return EE_OK;
  if (!x || !weight || !y) return fail(EE_ERR_INVALID, "x, weight and y are required");
  if (sum_out && !residual) return fail(EE_ERR_INVALID, "sum_out needs residual");
  if (ldx < d || ldy < d || (residual && ldr < d) || (sum_out && lds < d)) return fail(EE_ERR_INVALID, "row strides below d");
  if (!al16(x) || !al16(weight) || !al16(y) || (residual && !al16(residual)) || (sum_out && !al16(sum_out)) ||
      ldx % 8 || ldy % 8 || (residual && ldr % 8) || (sum_out && lds % 8))
    return fail(EE_ERR_MISALIGNED, "16-byte aligned rows with strides of 8 elements required");
  ee::AddNormArgs a;
  a.x = static_cast<const __half*>(x);
  a.ldx = ldx;
  a.res = static_cast<const __half*>(residual);
  a.ldr = ldr;
  a.sum_out = static_cast<__half*>(sum_out);
  a.lds = lds;
  a.w = static_cast<const __half*>(weight);
  a.y = static_cast<__half*>(y);
  a.ldy = ldy;
  a.M = M;
  a.d = static_cast<int>(d);
  a.eps = eps;
  return check_launch(ee::launch_add_rmsnorm(a, as_stream(stream)), "add_rmsnorm");
}

// ------------------------------------------------------------------ routing
int ee_route(const float* H, int64_t rows, double tau_low, double tau_high, int8_t* route, void* stream) {
  if (rows < 0) return fail(EE_ERR_INVALID, "rows < 0");
  if (rows == 0) return EE_OK;
  if (H == nullptr || route == nullptr) return fail(EE_ERR_INVALID, "H and route are required");
  return check_launch(ee::launch_route(H, rows, tau_low, tau_high, route, as_stream(stream)), "route");
}

int ee_route_batch_max(const float* H, int64_t n, double tau_low, double tau_high, float* max_out, int8_t* tier_out,
                       void* stream) {
  if (H == nullptr || n <= 0) return fail(EE_ERR_INVALID, "H is required and n must be >= 1");
  return check_launch(ee::launch_batch_max_route(H, n, tau_low, tau_high, max_out, tier_out, as_stream(stream)),
                      "batch_max_route");
}

// ------------------------------------------------------------------ weights
int ee_quantize_weights_int8(const void* W, int64_t N, int64_t K, int64_t ldw, int8_t* w_kn, int8_t* w_nk,
                             float* scale, int div_mode, void* stream) {
  if (W == nullptr || scale == nullptr) return fail(EE_ERR_INVALID, "W and scale are required");
  if (N <= 0 || K <= 0 || ldw < K || N > kMaxDim || K > kMaxDim) return fail(EE_ERR_INVALID, "bad shape");
  if (div_mode != 0 && div_mode != 1) return fail(EE_ERR_INVALID, "div_mode must be 0 or 1");
  return check_launch(ee::launch_quantize_weights(W, ldw, N, K, w_kn, w_nk, scale, div_mode, as_stream(stream)),
                      "quantize_weights");
}

int ee_pack_weights(const int8_t* w_kn, const float* scale, int64_t K, int64_t N, int8_t* w_i8_nk,
                    uint8_t* w_e4m3_nk, void* w_f16_nk, void* stream) {
  if (w_kn == nullptr) return fail(EE_ERR_INVALID, "w_kn is required");
  if (w_f16_nk != nullptr && scale == nullptr) return fail(EE_ERR_INVALID, "the fp16 pack needs the scale");
  if (K <= 0 || N <= 0 || K > kMaxDim || N > kMaxDim) return fail(EE_ERR_INVALID, "bad shape");
  return check_launch(ee::launch_pack_weights(w_kn, scale, K, N, w_i8_nk, w_e4m3_nk, w_f16_nk, as_stream(stream)),
                      "pack_weights");
}

// ------------------------------------------------------------------ activations
int ee_quant_rows_int8(const void* A, int64_t M, int64_t K, int64_t lda, int8_t* q, float* scale, void* stream) {
  int st = check_rows_input(A, M, K, lda);
  if (st != EE_OK) return st;
  if (M == 0) return EE_OK;
  if (q == nullptr || scale == nullptr || !al16(q)) return fail(EE_ERR_INVALID, "q (16-byte aligned) and scale are required");
  return pack_rows(A, lda, M, K, nullptr, ee::kINT8, nullptr, scale, reinterpret_cast<uint8_t*>(q), K, nullptr, 0,
                   as_stream(stream));
}

int ee_quant_rows_e4m3(const void* A, int64_t M, int64_t K, int64_t lda, uint8_t* q, float* scale, void* stream) {
  int st = check_rows_input(A, M, K, lda);
  if (st != EE_OK) return st;
  if (M == 0) return EE_OK;
  if (q == nullptr || scale == nullptr || !al16(q)) return fail(EE_ERR_INVALID, "q (16-byte aligned) and scale are required");
  return pack_rows(A, lda, M, K, nullptr, ee::kFP8, nullptr, scale, q, K, nullptr, 0, as_stream(stream));
}

// ------------------------------------------------------------------ GEMMs
static int gemm_single(int bucket, const void* A, const float* a_scale, const void* W, const float* w_scale, void* Y,
                       int64_t M, int64_t N, int64_t K, int64_t ldy, int out_mode, void* stream) {
  int st = check_gemm_shape(M, N, K, ldy);
  if (st != EE_OK) return st;
  if (M == 0) return EE_OK;
  if (A == nullptr || W == nullptr || Y == nullptr) return fail(EE_ERR_INVALID, "A, W and Y are required");
  if (!al16(A) || !al16(W) || !al16(Y)) return fail(EE_ERR_MISALIGNED, "A, W and Y must be 16-byte aligned");
  if (bucket != ee::kFP16 && out_mode == 0) {
    if (a_scale == nullptr || w_scale == nullptr) return fail(EE_ERR_INVALID, "scales are required");
    if (!al16(w_scale)) return fail(EE_ERR_MISALIGNED, "w_scale must be 16-byte aligned");
  }
  GemmOperands op;
  if (bucket == ee::kFP16) {
    op.a16 = A;
    op.ld16 = K;
  } else {
    op.a8 = A;
    op.ld8 = K;
  }
  op.w[bucket] = W;
  ee::GemmArgs args = base_args(M, N, K, Y, ldy, out_mode);
  args.counts[bucket] = static_cast<int>(M);
  args.sa = a_scale;
  args.sb = w_scale;
  return run_gemm(op, args, false, as_stream(stream));
}

int ee_gemm_int8(const int8_t* A, const float* a_scale, const int8_t* W_nk, const float* w_scale, void* Y,
                 int64_t M, int64_t N, int64_t K, int64_t ldy, void* stream) {
  return gemm_single(ee::kINT8, A, a_scale, W_nk, w_scale, Y, M, N, K, ldy, 0, stream);
}
int ee_gemm_fp8(const uint8_t* A, const float* a_scale, const uint8_t* W_nk, const float* w_scale, void* Y,
                int64_t M, int64_t N, int64_t K, int64_t ldy, void* stream) {
  return gemm_single(ee::kFP8, A, a_scale, W_nk, w_scale, Y, M, N, K, ldy, 0, stream);
}
int ee_gemm_fp16(const void* A, const void* W_nk, void* Y, int64_t M, int64_t N, int64_t K, int64_t ldy,
                 void* stream) {
  return gemm_single(ee::kFP16, A, nullptr, W_nk, nullptr, Y, M, N, K, ldy, 0, stream);
}
int ee_gemm_int8_acc(const int8_t* A, const int8_t* W_nk, int32_t* acc, int64_t M, int64_t N, int64_t K,
                     void* stream) {
  return gemm_single(ee::kINT8, A, nullptr, W_nk, nullptr, acc, M, N, K, N, 1, stream);
}
int ee_gemm_fp8_acc(const uint8_t* A, const uint8_t* W_nk, float* acc, int64_t M, int64_t N, int64_t K,
                    void* stream) {
  return gemm_single(ee::kFP8, A, nullptr, W_nk, nullptr, acc, M, N, K, N, 1, stream);
}
int ee_gemm_fp16_acc(const void* A, const void* W_nk, float* acc, int64_t M, int64_t N, int64_t K, void* stream) {
  return gemm_single(ee::kFP16, A, nullptr, W_nk, nullptr, acc, M, N, K, N, 1, stream);
}

size_t ee_linear_workspace_bytes(int64_t M, int64_t K) {
  if (M < 0 || K < 0) return 0;
  return linear_ws_bytes(M, K);
}

static int linear_8bit(int bucket, const void* A, int64_t lda, const void* W, const float* w_scale, void* Y,
                       int64_t M, int64_t N, int64_t K, int64_t ldy, void* ws, size_t ws_bytes, void* stream) {
  int st = check_gemm_shape(M, N, K, ldy);
  if (st != EE_OK) return st;
  if ((st = check_rows_input(A, M, K, lda)) != EE_OK) return st;
  if (M == 0) return EE_OK;
  if ((st = check_ws(ws, ws_bytes, linear_ws_bytes(M, K))) != EE_OK) return st;
  if (W == nullptr || w_scale == nullptr || Y == nullptr) return fail(EE_ERR_INVALID, "W, w_scale and Y are required");
  if (!al16(W) || !al16(Y) || !al16(w_scale)) return fail(EE_ERR_MISALIGNED, "W, w_scale and Y must be 16-byte aligned");
  LinearWs w = linear_ws(ws, M);
  if ((st = pack_rows(A, lda, M, K, nullptr, bucket, nullptr, w.sa, w.q, K, nullptr, 0, as_stream(stream))) != EE_OK)
    return st;
  return gemm_single(bucket, w.q, w.sa, W, w_scale, Y, M, N, K, ldy, 0, stream);
}

int ee_linear_int8(const void* A, int64_t lda, const int8_t* W_nk, const float* w_scale, void* Y, int64_t M,
                   int64_t N, int64_t K, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  return linear_8bit(ee::kINT8, A, lda, W_nk, w_scale, Y, M, N, K, ldy, workspace, workspace_bytes, stream);
}
int ee_linear_fp8(const void* A, int64_t lda, const uint8_t* W_e4m3_nk, const float* w_scale, void* Y, int64_t M,
                  int64_t N, int64_t K, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  return linear_8bit(ee::kFP8, A, lda, W_e4m3_nk, w_scale, Y, M, N, K, ldy, workspace, workspace_bytes, stream);
}

}  // extern "C"

// ------------------------------------------------------------------ allocation-free INT8 linear
// Scratch of ee_linear_int8_noalloc: a fixed block of device memory that lives in this
// library's own module, so the entry point never asks for memory at call time.  It
// holds the per-row activation scales (first 64 KiB, up to 16384 rows) followed by
// the quantised int8 activations (up to 16 MiB, i.e. M * K <= 2^24).  Every device
// that loads the library keeps this 16 MiB + 64 KiB block until the process exits.
static constexpr int64_t kNoAllocMaxRows = 16384;
static constexpr int64_t kNoAllocMaxQuantBytes = int64_t(1) << 24;
static constexpr size_t kNoAllocScaleBytes = size_t(kNoAllocMaxRows) * sizeof(float);
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScaleBytes + kNoAllocMaxQuantBytes];

namespace {
// Device address of g_noalloc_scratch, looked up once per device context.  In host code
// the symbol g_noalloc_scratch is only a host-side handle: its device address has to
// come from cudaGetSymbolAddress with that device current.  The lookup is keyed on the
// current context's unique id, so after cudaDeviceReset (which unloads the module and
// with it the array) the next call looks the new array up instead of writing through
// the old address.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

struct NoAllocSlot {
  std::mutex mu;
  std::atomic<unsigned long long> ctx_id{0};  // 0: not looked up yet (context ids start at 1)
  std::atomic<void*> ptr{nullptr};
};
NoAllocSlot g_noalloc_slots[64];

int current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (get_current == nullptr || get_id == nullptr) return fail(EE_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId unavailable");
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, id) != CUDA_SUCCESS)
    return fail(EE_ERR_CUDA, "no current CUDA context");
  return EE_OK;
}

int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(EE_ERR_UNSUPPORTED, "device ordinal %d >= 64", dev);
  e = cudaSetDevice(dev);  // initialises the device's primary context if nothing has yet
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  unsigned long long id = 0;
  int st = current_context_id(&id);
  if (st != EE_OK) return st;
  NoAllocSlot& slot = g_noalloc_slots[dev];
  if (slot.ctx_id.load(std::memory_order_acquire) != id) {
    std::lock_guard<std::mutex> lock(slot.mu);
    if (slot.ctx_id.load(std::memory_order_relaxed) != id) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
      slot.ptr.store(p, std::memory_order_relaxed);
      slot.ctx_id.store(id, std::memory_order_release);
    }
  }
  *out = slot.ptr.load(std::memory_order_relaxed);
  return EE_OK;
}
}  // namespace

extern "C" {

int ee_linear_int8_noalloc(const void* A, int64_t lda, const int8_t* W_nk, const float* w_scale, void* Y, int64_t M,
                           int64_t N, int64_t K, int64_t ldy, void* stream) {
  int st = check_gemm_shape(M, N, K, ldy);
  if (st != EE_OK) return st;
  if ((st = check_rows_input(A, M, K, lda)) != EE_OK) return st;
  if (M > kNoAllocMaxRows || M * K > kNoAllocMaxQuantBytes)
    return fail(EE_ERR_UNSUPPORTED,
                "ee_linear_int8_noalloc: M=%lld, K=%lld exceeds its fixed scratch (M <= %lld rows and "
                "M*K <= %lld bytes); use ee_linear_int8 with a caller-owned workspace",
                (long long)M, (long long)K, (long long)kNoAllocMaxRows, (long long)kNoAllocMaxQuantBytes);
  if (M == 0) return EE_OK;
  if (W_nk == nullptr || w_scale == nullptr || Y == nullptr) return fail(EE_ERR_INVALID, "W, w_scale and Y are required");
  if (!al16(W_nk) || !al16(Y) || !al16(w_scale)) return fail(EE_ERR_MISALIGNED, "W, w_scale and Y must be 16-byte aligned");
  void* scratch = nullptr;
  if ((st = noalloc_scratch(&scratch)) != EE_OK) return st;
  // Both regions are fully rewritten for rows [0, M) before the GEMM reads them, and
  // the GEMM's tensor map ends at row M, so nothing has to start at zero.
  float* sa = static_cast<float*>(scratch);
  uint8_t* q = static_cast<uint8_t*>(scratch) + kNoAllocScaleBytes;
  if ((st = pack_rows(A, lda, M, K, nullptr, ee::kINT8, nullptr, sa, q, K, nullptr, 0, as_stream(stream))) != EE_OK)
    return st;
  return gemm_single(ee::kINT8, q, sa, W_nk, w_scale, Y, M, N, K, ldy, 0, stream);
}

// ------------------------------------------------------------------ entropy-gated linear
size_t ee_gated_workspace_bytes(int64_t M, int64_t K) {
  if (M < 0 || K < 0) return 0;
  return gated_ws_bytes(M, K);
}

size_t ee_gated_workspace_split_bytes(int64_t M, int64_t K) {
  if (M < 0 || K < 0) return 0;
  return gated_ws_bytes(M, K) + split_area_bytes(M);
}

int ee_gate_rows(const void* logits, int64_t M, int64_t n, int64_t ld, double tau_low, double tau_high, float* H,
                 int8_t* route, int32_t* bucket_counts, void* workspace, size_t workspace_bytes, void* stream) {
  return ee::gate_rows_impl(logits, M, n, ld, tau_low, tau_high, H, route, bucket_counts, workspace, workspace_bytes,
                            stream, true);
}

int ee_gate_rows_keep(const void* logits, int64_t M, int64_t n, int64_t ld, double tau_low, double tau_high, float* H,
                      int8_t* route, int32_t* bucket_counts, void* workspace, size_t workspace_bytes, void* stream) {
  return ee::gate_rows_impl(logits, M, n, ld, tau_low, tau_high, H, route, bucket_counts, workspace, workspace_bytes,
                            stream, false);
}

size_t ee_gated_workspace_head_bytes(void) { return kWsHeadBytes; }
}  // extern "C"

// ee_gate_rows; clear_header = false skips zeroing the workspace header (ticket, counts,
// GEMM tile counter) for callers that zeroed it once: every kernel of the path leaves it
// zero again after a clean run, and without the memset node the router launch chains
// onto the previous kernel (programmatic dependent launch).
int ee::gate_rows_impl(const void* logits, int64_t M, int64_t n, int64_t ld, double tau_low, double tau_high,
                       float* H, int8_t* route, int32_t* bucket_counts, void* workspace, size_t workspace_bytes,
                       void* stream, bool clear_header) {
  if (M < 0 || M > kMaxDim) return fail(EE_ERR_INVALID, "bad M=%lld", (long long)M);
  int st = check_ws(workspace, workspace_bytes, gated_ws_bytes(M, 0));
  if (st != EE_OK) return st;
  if (logits == nullptr) return fail(EE_ERR_INVALID, "logits is NULL");
  if (n <= 0 || ld < n || n > kMaxDim) return fail(EE_ERR_INVALID, "bad n=%lld / ld=%lld", (long long)n, (long long)ld);
  if (reinterpret_cast<uintptr_t>(logits) & 1u) return fail(EE_ERR_MISALIGNED, "logits must be 2-byte aligned");
  cudaStream_t s = as_stream(stream);
  GatedWs w = gated_ws(workspace, M, 0);
  cudaError_t e = cudaSuccess;
  // ticket, counts, tile counters
  if (clear_header && (e = cudaMemsetAsync(workspace, 0, kWsHeadBytes, s)) != cudaSuccess)
    return cuda_fail(e, "cudaMemsetAsync");
  if (M > 0) {
    ee::SoftmaxArgs a;
    std::memset(&a, 0, sizeof(a));
    a.x = logits;
    a.ldx = ld;
    a.rows = M;
    a.n = static_cast<int>(n);
    a.S = 1;
    a.H = w.H;
    a.route = w.route;
    a.tau_low = tau_low;
    a.tau_high = tau_high;
    a.chunk_tab = w.chunk_tab;
    a.counts = w.counts;
    a.ticket = w.ticket;
    if ((st = check_launch(ee::launch_softmax_entropy(a, s), "softmax_entropy")) != EE_OK) return st;
  }
  if (H && M > 0 && (e = cudaMemcpyAsync(H, w.H, sizeof(float) * M, cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyAsync(H)");
  if (route && M > 0 && (e = cudaMemcpyAsync(route, w.route, M, cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyAsync(route)");
  if (bucket_counts &&
      (e = cudaMemcpyAsync(bucket_counts, w.counts, 3 * sizeof(int32_t), cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyAsync(counts)");
  return EE_OK;
}

extern "C" {

int ee_gate_entropies(const float* H, int64_t M, double tau_low, double tau_high, int8_t* route, int32_t* bucket_counts,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0 || M > kMaxDim) return fail(EE_ERR_INVALID, "bad M=%lld", (long long)M);
  int st = check_ws(workspace, workspace_bytes, gated_ws_bytes(M, 0));
  if (st != EE_OK) return st;
  if (H == nullptr && M > 0) return fail(EE_ERR_INVALID, "H is NULL");
  if (reinterpret_cast<uintptr_t>(H) & 3u) return fail(EE_ERR_MISALIGNED, "H must be 4-byte aligned");
  cudaStream_t s = as_stream(stream);
  GatedWs w = gated_ws(workspace, M, 0);
  cudaError_t e = cudaMemsetAsync(workspace, 0, kWsHeadBytes, s);  // ticket, counts, GEMM tile scheduler
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
  if (M > 0 && (st = check_launch(ee::launch_route_entropies(H, M, tau_low, tau_high, w.H, w.route, w.chunk_tab,
                                                              w.counts, w.ticket, s),
                                  "route_entropies")) != EE_OK)
    return st;
  if (route && M > 0 && (e = cudaMemcpyAsync(route, w.route, M, cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyAsync(route)");
  if (bucket_counts &&
      (e = cudaMemcpyAsync(bucket_counts, w.counts, 3 * sizeof(int32_t), cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
    return cuda_fail(e, "cudaMemcpyAsync(counts)");
  return EE_OK;
}

int ee_gated_workspace_layout(int64_t M, int64_t K, int64_t* offsets) {
  if (M < 0 || K < 0 || offsets == nullptr) return fail(EE_ERR_INVALID, "bad arguments");
  char* base = nullptr;
  GatedWs w = gated_ws(base, M, K);
  offsets[0] = reinterpret_cast<char*>(w.counts) - base;
  offsets[1] = reinterpret_cast<char*>(w.perm) - base;
  offsets[2] = reinterpret_cast<char*>(w.slot) - base;
  offsets[3] = reinterpret_cast<char*>(w.route) - base;
  offsets[4] = reinterpret_cast<char*>(w.H) - base;
  offsets[5] = reinterpret_cast<char*>(w.sa) - base;
  offsets[6] = reinterpret_cast<char*>(w.buf8) - base;
  offsets[7] = reinterpret_cast<char*>(w.buf16) - base;
  return EE_OK;
}

int ee_gated_pack(const void* A, int64_t lda, int64_t M, int64_t K, void* workspace, size_t workspace_bytes,
                  void* stream) {
  int st = check_rows_input(A, M, K, lda);
  if (st != EE_OK) return st;
  if (K % 16 != 0) return fail(EE_ERR_UNSUPPORTED, "K=%lld must be a multiple of 16", (long long)K);
  if ((st = check_ws(workspace, workspace_bytes, gated_ws_bytes(M, K))) != EE_OK) return st;
  if (M == 0) return EE_OK;
  GatedWs w = gated_ws(workspace, M, K);
  return pack_rows(A, lda, M, K, w.route, 0, &w, w.sa, w.buf8, K, w.buf16, K, as_stream(stream));
}

int ee_gated_gemm_packed(int64_t M, int64_t K, const int8_t* W_i8_nk, const uint8_t* W_e4m3_nk,
                         const void* W_f16_nk, const float* w_scale, int64_t N, void* Y, int64_t ldy,
                         void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_gemm_shape(M, N, K, ldy);
  if (st != EE_OK) return st;
  if ((st = check_ws(workspace, workspace_bytes, gated_ws_bytes(M, K))) != EE_OK) return st;
  if (M == 0) return EE_OK;
  if (!W_i8_nk || !W_e4m3_nk || !W_f16_nk || !w_scale || !Y)
    return fail(EE_ERR_INVALID, "all three weight packs, w_scale and Y are required");
  if (!al16(W_i8_nk) || !al16(W_e4m3_nk) || !al16(W_f16_nk) || !al16(w_scale) || !al16(Y))
    return fail(EE_ERR_MISALIGNED, "weights, w_scale and Y must be 16-byte aligned");
  GatedWs w = gated_ws(workspace, M, K);
  GemmOperands op;
  op.a8 = w.buf8;
  op.ld8 = K;
  op.a16 = w.buf16;
  op.ld16 = K;
  op.w[ee::kINT8] = W_i8_nk;
  op.w[ee::kFP8] = W_e4m3_nk;
  op.w[ee::kFP16] = W_f16_nk;
  ee::GemmArgs args = base_args(M, N, K, Y, ldy, 0);
  args.dyn_counts = w.counts;
  args.perm = w.perm;
  args.sa = w.sa;
  args.sb = w_scale;
  args.sched = w.sched;
  attach_split_area(args, workspace, workspace_bytes, M, K);
  return run_gemm(op, args, true, as_stream(stream));
}

int ee_gated_swiglu_packed(int64_t M, int64_t K, const int8_t* Wgu_i8_nk, const uint8_t* Wgu_e4m3_nk,
                           const void* Wgu_f16_nk, const float* wgu_scale, int64_t I, void* Y, int64_t ldy,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (I <= 0 || I % 128 != 0) return fail(EE_ERR_UNSUPPORTED, "I=%lld must be a positive multiple of 128", (long long)I);
  int st = check_gemm_shape(M, 2 * I, K, 2 * I);
  if (st != EE_OK) return st;
  if (ldy < I || ldy % 8 != 0) return fail(EE_ERR_MISALIGNED, "ldy=%lld must be >= I and a multiple of 8", (long long)ldy);
  if ((st = check_ws(workspace, workspace_bytes, gated_ws_bytes(M, K))) != EE_OK) return st;
  if (M == 0) return EE_OK;
  if (!Wgu_i8_nk || !Wgu_e4m3_nk || !Wgu_f16_nk || !wgu_scale || !Y)
    return fail(EE_ERR_INVALID, "all three weight packs, the scales and Y are required");
  if (!al16(Wgu_i8_nk) || !al16(Wgu_e4m3_nk) || !al16(Wgu_f16_nk) || !al16(wgu_scale) || !al16(Y))
    return fail(EE_ERR_MISALIGNED, "weights, scales and Y must be 16-byte aligned");
  GatedWs w = gated_ws(workspace, M, K);
  GemmOperands op;
  op.a8 = w.buf8;
  op.ld8 = K;
  op.a16 = w.buf16;
  op.ld16 = K;
  op.w[ee::kINT8] = Wgu_i8_nk;
  op.w[ee::kFP8] = Wgu_e4m3_nk;
  op.w[ee::kFP16] = Wgu_f16_nk;
  ee::GemmArgs args = base_args(M, 2 * I, K, Y, ldy, 2);
  args.dyn_counts = w.counts;
  args.perm = w.perm;
  args.sa = w.sa;
  args.sb = wgu_scale;
  args.sched = w.sched;
  attach_split_area(args, workspace, workspace_bytes, M, K);
  return run_gemm(op, args, true, as_stream(stream));
}

int ee_gated_gemm(const void* A, int64_t lda, int64_t M, int64_t K, const int8_t* W_i8_nk,
                  const uint8_t* W_e4m3_nk, const void* W_f16_nk, const float* w_scale, int64_t N, void* Y,
                  int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_gemm_shape(M, N, K, ldy);
  if (st != EE_OK) return st;
  if ((st = ee_gated_pack(A, lda, M, K, workspace, workspace_bytes, stream)) != EE_OK) return st;
  return ee_gated_gemm_packed(M, K, W_i8_nk, W_e4m3_nk, W_f16_nk, w_scale, N, Y, ldy, workspace, workspace_bytes,
                              stream);
}

int ee_gated_linear(const void* logits, int64_t n, int64_t ld_logits, const void* A, int64_t lda, int64_t M,
                    int64_t K, const int8_t* W_i8_nk, const uint8_t* W_e4m3_nk, const void* W_f16_nk,
                    const float* w_scale, int64_t N, double tau_low, double tau_high, float* H, int8_t* route,
                    int32_t* bucket_counts, void* Y, int64_t ldy, void* workspace, size_t workspace_bytes,
                    void* stream) {
  int st = check_gemm_shape(M, N, K, ldy);
  if (st != EE_OK) return st;
  if ((st = check_ws(workspace, workspace_bytes, gated_ws_bytes(M, K))) != EE_OK) return st;
  if ((st = ee_gate_rows(logits, M, n, ld_logits, tau_low, tau_high, H, route, bucket_counts, workspace,
                         workspace_bytes, stream)) != EE_OK)
    return st;
  return ee_gated_gemm(A, lda, M, K, W_i8_nk, W_e4m3_nk, W_f16_nk, w_scale, N, Y, ldy, workspace, workspace_bytes,
                       stream);
}

}  // extern "C"
