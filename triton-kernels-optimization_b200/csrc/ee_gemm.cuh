// ee_gemm.cuh - persistent, warp-specialised tcgen05 GEMM over the three precision
// buckets of the gated linear layer.  Included once, by ee_kernels.cu.
//
//   Y[perm[p], :] = epilogue_b( A_b[p, :] . W_b[:, :]^T )   for every position p of bucket b
//
// bucket INT8 : tcgen05.mma kind::i8     int8 x int8  -> int32 TMEM accumulator,
//               y = fp16((fp32(acc) * sa[p]) * sb[n])
// bucket FP8  : tcgen05.mma kind::f8f6f4 e4m3 x e4m3 -> fp32 accumulator,
//               y = fp16((acc * sa[p]) * sb[n])
// bucket FP16 : tcgen05.mma kind::f16    f16 x f16   -> fp32 accumulator, y = fp16(acc)
//
// Tiles are 128 x 256 (UMMA M x N, one CTA), K staged 128 bytes at a time (128 int8 /
// e4m3 or 64 fp16 elements) through a 4-deep TMA ring with 128-byte swizzle.
// Warp roles: warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 2..5
// epilogue (TMEM -> registers -> dequant -> scattered fp16 row stores).  The 512 TMEM
// columns hold two 256-column accumulators so the epilogue of one tile overlaps the
// MMAs of the next.  Tile order: FP16 tiles first (twice the tensor time of 8-bit),
// then FP8, then INT8; inside a bucket the row tile varies fastest, so CTAs that run
// together share a weight tile.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "ee_internal.h"
#include "ee_ptx.cuh"

namespace ee {

__device__ int g_device_error;  // sticky error word, read back by read_and_clear_device_error

constexpr int kAStageBytes = kBM * kBKBytes;  // 16 KB
constexpr int kGemmThreads = 192;
constexpr int kTmemCols = 2 * kBN;  // two accumulators
constexpr int kBarrierBytes = 384;
constexpr int kScaleBytes = 1024;  // the tile's 256 column scales, staged by the epilogue warps
// Single-CTA kernel, per tile width BN: B stage bytes, ring depth and shared memory.
// BN = 256: 48 KB stages x 4; BN = 64 (weight-streaming calls): 24 KB stages x 8.
template <int BN>
struct SingleCfg {
  static constexpr int kBStageBytes = BN * kBKBytes;
  static constexpr int kStageBytes = kAStageBytes + kBStageBytes;
  static constexpr int kStages = BN == kBN ? 4 : 8;
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;  // two accumulators (allocation >= 32 columns)
  static constexpr size_t kSmem =
      1024 /*alignment slack*/ + size_t(kStages) * kStageBytes + kBarrierBytes + kScaleBytes;
  static_assert(kSmem <= 227 * 1024, "single-CTA GEMM shared memory above the 227 KB per-CTA limit");
};

__device__ __forceinline__ int kblocks_of(int b, int K) {
  const int per = (b == kFP16) ? (kBKBytes / 2) : kBKBytes;  // elements per stage
  return (K + per - 1) / per;
}

// Work geometry of one call.  A work unit is one tile, or one K range of a tile whose K
// loop is split (spl[b] ranges per tile of bucket b).  Units run FP16 first (the longest
// K loops), then FP8, then INT8; inside a bucket the ranges of one tile are adjacent and
// the row tile varies fastest, so CTAs that run together share a weight tile.
struct TileGeo {
  int cnt[3], off[3], mtiles[3], tiles[3];
  int halfmt[3];  // the bucket's half row tile (last m-tile with at most bm / 2 rows), or -1
  int spl[3];     // K ranges per tile
  int gm[3];      // row tiles per raster group (tile_mn)
  int ntn, ntiles;
  int total;      // work units
};

// Makespan, in K stages per slot, of the call's units on `slots` CTAs (pairs) in the
// order the kernel hands them out: every FP16 unit (one cost, ca) first, then the 8-bit
// units (INT8 and FP8 have the same K loop: one cost, cb, for S[0] == S[1]), each unit to
// the slot that frees first.  A unit costs its stages + 1 (pipeline fill) +
// kSplitStoreCost when it stores a partial block (128 KiB per CTA).  Closed form: the
// FP16 units leave r = na mod slots slots one unit (ca) later than the other slots, at
// lo; the 8-bit units start in the merged order of the two lattices lo + k cb (slots - r
// slots) and lo + ca + k cb (r slots), so the last one starts where the nb-th of those
// times lies -- first ceil(ca / cb) per early slot alone, then `slots` per period cb.
// Costs measured on B200: one K stage of a 128 x 256 (pair: 256 x 256) tile about
// 0.4 us.  32-bit arithmetic: plan_splits only plans for K loops of at most
// kSplitMaxKBlocks stages and at most kSplitMaxTiles tiles.
constexpr int kSplitOverhead = 8;
constexpr int kSplitStoreCost = 2;
constexpr int kSplitBlocksPerStage = 12;
constexpr int kSplitMaxKBlocks = 1 << 12;
constexpr int kSplitMaxTiles = 1024;
__device__ __forceinline__ int split_makespan(const int (&tiles)[3], const int (&nkb)[3], const int (&S)[3],
                                              int slots) {
  const int na = tiles[2] * S[2], nb = (tiles[0] + tiles[1]) * S[0];
  const int ca = (nkb[2] + S[2] - 1) / S[2] + 1 + (S[2] > 1 ? kSplitStoreCost : 0);
  const int cb = (nkb[0] + S[0] - 1) / S[0] + 1 + (S[0] > 1 ? kSplitStoreCost : 0);
  const int q = na / slots, r = na - q * slots;
  const int lo = q * ca, hi = r > 0 ? lo + ca : lo;
  if (nb == 0) return hi;
  int start;  // of the last 8-bit unit, after lo
  if (r == 0) {
    start = ((nb - 1) / slots) * cb;
  } else {
    const int nlo = slots - r;
    const int k1 = (ca + cb - 1) / cb;  // units each early slot starts before the late ones free
    if (nb <= nlo * k1) {
      start = ((nb - 1) / nlo) * cb;
    } else {
      const int n2 = nb - nlo * k1 - 1;
      const int i = n2 / slots, rem = n2 - i * slots;
      start = ca + i * cb + (rem < r ? 0 : k1 * cb - ca);
    }
  }
  const int end = lo + start + cb;
  return end > hi ? end : hi;
}

// K-split plan, evaluated by one whole warp (the same result in every CTA and in the
// reduction kernel).  Lanes 0-15 score a common range length C = ceil(longest K loop /
// (l + 1)), each bucket split into ceil(nkb / C) ranges (ranges of all buckets about
// equally long); lanes 16-31 split only the FP16 tiles, into l - 14 ranges (the 8-bit
// tiles whole: their K loops are half as long).  Ranges of at least kSplitMinKBlocks
// stages, the partial blocks within part_blocks.  Score: split_makespan, plus for a plan
// with any split kSplitOverhead (the reduction pass's launch) and the reduction's reads
// of the split units' partial blocks (about one K stage of one slot per
// kSplitBlocksPerStage blocks).  The smallest score wins, ties to the lower lane, and a
// split must beat the whole tiles by a margin (1/8).
__device__ __forceinline__ void plan_splits_warp(TileGeo& g, const GemmArgs& a, int ranks, int lane) {
  g.spl[0] = g.spl[1] = g.spl[2] = 1;
  if (a.part == nullptr || a.split_slots <= 0 || a.part_blocks <= 0 || g.ntiles > kSplitMaxTiles) return;
  int nkb[3];
  const int tiles[3] = {g.tiles[0], g.tiles[1], g.tiles[2]};
  int maxkb = 0;
#pragma unroll
  for (int b = 0; b < 3; ++b) {
    nkb[b] = kblocks_of(b, a.K);
    if (tiles[b] > 0 && nkb[b] > maxkb) maxkb = nkb[b];
  }
  if (maxkb < 2 * kSplitMinKBlocks || maxkb > kSplitMaxKBlocks) return;
  int S[3];
  bool ok;
  if (lane < 16) {
    const int C = (maxkb + lane) / (lane + 1);
#pragma unroll
    for (int b = 0; b < 3; ++b) {
      const int sb = (nkb[b] + C - 1) / C;
      S[b] = sb < 1 ? 1 : (sb > kMaxKSplits ? kMaxKSplits : sb);
    }
    ok = lane == 0 || C >= kSplitMinKBlocks;
  } else {
    const int s16 = lane - 14;
    S[0] = S[1] = 1;
    S[2] = s16;
    ok = s16 <= kMaxKSplits && tiles[2] > 0 && tiles[0] + tiles[1] > 0 &&
         (nkb[2] + s16 - 1) / s16 >= kSplitMinKBlocks;
  }
  int units = 0, split_units = 0;
#pragma unroll
  for (int b = 0; b < 3; ++b) {
    units += tiles[b] * S[b];
    split_units += S[b] > 1 ? tiles[b] * S[b] : 0;
  }
  ok = ok && (lane == 0 || units * ranks <= a.part_blocks);
  int e = 1 << 30;
  if (ok)
    e = split_makespan(tiles, nkb, S, a.split_slots) +
        (split_units > 0 ? kSplitOverhead + split_units * ranks / kSplitBlocksPerStage : 0);
  const int e1 = __shfl_sync(0xffffffffu, e, 0);
  if (lane > 0 && 8ll * e >= 7ll * e1) e = 1 << 30;
  // argmin over the warp of (score, lane)
  unsigned long long key = (static_cast<unsigned long long>(static_cast<unsigned>(e)) << 8) | static_cast<unsigned>(lane);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
    key = other < key ? other : key;
  }
  const int lb = static_cast<int>(key & 0xffu);
#pragma unroll
  for (int b = 0; b < 3; ++b) {
    const int sb = __shfl_sync(0xffffffffu, S[b], lb);
    g.spl[b] = tiles[b] > 0 ? sb : 1;  // a bucket without tiles: nothing to reduce
  }
}

// half_tiles: the CTA-pair kernel runs a bucket's last row tile as an M = 128 pair tile
// when it holds at most 128 rows (instead of an M = 256 tile that is mostly padding).
// K splits only for 256-column tiles (one partial block per CTA of a tile).  Called by
// one whole warp (the split plan is spread over its lanes).
//
// Raster order of a bucket's tiles.  When the bucket's activation rows fit in L2 many
// times over (at most kRasterWholeBytes), every row tile of an N column is visited before
// the next column: CTAs running together share the weight tile and the rows stay in L2.
// Above that (tens of thousands of rows at large K) sweeping all rows per column would
// stream the activations from HBM once per wave, so the tiles go in groups of gm row
// tiles (about kRasterGroupBytes of activations): every column of the group's rows before
// the next group, the row tile fastest inside a group.
constexpr long long kRasterWholeBytes = 64ll << 20;
constexpr long long kRasterGroupBytes = 32ll << 20;
__device__ __forceinline__ int raster_group(int mtiles, int bm, int K, int b) {
  const long long per = static_cast<long long>(bm) * K * (b == kFP16 ? 2 : 1);  // bytes of one row tile
  if (per * mtiles <= kRasterWholeBytes) return mtiles > 0 ? mtiles : 1;
  const long long g = kRasterGroupBytes / per;
  return g < 1 ? 1 : (g > mtiles ? mtiles : static_cast<int>(g));
}
// tile lt of a bucket -> (row tile, column tile) in that order
__device__ __forceinline__ void tile_mn(int lt, int mtiles, int ntn, int gm, int& mt, int& nt) {
  const int per_group = gm * ntn;
  const int first = (lt / per_group) * gm;
  const int in = lt - (lt / per_group) * per_group;
  const int rows = mtiles - first < gm ? mtiles - first : gm;
  mt = first + in % rows;
  nt = in / rows;
}

__device__ __forceinline__ TileGeo make_geo_warp(const GemmArgs& a, int bm, int bn, bool half_tiles, int lane) {
  TileGeo g;
  if (a.dyn_counts != nullptr) {
#pragma unroll
    for (int b = 0; b < 3; ++b) g.cnt[b] = *(const volatile int32_t*)(a.dyn_counts + b);
  } else {
#pragma unroll
    for (int b = 0; b < 3; ++b) g.cnt[b] = a.counts[b];
  }
  g.off[0] = 0;
  g.off[1] = g.cnt[0];
  g.off[2] = g.cnt[0] + g.cnt[1];
  g.ntn = (a.N + bn - 1) / bn;
  g.ntiles = 0;
#pragma unroll
  for (int b = 0; b < 3; ++b) {
    g.mtiles[b] = (g.cnt[b] + bm - 1) / bm;
    g.tiles[b] = g.mtiles[b] * g.ntn;
    g.ntiles += g.tiles[b];
    const int rem = g.cnt[b] % bm;
    g.halfmt[b] = (half_tiles && rem >= 1 && rem <= bm / 2) ? g.mtiles[b] - 1 : -1;
    g.gm[b] = raster_group(g.mtiles[b], bm, a.K, b);
  }
  if (bn == kBN) {
    plan_splits_warp(g, a, bm == 2 * kBM ? 2 : 1, lane);
  } else {
    g.spl[0] = g.spl[1] = g.spl[2] = 1;
  }
  g.total = g.tiles[0] * g.spl[0] + g.tiles[1] * g.spl[1] + g.tiles[2] * g.spl[2];
  return g;
}

// the geometry of a CTA, computed by warp 0 into shared memory: the roles read the few
// fields they need per unit instead of holding all of it in registers
// (the first CTA also publishes the split plan for the reduction kernel)
__device__ __forceinline__ void make_geo_shared(TileGeo* sg, const GemmArgs& a, int bm, int bn, bool half_tiles) {
  if (threadIdx.x < 32) {
    const TileGeo g = make_geo_warp(a, bm, bn, half_tiles, static_cast<int>(threadIdx.x));
    if (threadIdx.x == 0) {
      *sg = g;
      if (blockIdx.x == 0 && a.split_plan != nullptr) {
        a.split_plan[0] = g.spl[0];
        a.split_plan[1] = g.spl[1];
        a.split_plan[2] = g.spl[2];
      }
    }
  }
  __syncthreads();
}

// One work unit: bucket, first position (row of A), first output column, half tile,
// K stages [kb0, kb1) and whether the tile is split.  Written out per bucket: a loop
// with an early return here kept TileGeo on the stack.
struct Unit {
  int b, pos0, n0, kb0, kb1;
  bool half, split;
};
__device__ __forceinline__ Unit unit_in(const TileGeo& g, int b, int u, int bm, int bn, int K) {
  const int S = g.spl[b];
  const int t = u / S, r = u % S;
  int mt, nt;
  tile_mn(t, g.mtiles[b], g.ntn, g.gm[b], mt, nt);
  const int nkb = kblocks_of(b, K);
  Unit w;
  w.b = b;
  w.pos0 = g.off[b] + mt * bm;
  w.n0 = nt * bn;
  w.half = mt == g.halfmt[b];
  w.split = S > 1;
  w.kb0 = r * nkb / S;  // S > 1 only for nkb <= kSplitMaxKBlocks
  w.kb1 = (r + 1) * nkb / S;
  return w;
}
__device__ __forceinline__ Unit decode_unit(const TileGeo& g, int v, int bm, int bn, int K) {
  const int u2 = g.tiles[2] * g.spl[2], u1 = g.tiles[1] * g.spl[1];
  if (v < u2) return unit_in(g, 2, v, bm, bn, K);
  v -= u2;
  if (v < u1) return unit_in(g, 1, v, bm, bn, K);
  v -= u1;
  return unit_in(g, 0, v, bm, bn, K);
}

// a split unit's raw accumulator -> its partial block.  Warp `quarter` stores TMEM chunk
// j (32 columns of its 32 lanes, from taddr) to sub-block quarter * 8 + j, laid out as [8
// groups of 4 columns][32 lanes][4]: each of a chunk's 8 stores writes 512 contiguous
// bytes.  Whole warp (tcgen05.ld is .sync.aligned).
constexpr int kPartSubWords = 32 * 32;  // one sub-block: 32 rows x 32 columns
__device__ __forceinline__ void store_partial(uint32_t* blk, int quarter, uint32_t taddr, int nchunks, int lane) {
#pragma unroll 1
  for (int j = 0; j < nchunks; ++j) {
    uint32_t r[32];
    __syncwarp();
    tmem_ld32(taddr + j * 32, r);
    tmem_ld_wait(r);
    uint4* d = reinterpret_cast<uint4*>(blk + (quarter * 8 + j) * kPartSubWords) + lane;
#pragma unroll
    for (int g = 0; g < 8; ++g) d[g * 32] = make_uint4(r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]);
  }
  __syncwarp();
}

// issue the 4 UMMAs (each K = 32 bytes) of one stage
template <int KIND, int BN>
__device__ __forceinline__ void mma_stage(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr, bool first) {
  constexpr uint32_t idesc = (KIND == kKindI8)   ? make_idesc(2u, 1u, kBM, BN)   // s32 <- s8 x s8
                             : (KIND == kKindF8) ? make_idesc(1u, 0u, kBM, BN)   // f32 <- e4m3 x e4m3
                                                 : make_idesc(1u, 0u, kBM, BN);  // f32 <- f16 x f16
  const uint64_t da = sdesc_k_sw128(a_addr);
  const uint64_t db = sdesc_k_sw128(b_addr);
#pragma unroll
  for (int k = 0; k < kBKBytes / 32; ++k) {
    // advancing the start address by 32 bytes = 2 in the descriptor's 16-byte units
    tc_mma<KIND>(d_tmem, da + 2u * k, db + 2u * k, idesc, (first && k == 0) ? 0u : 1u);
  }
}

// Epilogue of one 32-lane quarter of a 128 x 256 accumulator, in two parts.
// epilogue_prepare runs before the accumulator is ready: the thread's row (output row,
// activation scale); stage_scales then puts the tile's column scales into shared memory
// (each epilogue warp loads a quarter), so no global load is left on the drain's path.
// epilogue_drain reads TMEM 32 columns at a time, one chunk ahead of the math; each
// chunk's 32 column scales are read by every lane from the same shared-memory words
// (broadcast), the dequantisation runs on f32x2 pairs and the fp16 row segment leaves in
// 32-byte stores (full sectors) when the output rows allow it.
struct EpiRow {
  bool valid, v8;  // v8: 32-byte aligned output rows
  int64_t orow;
  float sa;
};

__device__ __forceinline__ EpiRow epilogue_prepare(const GemmArgs& args, const TileGeo& geo, int b, int pos, int n0,
                                                   int lane) {
  EpiRow e;
  // end of bucket b's positions, by selects: a runtime index into TileGeo would move
  // the whole struct to the stack
  const int end = (b == 0) ? geo.cnt[0] : (b == 1) ? geo.off[1] + geo.cnt[1] : geo.off[2] + geo.cnt[2];
  e.valid = pos < end;
  e.orow = e.valid ? (args.perm ? static_cast<int64_t>(args.perm[pos]) : static_cast<int64_t>(pos)) : 0;
  e.sa = (e.valid && b != kFP16 && args.out_mode != 1) ? args.sa[pos] : 1.f;
  e.v8 = (reinterpret_cast<uintptr_t>(args.Y) & 31u) == 0 && (args.ldy & 15) == 0;
  return e;
}

// The tile's BN column scales into shared memory (zero past N), one quarter per epilogue
// warp, between two barriers of the four epilogue warps: sc_free (every warp has drained
// the previous tile, so its scales may be overwritten) and sc_full (all quarters
// written).  k: tiles this warp has staged before.  False if a wait gave up.
template <int BN>
__device__ __forceinline__ bool stage_scales(const GemmArgs& args, int b, int n0, int quarter, int lane, float* s_sc,
                                             uint64_t* sc_full, uint64_t* sc_free, uint32_t k,
                                             const volatile int* abort) {
  constexpr int kPer = BN / 4;
  const bool need = b != kFP16 && args.out_mode != 1;
  float v[(kPer + 31) / 32];
#pragma unroll
  for (int i = 0; i < (kPer + 31) / 32; ++i) {
    const int j = quarter * kPer + i * 32 + lane;
    v[i] = (need && i * 32 + lane < kPer && n0 + j < args.N) ? __ldg(args.sb + n0 + j) : 0.f;
  }
  if (k > 0 && !mbar_wait(sc_free, (k - 1) & 1u, abort)) return false;
#pragma unroll
  for (int i = 0; i < (kPer + 31) / 32; ++i)
    if (i * 32 + lane < kPer) s_sc[quarter * kPer + i * 32 + lane] = v[i];
  __syncwarp();
  if (lane == 0) mbar_arrive(sc_full);
  return mbar_wait(sc_full, k & 1u, abort);
}

// the staged column scales c0 .. c0 + 31 of the tile, the same shared-memory words in
// every lane
__device__ __forceinline__ void tile_scales(const float* s_sc, int c0, float (&v)[32]) {
  const uint32_t a = smem_u32(s_sc + c0);
#pragma unroll
  for (int g = 0; g < 8; ++g)
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v[4 * g]), "=f"(v[4 * g + 1]), "=f"(v[4 * g + 2]), "=f"(v[4 * g + 3])
                 : "r"(a + 16u * g));
}

// the column scales of output columns nc .. nc + 31 from global memory (zero past N;
// N % 8 == 0): the reduction kernel's path
__device__ __forceinline__ void column_scales(const float* sb, int nc, int N, float (&v)[32]) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
    if (nc + 8 * g < N) {
      lo = __ldg(reinterpret_cast<const float4*>(sb + nc + 8 * g));
      hi = __ldg(reinterpret_cast<const float4*>(sb + nc + 8 * g + 4));
    }
    v[8 * g + 0] = lo.x; v[8 * g + 1] = lo.y; v[8 * g + 2] = lo.z; v[8 * g + 3] = lo.w;
    v[8 * g + 4] = hi.x; v[8 * g + 5] = hi.y; v[8 * g + 6] = hi.z; v[8 * g + 7] = hi.w;
  }
}

// 32 consecutive bytes (16 fp16) to global memory in one 256-bit store; p 32-byte aligned
__device__ __forceinline__ void st_global_32B(void* p, const uint32_t (&w)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]),
               "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// one 32-column chunk c of the drain (r: its accumulator values); stores only for valid
// rows and columns.  s_sc: the tile's staged column scales, or null to read them from
// global memory
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& args, const EpiRow& e, int b, int n0, int c,
                                               const uint32_t (&r)[32], const float* s_sc) {
  const int nc = n0 + c * 32;
  if (!e.valid || nc >= args.N) return;
  if (args.out_mode == 1) {
    uint32_t* y = static_cast<uint32_t*>(args.Y) + e.orow * args.ldy + nc;
#pragma unroll
    for (int g = 0; g < 8; ++g)
      if (nc + 4 * g < args.N) *reinterpret_cast<uint4*>(y + 4 * g) = make_uint4(r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]);
    return;
  }
  // fp16 pairs of the row segment: (acc * sa) * sb per element, each product rounded
  // (the f32x2 multiplies round each lane as the scalar ones do)
  uint32_t h[16];
  if (b == kFP16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const __half2 v = __floats2half2_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
      h[j] = *reinterpret_cast<const uint32_t*>(&v);
    }
  } else {
    float sbv[32];
    if (s_sc != nullptr)
      tile_scales(s_sc, c * 32, sbv);
    else
      column_scales(args.sb, nc, args.N, sbv);
    const float2 sa2 = make_float2(e.sa, e.sa);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 acc = (b == kINT8) ? make_float2(static_cast<float>(static_cast<int32_t>(r[2 * j])),
                                                    static_cast<float>(static_cast<int32_t>(r[2 * j + 1])))
                                      : make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
      const float2 f = __fmul2_rn(__fmul2_rn(acc, sa2), make_float2(sbv[2 * j], sbv[2 * j + 1]));
      const __half2 v = __floats2half2_rn(f.x, f.y);
      h[j] = *reinterpret_cast<const uint32_t*>(&v);
    }
  }
  __half* y = static_cast<__half*>(args.Y) + e.orow * args.ldy + nc;
  if (e.v8) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (nc + 16 * q + 16 <= args.N) {
        const uint32_t w[8] = {h[8 * q], h[8 * q + 1], h[8 * q + 2], h[8 * q + 3],
                               h[8 * q + 4], h[8 * q + 5], h[8 * q + 6], h[8 * q + 7]};
        st_global_32B(y + 16 * q, w);
      } else if (nc + 16 * q < args.N) {
        *reinterpret_cast<uint4*>(y + 16 * q) = make_uint4(h[8 * q], h[8 * q + 1], h[8 * q + 2], h[8 * q + 3]);
      }
    }
  } else {
#pragma unroll
    for (int g = 0; g < 4; ++g)
      if (nc + 8 * g < args.N)
        *reinterpret_cast<uint4*>(y + 8 * g) = make_uint4(h[4 * g], h[4 * g + 1], h[4 * g + 2], h[4 * g + 3]);
  }
}

// SwiGLU epilogue (out_mode 2): the weight rows come interleaved in groups of 128 --
// tile columns [0, 128) are gate channels n0/2 + [0, 128), columns [128, 256) the
// matching up channels -- and the output is h = silu(gate) * up with I = N/2 columns.
// Every value is rounded where the unfused sequence rounds it: gate and up to fp16 as
// the bucket's GEMM writes them, silu(g) = g / (1 + exp(-g)) in fp32 (IEEE division)
// to fp16, then the fp16 product -- what torch.nn.functional.silu(gate) * up computes
// on the GEMMs' fp16 outputs.
__device__ __forceinline__ float swiglu_dequant(uint32_t r, int b, float sa, float sb) {
  if (b == kFP16) return __uint_as_float(r);
  const float acc = (b == kINT8) ? static_cast<float>(static_cast<int32_t>(r)) : __uint_as_float(r);
  return __fmul_rn(__fmul_rn(acc, sa), sb);
}

__device__ __forceinline__ void swiglu_chunk(const GemmArgs& args, const EpiRow& e, int b, int n0, int c,
                                             const uint32_t (&rg)[32], const uint32_t (&ru)[32], const float* s_sc) {
  const int inter = args.N / 2;
  const int oc = n0 / 2 + c * 32;  // first output column of the chunk
  if (!e.valid || oc >= inter) return;
  float sg[32], su[32];
  if (b != kFP16) {
    if (s_sc != nullptr) {
      tile_scales(s_sc, c * 32, sg);
      tile_scales(s_sc, kBN / 2 + c * 32, su);
    } else {
      column_scales(args.sb, n0 + c * 32, args.N, sg);
      column_scales(args.sb, n0 + kBN / 2 + c * 32, args.N, su);
    }
  }
  __half* y = static_cast<__half*>(args.Y) + e.orow * args.ldy + oc;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    if (oc + 8 * g < inter) {
      uint4 out;
      __half* o = reinterpret_cast<__half*>(&out);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int j = 8 * g + k;
        const float gate = __half2float(__float2half_rn(swiglu_dequant(rg[j], b, e.sa, b == kFP16 ? 1.f : sg[j])));
        const float up = __half2float(__float2half_rn(swiglu_dequant(ru[j], b, e.sa, b == kFP16 ? 1.f : su[j])));
        const float act = __half2float(__float2half_rn(__fdiv_rn(gate, 1.f + expf(-gate))));
        o[k] = __float2half_rn(act * up);
      }
      *reinterpret_cast<uint4*>(y + 8 * g) = out;
    }
  }
}

__device__ __forceinline__ void epilogue_drain_swiglu(const GemmArgs& args, const EpiRow& e, int b, int n0,
                                                      uint32_t taddr, const float* s_sc) {
  uint32_t rg[32], ru[32];
#pragma unroll 1
  for (int c = 0; c < kBN / 64; ++c) {
    __syncwarp();
    tmem_ld32(taddr + c * 32, rg);
    tmem_ld32(taddr + kBN / 2 + c * 32, ru);
    tmem_ld_wait(rg);
    tmem_ld_wait(ru);
    swiglu_chunk(args, e, b, n0, c, rg, ru, s_sc);
  }
  __syncwarp();
}

// Drains the quarter's 256 columns (taddr: its lanes, first column); the whole warp
// calls it (tcgen05.ld is .sync.aligned).  The TMEM read of chunk c+1 is in flight
// while chunk c is converted and stored.
// nchunks TMEM chunks of 32 columns from taddr, output chunks chunk0 .. chunk0 + nchunks - 1
// of the tile (an even count: two per iteration).
template <int BN = kBN>
__device__ __forceinline__ void epilogue_drain(const GemmArgs& args, const EpiRow& e, int b, int n0, uint32_t taddr,
                                               const float* s_sc, int chunk0 = 0, int nchunks = BN / 32) {
  if constexpr (BN == kBN) {
    if (args.out_mode == 2) {
      epilogue_drain_swiglu(args, e, b, n0, taddr, s_sc);
      return;
    }
  }
  uint32_t ra[32], rb[32];
  __syncwarp();
  tmem_ld32(taddr, ra);
  tmem_ld_wait(ra);
#pragma unroll 1
  for (int c = 0; c < nchunks; c += 2) {
    __syncwarp();
    tmem_ld32(taddr + (c + 1) * 32, rb);
    epilogue_chunk(args, e, b, n0, chunk0 + c, ra, s_sc);
    tmem_ld_wait(rb);
    const bool more = c + 2 < nchunks;
    __syncwarp();
    if (more) tmem_ld32(taddr + (c + 2) * 32, ra);
    epilogue_chunk(args, e, b, n0, chunk0 + c + 1, rb, s_sc);
    if (more) tmem_ld_wait(ra);
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------------
// tile feed.  Static mode: tiles blockIdx.x, blockIdx.x + gridDim.x, ...  Dynamic mode
// (args.sched != nullptr): the producer warp takes tile blockIdx.x first (no claim: the
// first wave needs no counter round trip), then claims gridDim.x + the next value of a
// global counter, and publishes each tile through a ring of kTileRing shared-memory
// slots; the MMA warp and the four epilogue warps read the same sequence from the ring.
// Claiming in tile order (FP16 tiles first) gives longest-first list scheduling across
// the SMs.
// ---------------------------------------------------------------------------------
constexpr int kTileRing = 4;
constexpr uint32_t kRingConsumers = 5;  // MMA warp + 4 epilogue warps

struct Feed {
  uint32_t slot, phase;
  int next;  // static mode: the next tile; dynamic mode: the first tile, then -1
};

// producer side; returns the tile (>= total: no more work) or -1 if a wait gave up
__device__ __forceinline__ int feed_produce(Feed& f, bool dyn, int* ring, uint64_t* ring_full, uint64_t* ring_empty,
                                            uint32_t* counter, int lane, const volatile int* abort) {
  if (!dyn) {
    const int t = f.next;
    f.next += gridDim.x;
    return t;
  }
  if (!mbar_wait(&ring_empty[f.slot], f.phase ^ 1u, abort)) return -1;
  int t = 0;
  if (lane == 0) {
    t = f.next >= 0 ? f.next : static_cast<int>(gridDim.x + atomicAdd(counter, 1u));
    ring[f.slot] = t;
    mbar_arrive(&ring_full[f.slot]);
  }
  t = __shfl_sync(0xffffffffu, t, 0);
  f.next = -1;
  if (++f.slot == kTileRing) {
    f.slot = 0;
    f.phase ^= 1u;
  }
  return t;
}

// consumer side (whole warp); lane 0 releases the slot
__device__ __forceinline__ int feed_consume(Feed& f, bool dyn, const int* ring, uint64_t* ring_full,
                                            uint64_t* ring_empty, int lane, const volatile int* abort) {
  if (!dyn) {
    const int t = f.next;
    f.next += gridDim.x;
    return t;
  }
  if (!mbar_wait(&ring_full[f.slot], f.phase, abort)) return -1;
  const int t = *reinterpret_cast<const volatile int*>(&ring[f.slot]);
  __syncwarp();
  if (lane == 0) mbar_arrive(&ring_empty[f.slot]);
  if (++f.slot == kTileRing) {
    f.slot = 0;
    f.phase ^= 1u;
  }
  return t;
}

// the last CTA to leave resets the scheduler words for the next launch
__device__ __forceinline__ void feed_retire(const GemmArgs& args) {
  if (args.sched == nullptr || threadIdx.x != 0) return;
  __threadfence();
  const uint32_t prev = atomicAdd(&args.sched[1], 1u);
  if (prev == gridDim.x - 1) {
    atomicExch(&args.sched[0], 0u);
    atomicExch(&args.sched[1], 0u);
  }
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gated_gemm_kernel(const __grid_constant__ CUtensorMap tm_a8, const __grid_constant__ CUtensorMap tm_a16,
                      const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                      const __grid_constant__ CUtensorMap tm_w2, const GemmArgs args) {
  using Cfg = SingleCfg<BN>;
  constexpr int kStages = Cfg::kStages;
  constexpr int kBStageBytes = Cfg::kBStageBytes;
  constexpr int kStageBytes = Cfg::kStageBytes;
  constexpr int kTmemCols = Cfg::kTmemCols;
  static_assert((2 * kStages + 7 + 2 * kTileRing) * 8 + 8 + 4 * kTileRing <= kBarrierBytes,
                "single-CTA GEMM barrier region overflows");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kAStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kStages * kBStageBytes);
  uint64_t* full = bars;                         // [kStages] TMA -> MMA
  uint64_t* empty = bars + kStages;              // [kStages] MMA -> TMA
  uint64_t* acc_full = bars + 2 * kStages;       // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;            // [2] epilogue -> MMA
  uint64_t* drain = acc_empty + 2;               // MMA drain on abort
  uint64_t* ring_full = drain + 1;               // [kTileRing] producer -> consumers
  uint64_t* ring_empty = ring_full + kTileRing;  // [kTileRing] consumers -> producer
  uint64_t* sc_full = ring_empty + kTileRing;     // the tile's column scales staged (4 epilogue warps)
  uint64_t* sc_free = sc_full + 1;                // the previous tile's scales read (4 epilogue warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sc_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* ring = const_cast<int*>(abort_flag + 1);  // [kTileRing] tile indices
  float* s_sc = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + kBarrierBytes);  // [BN]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // barriers and descriptor prefetch first: they read nothing an earlier kernel writes
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // one arrive per epilogue warp
    }
    mbar_init(drain, 1);
    for (int i = 0; i < kTileRing; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], kRingConsumers);
    }
    mbar_init(sc_full, 4);
    mbar_init(sc_free, 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a8);
    tma_prefetch_desc(&tm_a16);
    tma_prefetch_desc(&tm_w0);
    tma_prefetch_desc(&tm_w1);
    tma_prefetch_desc(&tm_w2);
  }
  griddep_wait();  // bucket counts, packed rows and the tile counter come from earlier kernels
  griddep_launch_dependents();
  // the geometry lives in shared memory: the roles read the few fields they need per
  // unit instead of holding all of it in registers for the whole kernel
  __shared__ TileGeo s_geo;
  make_geo_shared(&s_geo, args, kBM, BN, false);
  const TileGeo& geo = s_geo;
  if (static_cast<int>(blockIdx.x) >= geo.total) {  // uniform for the whole CTA
    feed_retire(args);
    return;
  }
  const bool dyn = args.sched != nullptr;

  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int K = args.K;
  Feed feed{0u, 0u, static_cast<int>(blockIdx.x)};
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    uint32_t stage = 0, phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;  // per stage: load in flight, its phase parity
    bool failed = false;
    bool drop = args.drop_load_cta == static_cast<int>(blockIdx.x) + 1;  // test hook (GemmArgs)
    for (;;) {
      const int t = feed_produce(feed, dyn, ring, ring_full, ring_empty, args.sched, lane, abort_flag);
      if (t < 0) {
        failed = true;
        break;
      }
      if (t >= geo.total) break;
      const Unit w = decode_unit(geo, t, kBM, BN, K);
      const int b = w.b, pos0 = w.pos0, n0 = w.n0;
      const int kstep = (b == kFP16) ? kBKBytes / 2 : kBKBytes;
      const CUtensorMap* ta = (b == kFP16) ? &tm_a16 : &tm_a8;
      const CUtensorMap* tw = (b == kINT8) ? &tm_w0 : (b == kFP8 ? &tm_w1 : &tm_w2);
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
          failed = true;
          break;
        }
        if (!drop) {
          if (lane == 0) {
            mbar_arrive_expect_tx(&full[stage], kStageBytes);
            tma_load_2d(sA + stage * kAStageBytes, ta, &full[stage], kb * kstep, pos0);
            tma_load_2d(sB + stage * kBStageBytes, tw, &full[stage], kb * kstep, n0);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        }
        drop = false;
        __syncwarp();
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (failed) break;
    }
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
      // let the copies already issued land before the shared memory goes away
      for (int s = 0; s < kStages; ++s)
        if (issued_mask & (1u << s)) (void)mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    uint32_t stage = 0, phase = 0, ab = 0, aphase = 0;
    bool failed = false;
    for (;;) {
      const int t = feed_consume(feed, dyn, ring, ring_full, ring_empty, lane, abort_flag);
      if (t < 0) {
        failed = true;
        break;
      }
      if (t >= geo.total) break;
      const Unit w = decode_unit(geo, t, kBM, BN, K);
      const int b = w.b;
      if (!mbar_wait(&acc_empty[ab], aphase ^ 1u, abort_flag)) {
        failed = true;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + ab * BN;
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(sA + stage * kAStageBytes);
          const uint32_t b_addr = smem_u32(sB + stage * kBStageBytes);
          if (b == kINT8)
            mma_stage<kKindI8, BN>(d_tmem, a_addr, b_addr, kb == w.kb0);
          else if (b == kFP8)
            mma_stage<kKindF8, BN>(d_tmem, a_addr, b_addr, kb == w.kb0);
          else
            mma_stage<kKindF16, BN>(d_tmem, a_addr, b_addr, kb == w.kb0);
          tc_commit(&empty[stage]);  // frees the stage once these MMAs have read it
        }
        __syncwarp();
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (failed) break;
      if (lane == 0) tc_commit(&acc_full[ab]);
      __syncwarp();
      ab ^= 1u;
      if (ab == 0) aphase ^= 1u;
    }
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
        tc_commit(drain);  // completes once every MMA issued so far has finished
      }
      __syncwarp();
      (void)mbar_wait(drain, 0u, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lanes this warp may access: 32*quarter ..
    uint32_t ab = 0, aphase = 0, staged = 0;
    for (;;) {
      const int t = feed_consume(feed, dyn, ring, ring_full, ring_empty, lane, abort_flag);
      bool failed = t < 0;
      if (!failed && t >= geo.total) break;
      Unit w;
      if (failed) {
        w.b = 0;
        w.pos0 = w.n0 = 0;
        w.split = false;
      } else {
        w = decode_unit(geo, t, kBM, BN, K);
      }
      const int b = w.b, n0 = w.n0;
      const EpiRow er = epilogue_prepare(args, geo, b, w.pos0 + quarter * 32 + lane, n0, lane);
      if (!failed && !stage_scales<BN>(args, b, n0, quarter, lane, s_sc, sc_full, sc_free, staged++, abort_flag))
        failed = true;
      if (!failed && !mbar_wait(&acc_full[ab], aphase, abort_flag)) failed = true;
      if (failed) {
        if (lane == 0) {
          atomicOr(&g_device_error, kErrWaitTimeout);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ab * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      if (w.split)  // a K range of a split tile: raw partial, reduced by reduce_partials_kernel
        store_partial(args.part + static_cast<size_t>(t) * (kPartBlockBytes / 4), quarter, taddr, BN / 32, lane);
      else
        epilogue_drain<BN>(args, er, b, n0, taddr, s_sc);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acc_empty[ab]);
        mbar_arrive(sc_free);
      }
      ab ^= 1u;
      if (ab == 0) aphase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
  feed_retire(args);
}

// ---------------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2).  A cluster of two CTAs on neighbouring SMs
// computes a 256 x 256 tile: each CTA stages 128 rows of A and 128 rows of B (half of
// the tile's output columns) per 128-byte K stage, the leader CTA issues M=256 x N=256
// UMMAs that read both CTAs' stages, and each CTA's TMEM holds its own 128 x 256 half
// of the accumulator.  Per FLOP every CTA moves a third less operand data than the
// single-CTA 128 x 256 tile, and the smaller stages allow a 6-deep ring.
//   full[s]      leader only: both CTAs' TMA bytes of stage s (leader arms 64 KB)
//   empty[s]     both CTAs: the leader's commit frees stage s in both (multicast commit)
//   acc_full[i]  both CTAs: accumulator i is complete (multicast commit)
//   acc_empty[i] leader only: 8 arrivals, the four epilogue warps of each CTA
// Tiles are dealt statically (pair p takes p, p + pairs, ...) or, when the call carries
// scheduler words, claimed dynamically by each pair's leader (pair_feed_publish).
// ---------------------------------------------------------------------------------

// tile feed of a CTA pair: static (pair p: p, p + pairs, ...) or dynamic -- the leader's
// producer takes tile p first, then claims pairs + the next counter value, and publishes
// each tile into the tile ring of both CTAs (its own by a
// local store, the peer's through distributed shared memory, each followed by an arrive
// on that CTA's ring_full); the five consumers of each CTA (MMA issuer or the peer's
// producer, four epilogue warps) release the slot on the leader's ring_empty.
struct PairFeed {
  uint32_t slot, phase;
  int next;  // static mode: the next tile; dynamic mode: the first tile, then -1
};

__device__ __forceinline__ int pair_feed_publish(PairFeed& f, bool dyn, int* ring, uint64_t* ring_full,
                                                 uint64_t* ring_empty, uint32_t* counter, int npairs, int lane,
                                                 const volatile int* abort) {
  if (!dyn) {
    const int t = f.next;
    f.next += npairs;
    return t;
  }
  if (!mbar_wait<true>(&ring_empty[f.slot], f.phase ^ 1u, abort)) return -1;
  int t = 0;
  if (lane == 0) {
    t = f.next >= 0 ? f.next : npairs + static_cast<int>(atomicAdd(counter, 1u));
    ring[f.slot] = t;
    mbar_arrive(&ring_full[f.slot]);
    st_shared_cluster_u32(map_to_cta(smem_u32(&ring[f.slot]), 1), static_cast<uint32_t>(t));
    mbar_arrive_cluster(map_to_cta(smem_u32(&ring_full[f.slot]), 1));
  }
  t = __shfl_sync(0xffffffffu, t, 0);
  f.next = -1;
  if (++f.slot == kTileRing) {
    f.slot = 0;
    f.phase ^= 1u;
  }
  return t;
}

__device__ __forceinline__ int pair_feed_consume(PairFeed& f, bool dyn, const int* ring, uint64_t* ring_full,
                                                 uint64_t* ring_empty, int npairs, int lane,
                                                 const volatile int* abort) {
  if (!dyn) {
    const int t = f.next;
    f.next += npairs;
    return t;
  }
  if (!mbar_wait<true>(&ring_full[f.slot], f.phase, abort)) return -1;
  const int t = *reinterpret_cast<const volatile int*>(&ring[f.slot]);
  __syncwarp();
  if (lane == 0) mbar_arrive_cluster(map_to_cta(smem_u32(&ring_empty[f.slot]), 0));
  if (++f.slot == kTileRing) {
    f.slot = 0;
    f.phase ^= 1u;
  }
  return t;
}

// leader CTAs count themselves out; the last one resets the scheduler words
__device__ __forceinline__ void feed_retire_pair(const GemmArgs& args, int npairs) {
  if (args.sched == nullptr || threadIdx.x != 0) return;
  __threadfence();
  const uint32_t prev = atomicAdd(&args.sched[1], 1u);
  if (prev == static_cast<uint32_t>(npairs) - 1) {
    atomicExch(&args.sched[0], 0u);
    atomicExch(&args.sched[1], 0u);
  }
}

constexpr int kPairRows = 256;
#ifndef EE_PAIR_STAGES
#define EE_PAIR_STAGES 7  // 32 KB per stage per CTA: 7 is the most that fits in 227 KB
#endif
constexpr int kStagesPair = EE_PAIR_STAGES;
constexpr int kHalfStageBytes = 128 * kBKBytes;  // 16 KB: one operand half of one CTA
constexpr int kStageBytesPair = 2 * kHalfStageBytes;
constexpr size_t kGemmSmemPair = 1024 + size_t(kStagesPair) * kStageBytesPair + kBarrierBytes + kScaleBytes;
static_assert(kGemmSmemPair <= 227 * 1024, "pair GEMM shared memory above the 227 KB per-CTA limit");
// barrier region: 2 per stage, 2 x 2 accumulator, drain, 2 per ring slot; then the TMEM
// slot, the abort word and the ring itself
static_assert((2 * kStagesPair + 7 + 2 * kTileRing) * 8 + 8 + 4 * kTileRing <= kBarrierBytes,
              "pair GEMM barrier region overflows");

template <int KIND>
__device__ __forceinline__ void mma_stage_pair(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr, bool first) {
  constexpr uint32_t idesc = (KIND == kKindI8)   ? make_idesc(2u, 1u, kPairRows, kBN)
                             : (KIND == kKindF8) ? make_idesc(1u, 0u, kPairRows, kBN)
                                                 : make_idesc(1u, 0u, kPairRows, kBN);
  const uint64_t da = sdesc_k_sw128(a_addr);
  const uint64_t db = sdesc_k_sw128(b_addr);
#pragma unroll
  for (int k = 0; k < kBKBytes / 32; ++k)
    tc_mma_pair<KIND>(d_tmem, da + 2u * k, db + 2u * k, idesc, (first && k == 0) ? 0u : 1u);
}

// M = 128 pair tile: each CTA supplies 64 rows of A; the accumulator of CTA r holds rows
// 64 r .. 64 r + 63 with columns [0, 128) in TMEM lanes 0..63 and columns [128, 256) in
// lanes 64..127, both at TMEM columns [0, 128) (measured on B200 with a probe MMA of
// known operands: every one of the 128 x 128 results at that place).
template <int KIND>
__device__ __forceinline__ void mma_stage_pair_half(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr, bool first) {
  constexpr uint32_t idesc = (KIND == kKindI8)   ? make_idesc(2u, 1u, kPairRows / 2, kBN)
                             : (KIND == kKindF8) ? make_idesc(1u, 0u, kPairRows / 2, kBN)
                                                 : make_idesc(1u, 0u, kPairRows / 2, kBN);
  const uint64_t da = sdesc_k_sw128(a_addr);
  const uint64_t db = sdesc_k_sw128(b_addr);
#pragma unroll
  for (int k = 0; k < kBKBytes / 32; ++k)
    tc_mma_pair<KIND>(d_tmem, da + 2u * k, db + 2u * k, idesc, (first && k == 0) ? 0u : 1u);
}

// A half tile's epilogue: warp quarter q drains rows (q & 1) * 32 + lane of its CTA's 64
// and output columns (q >> 1) * 128 .. + 127 -- TMEM lanes 32 q .., columns 0 .. 127:
// epilogue_drain over 4 chunks starting at chunk (q >> 1) * 4.

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gated_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a8, const __grid_constant__ CUtensorMap tm_a16,
                           const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                           const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_a8h,
                           const __grid_constant__ CUtensorMap tm_a16h, const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStagesPair * kHalfStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kStagesPair * kHalfStageBytes);
  uint64_t* full = bars;                        // [kStagesPair]
  uint64_t* empty = bars + kStagesPair;         // [kStagesPair]
  uint64_t* acc_full = bars + 2 * kStagesPair;  // [2]
  uint64_t* acc_empty = acc_full + 2;           // [2]
  uint64_t* drain = acc_empty + 2;
  uint64_t* ring_full = drain + 1;               // [kTileRing] both CTAs: tile published
  uint64_t* ring_empty = ring_full + kTileRing;  // [kTileRing] leader: 10 consumers released the slot
  uint64_t* sc_full = ring_empty + kTileRing;     // this CTA's column scales staged (4 epilogue warps)
  uint64_t* sc_free = sc_full + 1;                // the previous tile's scales read (4 epilogue warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sc_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* ring = const_cast<int*>(abort_flag + 1);  // [kTileRing]
  float* s_sc = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + kBarrierBytes);  // [kBN]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  // barriers and descriptor prefetch first: they read nothing an earlier kernel writes
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesPair; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(drain, 1);
    for (int i = 0; i < kTileRing; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 2 * kRingConsumers);  // MMA / producer + 4 epilogue warps, x 2 CTAs
    }
    mbar_init(sc_full, 4);
    mbar_init(sc_free, 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a8);
    tma_prefetch_desc(&tm_a16);
    tma_prefetch_desc(&tm_w0);
    tma_prefetch_desc(&tm_w1);
    tma_prefetch_desc(&tm_w2);
  }
  griddep_wait();  // bucket counts, packed rows and the tile counter come from earlier kernels
  griddep_launch_dependents();
  // half tiles need each thread's gate and up columns in one lane: not with SwiGLU.  The
  // geometry lives in shared memory (see gated_gemm_kernel).
  __shared__ TileGeo s_geo;
  make_geo_shared(&s_geo, args, kPairRows, kBN, args.out_mode != 2);
  const TileGeo& geo = s_geo;
  if (pair >= geo.total) {  // the same decision in both CTAs of the pair
    if (leader) feed_retire_pair(args, npairs);
    return;
  }
  const bool dyn = args.sched != nullptr;

  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int K = args.K;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    uint32_t stage = 0, phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    bool failed = false;
    PairFeed feed{0u, 0u, pair};
    for (;;) {
      const int t = leader ? pair_feed_publish(feed, dyn, ring, ring_full, ring_empty, args.sched, npairs, lane, abort_flag)
                           : pair_feed_consume(feed, dyn, ring, ring_full, ring_empty, npairs, lane, abort_flag);
      if (t < 0) {
        failed = true;
        break;
      }
      if (t >= geo.total) break;
      const Unit w = decode_unit(geo, t, kPairRows, kBN, K);
      const int b = w.b, pos0 = w.pos0, n0 = w.n0;
      const bool half = w.half;
      const int kstep = (b == kFP16) ? kBKBytes / 2 : kBKBytes;
      const CUtensorMap* ta = half ? ((b == kFP16) ? &tm_a16h : &tm_a8h) : ((b == kFP16) ? &tm_a16 : &tm_a8);
      const CUtensorMap* tw = (b == kINT8) ? &tm_w0 : (b == kFP8 ? &tm_w1 : &tm_w2);
      const int arow = pos0 + static_cast<int>(rank) * (half ? 64 : 128);
      const uint32_t stage_tx = half ? 2u * (kHalfStageBytes / 2 + kHalfStageBytes) : 2u * kStageBytesPair;
      const int brow = n0 + static_cast<int>(rank) * (kBN / 2);
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
          failed = true;
          break;
        }
        if (lane == 0) {
          if (leader) mbar_arrive_expect_tx(&full[stage], stage_tx);
          const uint32_t bar = map_to_cta(smem_u32(&full[stage]), 0);
          tma_load_2d_pair(sA + stage * kHalfStageBytes, ta, bar, kb * kstep, arow);
          tma_load_2d_pair(sB + stage * kHalfStageBytes, tw, bar, kb * kstep, brow);
        }
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        __syncwarp();
        if (++stage == kStagesPair) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (failed) break;
    }
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
      if (leader)
        for (int s = 0; s < kStagesPair; ++s)
          if (issued_mask & (1u << s)) (void)mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (leader) {
      uint32_t stage = 0, phase = 0, ab = 0, aphase = 0;
      bool failed = false;
      PairFeed feed{0u, 0u, pair};
      for (;;) {
        const int t = pair_feed_consume(feed, dyn, ring, ring_full, ring_empty, npairs, lane, abort_flag);
        if (t < 0) {
          failed = true;
          break;
        }
        if (t >= geo.total) break;
        const Unit w = decode_unit(geo, t, kPairRows, kBN, K);
        const int b = w.b;
        const bool half = w.half;
        if (!mbar_wait<true>(&acc_empty[ab], aphase ^ 1u, abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ab * kBN;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const bool first = kb == w.kb0;
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            failed = true;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = smem_u32(sA + stage * kHalfStageBytes);
            const uint32_t b_addr = smem_u32(sB + stage * kHalfStageBytes);
            if (half) {
              if (b == kINT8)
                mma_stage_pair_half<kKindI8>(d_tmem, a_addr, b_addr, first);
              else if (b == kFP8)
                mma_stage_pair_half<kKindF8>(d_tmem, a_addr, b_addr, first);
              else
                mma_stage_pair_half<kKindF16>(d_tmem, a_addr, b_addr, first);
            } else if (b == kINT8) {
              mma_stage_pair<kKindI8>(d_tmem, a_addr, b_addr, first);
            } else if (b == kFP8) {
              mma_stage_pair<kKindF8>(d_tmem, a_addr, b_addr, first);
            } else {
              mma_stage_pair<kKindF16>(d_tmem, a_addr, b_addr, first);
            }
            tc_commit_pair_both(&empty[stage], 0x3);
          }
          __syncwarp();
          if (++stage == kStagesPair) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (failed) break;
        if (lane == 0) tc_commit_pair_both(&acc_full[ab], 0x3);
        __syncwarp();
        ab ^= 1u;
        if (ab == 0) aphase ^= 1u;
      }
      if (failed) {
        if (lane == 0) {
          atomicOr(&g_device_error, kErrWaitTimeout);
          *abort_flag = 1;
          tc_commit_pair_local(drain);
        }
        __syncwarp();
        (void)mbar_wait(drain, 0u, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    uint32_t ab = 0, aphase = 0, staged = 0;
    const uint32_t leader_acc_empty0 = map_to_cta(smem_u32(&acc_empty[0]), 0);
    PairFeed feed{0u, 0u, pair};
    for (;;) {
      const int t = pair_feed_consume(feed, dyn, ring, ring_full, ring_empty, npairs, lane, abort_flag);
      if (t < 0) {
        if (lane == 0) {
          atomicOr(&g_device_error, kErrWaitTimeout);
          *abort_flag = 1;
        }
        break;
      }
      if (t >= geo.total) break;
      const Unit w = decode_unit(geo, t, kPairRows, kBN, K);
      const int b = w.b, n0 = w.n0;
      const bool half = w.half;
      const int row = half ? static_cast<int>(rank) * 64 + (quarter & 1) * 32 + lane
                           : static_cast<int>(rank) * 128 + quarter * 32 + lane;
      const EpiRow er = epilogue_prepare(args, geo, b, w.pos0 + row, n0, lane);
      if (!stage_scales<kBN>(args, b, n0, quarter, lane, s_sc, sc_full, sc_free, staged++, abort_flag) ||
          !mbar_wait(&acc_full[ab], aphase, abort_flag)) {
        if (lane == 0) {
          atomicOr(&g_device_error, kErrWaitTimeout);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ab * kBN + (static_cast<uint32_t>(quarter * 32) << 16);
      if (w.split)  // a K range of a split tile: raw partial of this CTA's half
        store_partial(args.part + (2 * static_cast<size_t>(t) + rank) * (kPartBlockBytes / 4), quarter, taddr,
                      half ? 4 : kBN / 32, lane);
      else
        epilogue_drain(args, er, b, n0, taddr, s_sc, half ? (quarter >> 1) * 4 : 0, half ? 4 : kBN / 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_cluster(leader_acc_empty0 + ab * static_cast<uint32_t>(sizeof(uint64_t)));
        mbar_arrive(sc_free);
      }
      ab ^= 1u;
      if (ab == 0) aphase ^= 1u;
    }
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still signal it or read its stages
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
  if (leader) feed_retire_pair(args, npairs);
}

// ---------------------------------------------------------------------------------
// Reduction of the K-split tiles, launched after either GEMM kernel (programmatic
// dependent launch: it starts with the grid dependency wait, so the partial blocks are
// complete).  Block = (tile, CTA of the tile, warp quarter q), 8 warps: warp j adds the
// ranges of output chunk j of the quarter's 32 rows (4 chunks in a half tile; with the
// SwiGLU epilogue warp j < 4 takes gate chunk j and up chunk j + 4) in range order --
// int32 for INT8, fp32 otherwise, so the result does not depend on timing -- and runs
// the tile's epilogue on the sums: the same row, column and scale mapping as the GEMM
// kernels' own epilogue.
// ---------------------------------------------------------------------------------
constexpr int kReduceThreads = 256;

__device__ __forceinline__ void add_partial(uint32_t (&r)[32], const uint4 (&v)[8], bool as_int) {
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const uint32_t w[4] = {v[g].x, v[g].y, v[g].z, v[g].w};
#pragma unroll
    for (int k = 0; k < 4; ++k)
      r[4 * g + k] = as_int ? static_cast<uint32_t>(static_cast<int32_t>(r[4 * g + k]) + static_cast<int32_t>(w[k]))
                            : __float_as_uint(__uint_as_float(r[4 * g + k]) + __uint_as_float(w[k]));
  }
}

// sum over ranges s = 0 .. S-1 of sub-block `sub` of blocks blk0 + s * stride, added in
// range order (one range's 8 loads in flight per thread; two blocks per SM keep the
// memory system busy)
__device__ __forceinline__ void sum_partial_chunk(const uint32_t* part, size_t blk0, size_t stride, int S, int sub,
                                                  int lane, bool as_int, uint32_t (&r)[32]) {
  constexpr size_t kBlockVecs = kPartBlockBytes / 16;
  const uint4* src = reinterpret_cast<const uint4*>(part) + blk0 * kBlockVecs + sub * (kPartSubWords / 4) + lane;
  uint4 v[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) v[g] = __ldcg(src + g * 32);
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    r[4 * g] = v[g].x;
    r[4 * g + 1] = v[g].y;
    r[4 * g + 2] = v[g].z;
    r[4 * g + 3] = v[g].w;
  }
#pragma unroll 1
  for (int s = 1; s < S; ++s) {
    const uint4* p = src + static_cast<size_t>(s) * stride * kBlockVecs;
#pragma unroll
    for (int g = 0; g < 8; ++g) v[g] = __ldcg(p + g * 32);
    add_partial(r, v, as_int);
  }
}

__global__ void __launch_bounds__(kReduceThreads, 2) reduce_partials_kernel(const GemmArgs args, int bm, int ranks,
                                                                         int half_tiles) {
  griddep_wait();  // every partial block of the GEMM before it in the stream is written
  griddep_launch_dependents();
  // the GEMM's split plan (the same as planning again, without the cost)
  int spl[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) spl[i] = __ldcg(args.split_plan + i);
  if (spl[0] <= 1 && spl[1] <= 1 && spl[2] <= 1) return;  // every tile was written whole
  GemmArgs base = args;
  base.part = nullptr;  // tile geometry without planning
  TileGeo geo = make_geo_warp(base, bm, kBN, half_tiles != 0, 0);
#pragma unroll
  for (int i = 0; i < 3; ++i) geo.spl[i] = spl[i] < 1 ? 1 : spl[i];
  const int q = static_cast<int>(blockIdx.x & 3u);
  const int rank = static_cast<int>(blockIdx.x >> 2) % ranks;
  const int T = static_cast<int>(blockIdx.x >> 2) / ranks;
  if (T >= geo.ntiles) return;
  // the tile's bucket (FP16 tiles first, then FP8, then INT8), by selects
  const int t2 = geo.tiles[2], t1 = geo.tiles[1];
  const int b = T < t2 ? 2 : (T < t2 + t1 ? 1 : 0);
  const int lt = b == 2 ? T : (b == 1 ? T - t2 : T - t2 - t1);
  const int S = b == 2 ? geo.spl[2] : (b == 1 ? geo.spl[1] : geo.spl[0]);
  if (S <= 1) return;  // written by the GEMM kernel itself
  const int mtiles = b == 2 ? geo.mtiles[2] : (b == 1 ? geo.mtiles[1] : geo.mtiles[0]);
  const int halfmt = b == 2 ? geo.halfmt[2] : (b == 1 ? geo.halfmt[1] : geo.halfmt[0]);
  const int off = b == 2 ? geo.off[2] : (b == 1 ? geo.off[1] : geo.off[0]);
  const int gm = b == 2 ? geo.gm[2] : (b == 1 ? geo.gm[1] : geo.gm[0]);
  int mt, nt;
  tile_mn(lt, mtiles, geo.ntn, gm, mt, nt);
  const bool half = mt == halfmt;
  const int pos0 = off + mt * bm, n0 = nt * kBN;
  const int ubase = b == 2 ? 0 : (b == 1 ? t2 * geo.spl[2] : t2 * geo.spl[2] + t1 * geo.spl[1]);
  const int u0 = ubase + lt * S;  // the tile's first unit
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = ranks == 2 ? (half ? rank * 64 + (q & 1) * 32 + lane : rank * 128 + q * 32 + lane) : q * 32 + lane;
  const size_t blk0 = static_cast<size_t>(u0) * ranks + rank;
  const bool as_int = b == kINT8;
  if (args.out_mode == 2) {
    if (warp >= 4) return;
    const EpiRow er = epilogue_prepare(args, geo, b, pos0 + row, n0, lane);
    uint32_t rg[32], ru[32];
    sum_partial_chunk(args.part, blk0, ranks, S, q * 8 + warp, lane, as_int, rg);
    sum_partial_chunk(args.part, blk0, ranks, S, q * 8 + warp + 4, lane, as_int, ru);
    swiglu_chunk(args, er, b, n0, warp, rg, ru, nullptr);
    return;
  }
  const int nchunks = half ? 4 : kBN / 32;
  if (warp >= nchunks) return;
  const EpiRow er = epilogue_prepare(args, geo, b, pos0 + row, n0, lane);
  uint32_t r[32];
  sum_partial_chunk(args.part, blk0, ranks, S, q * 8 + warp, lane, as_int, r);
  epilogue_chunk(args, er, b, n0, (half ? (q >> 1) * 4 : 0) + warp, r, nullptr);
}

}  // namespace ee
