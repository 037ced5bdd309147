// ee_gemm_skinny.cuh - the gated GEMM for calls of at most 128 rows, where the run time
// is the weight stream from HBM (decode-sized batches; 16 rows of the Llama-3-8B
// projections move 8-16 bytes of weight per multiply-add).
//
// Operands swap roles: a tile is 128 output channels (weight rows: the UMMA M) x the
// bucket's rows padded to NB (the UMMA N = 16 .. 128), so a K stage is the 16 KB weight
// box plus NB x 128 bytes of activations instead of a 128-row activation box that is
// mostly padding.  K is split across the CTAs of a thread-block cluster (cluster size S,
// a launch attribute): CTA r of the cluster streams K blocks [r nkb / S, (r+1) nkb / S)
// into its own TMEM accumulator, writes it to its shared memory, and after one cluster
// barrier CTA r reduces the columns c = r, r + S, .. over the S partials in rank order
// (distributed shared memory reads) and runs the epilogue for those rows -- integer sums
// for the INT8 bucket (exact), fp32 sums in a fixed order for FP8 / FP16 (deterministic).
// A second cluster barrier keeps every CTA's partials alive until all readers are done.
//
// Grid: x = S x ceil(N / 128) (cluster = S consecutive CTAs of one channel tile),
// y = bucket (FP16, FP8, INT8: the longest weight streams are dealt first).  One tile per
// CTA, two CTAs per SM where the stages allow.  Warp roles as in the persistent kernel:
// warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 2-5 epilogue (thread =
// output channel = TMEM lane).  Every wait is bounded; a CTA whose wait gave up records
// the error, drains its own copies and MMAs, and still takes part in both cluster
// barriers, so no peer waits on it.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "ee_gemm.cuh"
#include "ee_internal.h"
#include "ee_ptx.cuh"

namespace ee {

constexpr int kSkinnyThreads = 192;
constexpr int kSkinnyRows = 128;  // output channels per tile (UMMA M)

template <int NB>
struct SkinnyCfg {
  static_assert(NB == 16 || NB == 32 || NB == 64 || NB == 128, "activation rows per tile");
  static constexpr int kWStageBytes = kSkinnyRows * kBKBytes;  // 16 KB
  static constexpr int kAStageBytes = NB * kBKBytes;           // 2 .. 16 KB
  static constexpr int kStageBytes = kWStageBytes + kAStageBytes;
  // NB <= 64: two CTAs per SM (half of the 228 KB each); NB = 128: one CTA per SM
  static constexpr int kBudget = NB <= 64 ? 112 * 1024 : 226 * 1024;
  static constexpr int kStagesRaw = (kBudget - 1024 - 256) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kTmemCols = NB < 32 ? 32 : NB;
  static constexpr size_t kRedBytes = size_t(NB) * kSkinnyRows * 4;  // one CTA's partial accumulator
  static constexpr size_t kSmem = 1024 + size_t(kStages) * kStageBytes + 256;
  static_assert(kStages >= 3, "skinny GEMM ring too shallow");
  static_assert(kRedBytes <= size_t(kStages) * kStageBytes, "partials must fit in the drained ring");
  static_assert(kSmem <= 227 * 1024, "skinny GEMM shared memory above the 227 KB per-CTA limit");
};

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t ld_shared_cluster_u32(uint32_t cluster_addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
  return v;
}

// issue the 4 UMMAs (K = 32 bytes each) of one stage: D[128 x NB] (+)= W[128 x 128 B] A[NB x 128 B]^T
template <int KIND, int NB>
__device__ __forceinline__ void mma_stage_skinny(uint32_t d_tmem, uint32_t w_addr, uint32_t a_addr, bool first) {
  constexpr uint32_t idesc = (KIND == kKindI8) ? make_idesc(2u, 1u, kSkinnyRows, NB)    // s32 <- s8 x s8
                                               : make_idesc(1u, 0u, kSkinnyRows, NB);   // f32 <- e4m3 / f16
  const uint64_t dw = sdesc_k_sw128(w_addr);
  const uint64_t da = sdesc_k_sw128(a_addr);
#pragma unroll
  for (int k = 0; k < kBKBytes / 32; ++k) tc_mma<KIND>(d_tmem, dw + 2u * k, da + 2u * k, idesc, (first && k == 0) ? 0u : 1u);
}

// y[orow, channel n] from one accumulator value (the persistent kernel's dequantisation:
// INT8 fp16((fp32(acc) sa) sb), FP8 fp16((acc sa) sb), FP16 fp16(acc))
__device__ __forceinline__ void skinny_store(const GemmArgs& args, int b, int64_t orow, int n, float sa, float sb,
                                             uint32_t acc) {
  if (args.out_mode == 1) {
    static_cast<uint32_t*>(args.Y)[orow * args.ldy + n] = acc;
    return;
  }
  float v;
  if (b == kFP16)
    v = __uint_as_float(acc);
  else if (b == kINT8)
    v = __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(acc)), sa), sb);
  else
    v = __fmul_rn(__fmul_rn(__uint_as_float(acc), sa), sb);
  static_cast<__half*>(args.Y)[orow * args.ldy + n] = __float2half_rn(v);
}

// Output row and activation scale of every column (bucket row) of the tile, spread over
// the lanes: column c lives in lane c % 32, slot c / 32, and reaches the other lanes by
// shuffles (one global load per lane instead of one per column and thread).
template <int NB>
struct SkinnyCols {
  static constexpr int kSlots = NB < 32 ? 1 : NB / 32;
  int orow[kSlots];
  float sa[kSlots];
  __device__ __forceinline__ void load(const GemmArgs& args, int b, int pos0, int Mb, int lane) {
#pragma unroll
    for (int j = 0; j < kSlots; ++j) {
      const int c = j * 32 + lane;
      const bool ok = c < Mb;
      orow[j] = ok ? (args.perm ? args.perm[pos0 + c] : pos0 + c) : 0;
      sa[j] = (ok && b != kFP16 && args.out_mode != 1) ? args.sa[pos0 + c] : 1.f;
    }
  }
  // column c (any value below NB; the slot is picked by selects, not a runtime index)
  __device__ __forceinline__ void get(int c, int64_t& o, float& s) const {
    const int j = c >> 5;
    int oo = orow[0];
    float ss = sa[0];
#pragma unroll
    for (int k = 1; k < kSlots; ++k) {
      oo = (j == k) ? orow[k] : oo;
      ss = (j == k) ? sa[k] : ss;
    }
    o = __shfl_sync(0xffffffffu, oo, c & 31);
    s = __shfl_sync(0xffffffffu, ss, c & 31);
  }
};

template <int NB>
__global__ void __launch_bounds__(kSkinnyThreads, 1)
    gated_gemm_skinny_kernel(const __grid_constant__ CUtensorMap tm_a8, const __grid_constant__ CUtensorMap tm_a16,
                             const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                             const __grid_constant__ CUtensorMap tm_w2, const GemmArgs args) {
  using Cfg = SkinnyCfg<NB>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;                                     // [kStages] weight boxes (1024-aligned: 16 KB each)
  uint8_t* sA = smem + kStages * Cfg::kWStageBytes;       // [kStages] activation boxes
  uint32_t* red = reinterpret_cast<uint32_t*>(smem);      // [NB][128] partials, over the drained ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * Cfg::kStageBytes);
  uint64_t* full = bars;               // [kStages]
  uint64_t* empty = bars + kStages;    // [kStages]
  uint64_t* acc_full = bars + 2 * kStages;
  uint64_t* drain = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  static_assert((2 * kStages + 2) * 8 + 8 <= 256, "skinny GEMM barrier region overflows");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t S = cluster_nctarank();
  const uint32_t rank = cluster_ctarank();
  const int n0 = static_cast<int>(blockIdx.x / S) * kSkinnyRows;
  const int b = 2 - static_cast<int>(blockIdx.y);  // FP16, FP8, INT8
  const int nkb = kblocks_of(b, args.K);
  const int kb0 = static_cast<int>((static_cast<int64_t>(rank) * nkb) / S);
  const int kb1 = static_cast<int>((static_cast<int64_t>(rank + 1) * nkb) / S);
  const int kstep = (b == kFP16) ? kBKBytes / 2 : kBKBytes;
  const CUtensorMap* ta = (b == kFP16) ? &tm_a16 : &tm_a8;
  const CUtensorMap* tw = (b == kINT8) ? &tm_w0 : (b == kFP8 ? &tm_w1 : &tm_w2);

  // ---- before the previous kernel has finished: nothing here reads its results
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // The weights are never produced by an earlier kernel of the stream (packs are written by
  // plain launches, which complete before anything after them starts), so the first ring's
  // weight boxes load now; their full barriers get the activation bytes and the arrival later.
  const int pre = (kb1 - kb0) < kStages ? (kb1 - kb0) : kStages;
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(ta);
    tma_prefetch_desc(tw);
    for (int s = 0; s < pre; ++s) {
      mbar_expect_tx(&full[s], Cfg::kWStageBytes);
      tma_load_2d(sW + s * Cfg::kWStageBytes, tw, &full[s], (kb0 + s) * kstep, n0);
    }
  }
  griddep_wait();  // bucket counts and packed rows come from earlier kernels
  griddep_launch_dependents();
  int cnt[3];
#pragma unroll
  for (int i = 0; i < 3; ++i)
    cnt[i] = args.dyn_counts ? *(const volatile int32_t*)(args.dyn_counts + i) : args.counts[i];
  const int Mb = (b == 0) ? cnt[0] : (b == 1) ? cnt[1] : cnt[2];
  const int pos0 = (b == 0) ? 0 : (b == 1) ? cnt[0] : cnt[0] + cnt[1];
  // the same for every CTA of the cluster (same bucket): the whole cluster leaves together
  if (Mb <= 0 || Mb > NB) {
    if (Mb > NB && threadIdx.x == 0) atomicOr(&g_device_error, kErrShape);
    if (warp == 0) {  // let the early weight loads land before the shared memory goes away
      if (lane == 0)
        for (int s = 0; s < pre; ++s) mbar_arrive(&full[s]);
      __syncwarp();
      for (int s = 0; s < pre; ++s) (void)mbar_wait(&full[s], 0u, nullptr);
    }
    return;
  }

  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);  // after griddep_wait: an earlier GEMM may still hold TMEM
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    uint32_t stage = 0, phase = 0, issued_mask = 0, issued_parity = 0;
    bool failed = false;
    for (int kb = kb0; kb < kb1; ++kb) {
      const bool early = kb - kb0 < pre;  // weight box already in flight, stage never used
      if (!early && !mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
        failed = true;
        break;
      }
      if (lane == 0) {
        if (early) {
          mbar_arrive_expect_tx(&full[stage], Cfg::kAStageBytes);
        } else {
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          tma_load_2d(sW + stage * Cfg::kWStageBytes, tw, &full[stage], kb * kstep, n0);
        }
        tma_load_2d(sA + stage * Cfg::kAStageBytes, ta, &full[stage], kb * kstep, pos0);
      }
      issued_mask |= 1u << stage;
      issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
      __syncwarp();
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
      for (int s = 0; s < kStages; ++s)
        if (issued_mask & (1u << s)) (void)mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    uint32_t stage = 0, phase = 0;
    bool failed = false;
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!mbar_wait(&full[stage], phase, abort_flag)) {
        failed = true;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t w_addr = smem_u32(sW + stage * Cfg::kWStageBytes);
        const uint32_t a_addr = smem_u32(sA + stage * Cfg::kAStageBytes);
        if (b == kINT8)
          mma_stage_skinny<kKindI8, NB>(tmem_base, w_addr, a_addr, kb == kb0);
        else if (b == kFP8)
          mma_stage_skinny<kKindF8, NB>(tmem_base, w_addr, a_addr, kb == kb0);
        else
          mma_stage_skinny<kKindF16, NB>(tmem_base, w_addr, a_addr, kb == kb0);
        tc_commit(&empty[stage]);
      }
      __syncwarp();
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (lane == 0) {
      if (failed) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
      tc_commit(failed ? drain : acc_full);  // completes once every MMA issued so far has finished
    }
    __syncwarp();
    if (failed) (void)mbar_wait(drain, 0u, nullptr);
  } else {
    // ------------------------------------------------------------ epilogue, part 1
    const int quarter = warp & 3;
    const int ch = quarter * 32 + lane;  // TMEM lane = output channel n0 + ch
    const int n = n0 + ch;
    const bool has_k = kb1 > kb0;        // a split without K blocks contributes zeros
    bool failed = !mbar_wait(acc_full, 0u, abort_flag);
    if (failed && lane == 0) {
      atomicOr(&g_device_error, kErrWaitTimeout);
      *abort_flag = 1;
    }
    tc_fence_after();
    const float sb = (b != kFP16 && args.out_mode != 1 && n < args.N) ? __ldg(args.sb + n) : 1.f;
    SkinnyCols<NB> cols;
    if (S == 1) cols.load(args, b, pos0, Mb, lane);
#pragma unroll
    for (int c0 = 0; c0 < NB; c0 += 32) {
      uint32_t r[32];
      __syncwarp();
      tmem_ld32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + c0, r);
      tmem_ld_wait(r);
      if (!has_k || failed) {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;
      }
      if (S == 1) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (c0 + i < NB) {
            int64_t orow;
            float sa;
            cols.get(c0 + i, orow, sa);
            if (!failed && n < args.N && c0 + i < Mb) skinny_store(args, b, orow, n, sa, sb, r[i]);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c0 + i < NB) red[(c0 + i) * kSkinnyRows + ch] = r[i];
      }
    }
    tc_fence_before();
  }

  if (S > 1) {
    cluster_sync_all();  // every CTA's partials are in its shared memory
    if (warp >= 2) {
      // ---------------------------------------------------------- epilogue, part 2
      const int ch = (warp & 3) * 32 + lane;
      const int n = n0 + ch;
      const float sb = (b != kFP16 && args.out_mode != 1 && n < args.N) ? __ldg(args.sb + n) : 1.f;
      SkinnyCols<NB> cols;
      cols.load(args, b, pos0, Mb, lane);
      const uint32_t red_base = smem_u32(red);
      // four of this CTA's columns at a time, every rank's partial of them in flight at once
      for (int c0 = static_cast<int>(rank); c0 < Mb; c0 += 4 * static_cast<int>(S)) {
        uint32_t v[4][kSkinnyMaxSplits];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + u * static_cast<int>(S);
          const uint32_t addr = red_base + static_cast<uint32_t>((c * kSkinnyRows + ch) * 4);
#pragma unroll
          for (int q = 0; q < kSkinnyMaxSplits; ++q)
            v[u][q] = (c < Mb && q < static_cast<int>(S)) ? ld_shared_cluster_u32(map_to_cta(addr, q)) : 0u;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + u * static_cast<int>(S);
          uint32_t sum_i = 0;
          float sum_f = 0.f;
#pragma unroll
          for (int q = 0; q < kSkinnyMaxSplits; ++q) {
            if (q < static_cast<int>(S)) {
              if (b == kINT8)
                sum_i += v[u][q];  // int32 partials: exact in any order
              else
                sum_f += __uint_as_float(v[u][q]);  // rank order
            }
          }
          int64_t orow;
          float sa;
          cols.get(c, orow, sa);  // the whole warp: c is the same in every lane
          if (c < Mb && n < args.N && *abort_flag == 0)
            skinny_store(args, b, orow, n, sa, sb, b == kINT8 ? sum_i : __float_as_uint(sum_f));
        }
      }
    }
    cluster_sync_all();  // no CTA leaves while a peer may still read its partials
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace ee
