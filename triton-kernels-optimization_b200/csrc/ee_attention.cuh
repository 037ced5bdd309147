// ee_attention.cuh - causal flash attention with the online entropy of every query row,
// on tcgen05: the router input of the Llama block without materialising the
// [B, H, S, S] probabilities (the reference's transformers attention returns them and
// computes -sum p log(p + 1e-10) in torch, EE/python/dispatch.py:236-245).
//
// Persistent: one CTA per SM (its 165 / 231 KB of shared memory), 384 threads, taking work
// units of (batch, query head, 256 query rows = two 128-row query tiles) longest causal
// unit first; every barrier's phase runs on across the units, the next unit's Q loads as
// soon as both issuers' last S MMAs of the current unit completed, and the first P V of a
// unit (which overwrites O) waits until the previous unit's O is read out, so a unit's
// loads and first scores overlap the previous unit's last tiles and output.  Roles:
//   warp 0     TMA producer: both Q tiles once, then K and V^T tiles of 128 keys into
//              rings (K 2 deep; V 2 deep at head_dim 64, 1 at 128);
//   warps 1-2  UMMA issuers, one thread each, warp 1 + w for query tile w (warp 1 also owns
//              TMEM): S_w = Q_w K_j^T (M 128, N KT) into the S buffer of tile w, O_w +=
//              P_w V_j (M 128, N d) into its O accumulator, in the order S_w,0 |
//              S_w,j+1 P_w V_j | ...: the next S is issued as soon as the softmax holds
//              the current one in registers, so it runs under that softmax's
//              exponentials, and neither tile's issue waits on the other's softmax.
//              Each issuer commits its share of every K / V stage's release (the empty
//              barriers count two), tile 0's issuer also for the key tiles past its
//              causal reach;
//   warp 3     idle (it completes the producer warpgroup, which hands its registers to
//              the softmax warpgroups);
//   warps 4-11 warpgroup w = query tile w, one whole row per thread: scores from TMEM into
//              registers with the reference's fp16 roundings (fp16 Q K^T, times the scale,
//              fp16), causal / length mask, row max; the reference point m of the
//              exponentials moves only when the max outgrows it by more than 2^8, and
//              then O_w is rescaled once in TMEM (tcgen05.ld / st) with l and t; P =
//              2^(x log2 e - m) as fp16 into shared memory in the UMMA SW128 K-major
//              layout; at the end O_w / l and H = ln(l) - t / l.
// No barrier couples the two warpgroups.  V is consumed transposed (V^T [d, keys] per
// head, written by transpose_v_kernel) so both UMMA operands of P V are K-major.  Every
// wait is bounded (2 s); on expiry the CTA records an error word, drains its own MMAs and
// TMA loads, frees TMEM and exits.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "ee_gemm.cuh"  // the device error word shared by every kernel of the library
#include "ee_internal.h"
#include "ee_ptx.cuh"

namespace ee {

constexpr int kAttnThreads = 384;  // producer warpgroup (TMA, MMA, two idle warps), two softmax warpgroups
// registers per thread: 168 at launch (384 threads, one CTA per SM); the producer
// warpgroup gives its share to the softmax warpgroups (104 + 2 x 200 <= 3 x 168)
constexpr int kAttnLaunchRegs = 168;
constexpr int kAttnProducerRegs = 104;
constexpr int kAttnSoftmaxRegs = 200;
static_assert(kAttnProducerRegs + 2 * kAttnSoftmaxRegs <= 3 * kAttnLaunchRegs, "register split above the launch budget");
constexpr int kAttnTileBytes = kAttnTile * 128;  // one 128-byte-wide swizzled box of 128 rows: 16 KB

template <int D>
struct AttnCfg {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  // keys per K / V tile: 128 for both head dims (a tcgen05.mma costs about the same
  // whatever its N, so the S MMA is made as wide as TMEM allows: 2 x (128 S + D O) columns)
  static constexpr int KT = 128;
  static constexpr int kKBlocks = D / 64;                      // 128-byte column blocks of Q / K rows
  static constexpr int kVBlocks = KT / 64;                     // 128-byte column blocks of V^T rows (keys)
  static constexpr int kQTileBytes = kKBlocks * kAttnTileBytes;  // one 128-row Q tile
  static constexpr int kKBytes = kKBlocks * KT * 128;          // one K tile: KT rows x D
  static constexpr int kVBytes = kVBlocks * D * 128;           // one V^T tile: D rows x KT keys
  static constexpr int kPBytes = kVBlocks * kAttnTileBytes;    // one P tile: 128 rows x KT keys
  // ring depths: K 2, V 2 at head_dim 64; K 2, V 1 at 128 (shared memory: 230.7 KB)
  static constexpr int kKStages = 2;
  static constexpr int kVStages = D == 64 ? 2 : 1;
  static constexpr int kBarrierBytes = 256;
  static constexpr size_t kSmem = 1024 + 2 * size_t(kQTileBytes) + kKStages * size_t(kKBytes) +
                                  kVStages * size_t(kVBytes) + 2 * size_t(kPBytes) + kBarrierBytes;
  static_assert(kSmem <= 227 * 1024, "attention shared memory above the 227 KB per-CTA limit");
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kTmemS = 0;        // S of warpgroup w: columns [w KT, (w + 1) KT)
  static constexpr uint32_t kTmemO = 2 * KT;   // O of warpgroup w: columns [2 KT + w D, 2 KT + (w + 1) D)
  static_assert(2 * KT + 2 * D <= 512, "TMEM columns");
};

struct AttnArgs {
  int64_t B, Hq, Hkv, S, S_pad;  // S_pad: V^T row length (keys), a multiple of 64
  float scale;                   // softmax scale (head_dim^-0.5)
  int causal;
  __half* O;                     // [B, S, Hq, D]
  float* H;                      // [B, Hq, S] entropy of each query row (nats)
  float2* ml;                    // nullable [B, Hq, S]: each row's exponent reference m (base 2) and
                                 // l = sum 2^(x log2 e - m), for attention_entropy_exact_kernel
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr unsigned short kHalfLowest = 0xFBFFu;  // -65504

// fp16 pair {lo, hi} (lo in the low half), both rounded to nearest
__device__ __forceinline__ uint32_t pack_half2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// fp16(fp32(fp16(s)) * scale) for two raw fp32 scores when the scale is an fp16 number
// (head_dim 64: 1/8): the fp32 product of two
// fp16 numbers is exact, so its fp16 rounding is the correctly rounded fp16 product --
// one mul.rn.f16x2 (no flush to zero: fp16 subnormals round as in the fp32 path)
__device__ __forceinline__ __half2 scaled_scores_f16(uint32_t s0, uint32_t s1, uint32_t sch2) {
  const uint32_t h = pack_half2_rn(__uint_as_float(s0), __uint_as_float(s1));
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(sch2));
  return *reinterpret_cast<const __half2*>(&r);
}

// fp16(fp32(fp16(s)) * scale) for two raw fp32 scores: the rounding of an fp16 matmul
// output, then the fp16 tensor times a Python float (computed in fp32, rounded to fp16)
__device__ __forceinline__ __half2 scaled_scores(uint32_t s0, uint32_t s1, float2 sc2) {
  const uint32_t h = pack_half2_rn(__uint_as_float(s0), __uint_as_float(s1));
  const float2 x = __fmul2_rn(__half22float2(*reinterpret_cast<const __half2*>(&h)), sc2);
  const uint32_t r = pack_half2_rn(x.x, x.y);
  return *reinterpret_cast<const __half2*>(&r);
}

// byte offset of element (row, col) of a [128 rows x 128 fp16] tile stored as two
// SW128 K-major boxes (cols 0..63, then 64..127): 16-byte chunk index XOR row % 8
__device__ __forceinline__ uint32_t p_offset(int row, int col) {
  return static_cast<uint32_t>((col >> 6) * kAttnTileBytes + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) +
                               ((col & 7) << 1));
}

// The work unit t of a launch: (batch, query head, 256 query rows), longest causal units
// first over the whole grid (all (batch, head) pairs of the last query chunk, then the
// chunk before, ...).  The CTAs deal the units in rounds of gridDim.x, in "snake" order:
// round r gives unit r * gridDim.x + p to CTA p in even rounds and to CTA gridDim.x - 1 - p
// in odd ones, which evens out the CTAs' sums of unit lengths (within ~1-2 % of greedy
// longest-first dealing on the bench's shapes, against 6-14 % for plain round robin).
__device__ __forceinline__ int64_t attn_unit_index(int64_t r, int64_t nunits) {
  const int64_t p = (r & 1) ? static_cast<int64_t>(gridDim.x - 1 - blockIdx.x) : static_cast<int64_t>(blockIdx.x);
  const int64_t t = r * gridDim.x + p;
  return t < nunits ? t : -1;
}
struct AttnUnit {
  int64_t b, h, bh, q0;
  int nkv0, nkv1;               // key tiles query tile 0 / 1 sees
  int q_row0, k_row0, v_row0;   // rows in Q [B*Hq*S, D], K [B*Hkv*S, D], V^T [B*Hkv*D, S_pad]
};
template <int D>
__device__ __forceinline__ AttnUnit attn_unit(const AttnArgs& args, int64_t t) {
  constexpr int KT = AttnCfg<D>::KT;
  const int64_t nqc = (args.S + 2 * kAttnTile - 1) / (2 * kAttnTile);
  const int64_t nbh = args.B * args.Hq;
  AttnUnit u;
  const int64_t qc = nqc - 1 - t / nbh;
  u.bh = t % nbh;
  u.b = u.bh / args.Hq;
  u.h = u.bh % args.Hq;
  const int64_t hk = u.h / (args.Hq / args.Hkv);
  u.q0 = qc * 2 * kAttnTile;
  const int nkv_all = static_cast<int>((args.S + KT - 1) / KT);
  const int reach0 = static_cast<int>((u.q0 + kAttnTile + KT - 1) / KT);
  const int reach1 = static_cast<int>((u.q0 + 2 * kAttnTile + KT - 1) / KT);
  u.nkv0 = args.causal ? (reach0 < nkv_all ? reach0 : nkv_all) : nkv_all;
  u.nkv1 = args.causal ? (reach1 < nkv_all ? reach1 : nkv_all) : nkv_all;
  u.q_row0 = static_cast<int>(u.bh * args.S + u.q0);
  u.k_row0 = static_cast<int>((u.b * args.Hkv + hk) * args.S);
  u.v_row0 = static_cast<int>((u.b * args.Hkv + hk) * D);
  return u;
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
    flash_attention_entropy_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                                   const __grid_constant__ CUtensorMap tm_vt, const AttnArgs args) {
  using Cfg = AttnCfg<D>;
  constexpr int KT = Cfg::KT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // [2 query tiles]
  uint8_t* sK = sQ + 2 * Cfg::kQTileBytes;              // [kKStages]
  uint8_t* sV = sK + Cfg::kKStages * Cfg::kKBytes;      // [kVStages]
  uint8_t* sP = sV + Cfg::kVStages * Cfg::kVBytes;      // [2 warpgroups]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * Cfg::kPBytes);
  uint64_t* q_full = bars;
  constexpr int NS = Cfg::kKStages, NV = Cfg::kVStages;
  uint64_t* k_full = bars + 1;                 // [kKStages]
  uint64_t* k_empty = bars + 1 + NS;           // [kKStages]
  uint64_t* v_full = bars + 1 + 2 * NS;        // [kVStages]
  uint64_t* v_empty = bars + 1 + 2 * NS + NV;  // [kVStages]
  uint64_t* s_full = bars + 1 + 2 * NS + 2 * NV;  // [2 warpgroups] S_w ready (MMA commit)
  uint64_t* s_free = s_full + 2;          // [2] S_w read into registers (4 warps)
  uint64_t* p_full = s_full + 4;          // [2] P_w written, O_w corrected (4 warps)
  uint64_t* o_done = s_full + 6;          // [2] P_w V done: P_w free, O_w stable (MMA commit)
  uint64_t* drain = s_full + 8;           // [2] MMA drain on abort, one per issuing thread
  uint64_t* q_empty = s_full + 10;        // both issuers' S MMAs of a unit done: Q may reload
  uint64_t* o_free = s_full + 11;         // [2] O_w of the finished unit read out (4 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 13);
  static_assert((1 + 2 * NS + 2 * NV + 13) * 8 + 8 <= Cfg::kBarrierBytes, "attention barrier region overflows");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nunits = args.B * args.Hq * ((args.S + 2 * kAttnTile - 1) / (2 * kAttnTile));

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 2);  // one commit per issuing thread
    for (int i = 0; i < NS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 2);  // one commit per issuing thread
    }
    for (int i = 0; i < NV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);  // the four warps of the warpgroup
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 4);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_vt);
  }
  griddep_wait();  // Q, K, V^T may come from the previous kernel in the stream
  if (warp == 1) {  // after the wait: a kernel still draining before this one may hold TMEM
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // the register budgets change inside each role's branch: code after a join would be
  // compiled for the smaller budget
  if (warp < 4) {
  warpgroup_reg_dealloc<kAttnProducerRegs>();
  if (warp == 0) {
    // -------------------------------------------------------------- TMA producer
    bool failed = false;
    uint32_t k_issued = 0, v_issued = 0;  // bit s: stage s has received a load (for the abort drain)
    uint32_t k_par = 0, v_par = 0;        // bit s: phase parity of stage s's last load
    uint32_t kt = 0, vt = 0;              // K / V tiles loaded so far (all units)
    int q_loads = 0;                      // Q loads issued (one per unit)
    int64_t t;
    for (int64_t r = 0; !failed && (t = attn_unit_index(r, nunits)) >= 0; ++r) {
      const AttnUnit un = attn_unit<D>(args, t);
      const int nkv_max = un.nkv1;
      // Q of this unit, once both issuers' S MMAs of the previous unit have read the old Q
      if (q_loads > 0 && !mbar_wait_warp(q_empty, static_cast<uint32_t>(q_loads - 1) & 1u, abort_flag)) {
        failed = true;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full, 2 * Cfg::kQTileBytes);
        for (int q = 0; q < 2; ++q)
          for (int kb = 0; kb < Cfg::kKBlocks; ++kb)
            tma_load_2d(sQ + q * Cfg::kQTileBytes + kb * kAttnTileBytes, &tm_q, q_full, kb * 64, un.q_row0 + q * kAttnTile);
      }
      ++q_loads;
      __syncwarp();
      // K runs one tile ahead of V: S_{j+1} is issued (as soon as the softmax holds S_j)
      // before P V_j (once P_j is written)
      auto load_k = [&](int j) -> bool {
        const int s = kt % NS;
        const uint32_t ph = (kt / NS) & 1u;
        if (!mbar_wait_warp(&k_empty[s], ph ^ 1u, abort_flag)) return false;
        if (lane == 0) {
          mbar_arrive_expect_tx(&k_full[s], Cfg::kKBytes);
          for (int kb = 0; kb < Cfg::kKBlocks; ++kb)
            tma_load_2d(sK + s * Cfg::kKBytes + kb * (KT * 128), &tm_k, &k_full[s], kb * 64, un.k_row0 + j * KT);
        }
        k_issued |= 1u << s;
        k_par = (k_par & ~(1u << s)) | (ph << s);
        ++kt;
        __syncwarp();
        return true;
      };
      auto load_v = [&](int j) -> bool {
        const int sv = vt % NV;
        const uint32_t phv = (vt / NV) & 1u;
        if (!mbar_wait_warp(&v_empty[sv], phv ^ 1u, abort_flag)) return false;
        if (lane == 0) {
          mbar_arrive_expect_tx(&v_full[sv], Cfg::kVBytes);
          for (int vb = 0; vb < Cfg::kVBlocks; ++vb)
            tma_load_2d(sV + sv * Cfg::kVBytes + vb * (D * 128), &tm_vt, &v_full[sv], j * KT + vb * 64, un.v_row0);
        }
        v_issued |= 1u << sv;
        v_par = (v_par & ~(1u << sv)) | (phv << sv);
        ++vt;
        __syncwarp();
        return true;
      };
      if (!load_k(0)) {
        failed = true;
        break;
      }
      for (int j = 0; j < nkv_max; ++j) {
        if (j + 1 < nkv_max && !load_k(j + 1)) {
          failed = true;
          break;
        }
        if (!load_v(j)) {
          failed = true;
          break;
        }
      }
    }
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
      // let the loads already issued land before the CTA can exit (bounded, no abort)
      if (q_loads > 0) (void)mbar_wait(q_full, static_cast<uint32_t>(q_loads - 1) & 1u, nullptr);
      for (int s = 0; s < NS; ++s)
        if (k_issued & (1u << s)) (void)mbar_wait(&k_full[s], (k_par >> s) & 1u, nullptr);
      for (int s = 0; s < NV; ++s)
        if (v_issued & (1u << s)) (void)mbar_wait(&v_full[s], (v_par >> s) & 1u, nullptr);
    }
  } else if (warp == 1 || warp == 2) {
    // -------------------------------------------------------------- UMMA issuers
    // One thread per query tile w = warp - 1.  Per unit: S_w,0, then per key tile j:
    // S_w,j+1, P_w V_j -- the tensor core works for one warpgroup while the other one runs
    // its softmax.  For the key tiles past its causal reach it still takes part in the K /
    // V rings (waits for the stage, commits its share of the release).  Counters run over
    // all units of the CTA: kt / vt the K / V tiles, g the tiles of query tile w.
    constexpr uint32_t idesc_s = make_idesc(1u, 0u, kAttnTile, KT);  // f32 <- f16 x f16, 128 x KT
    constexpr uint32_t idesc_o = make_idesc(1u, 0u, kAttnTile, D);   // f32 <- f16 x f16, 128 x D
    const int w = warp - 1;
    bool failed = false;
    uint32_t kt = 0, vt = 0, g = 0;
    int units = 0;
    auto issue_s = [&](uint32_t kidx, uint32_t gidx) -> bool {
      const int s = kidx % NS;
      if (!mbar_wait(&k_full[s], (kidx / NS) & 1u, abort_flag) ||
          !mbar_wait(&s_free[w], (gidx & 1u) ^ 1u, abort_flag))
        return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t dst = tmem_base + Cfg::kTmemS + w * KT;
        for (int kb = 0; kb < Cfg::kKBlocks; ++kb) {
          const uint64_t da = sdesc_k_sw128(smem_u32(sQ + w * Cfg::kQTileBytes + kb * kAttnTileBytes));
          const uint64_t db = sdesc_k_sw128(smem_u32(sK + s * Cfg::kKBytes + kb * (KT * 128)));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma<kKindF16>(dst, da + 2u * k, db + 2u * k, idesc_s, (kb == 0 && k == 0) ? 0u : 1u);
        }
        tc_commit(&s_full[w]);
      }
      __syncwarp();
      return true;
    };
    auto issue_pv = [&](uint32_t vidx, uint32_t gidx, bool first) -> bool {
      const int s = vidx % NV;
      if (!mbar_wait(&v_full[s], (vidx / NV) & 1u, abort_flag) ||
          !mbar_wait(&p_full[w], gidx & 1u, abort_flag))
        return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t dst = tmem_base + Cfg::kTmemO + w * D;
        for (int vb = 0; vb < Cfg::kVBlocks; ++vb) {
          const uint64_t da = sdesc_k_sw128(smem_u32(sP + w * Cfg::kPBytes + vb * kAttnTileBytes));
          const uint64_t db = sdesc_k_sw128(smem_u32(sV + s * Cfg::kVBytes + vb * (D * 128)));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma<kKindF16>(dst, da + 2u * k, db + 2u * k, idesc_o, (first && vb == 0 && k == 0) ? 0u : 1u);
        }
        tc_commit(&o_done[w]);
      }
      __syncwarp();
      return true;
    };
    int64_t t;
    for (int64_t r = 0; !failed && (t = attn_unit_index(r, nunits)) >= 0; ++r, ++units) {
      const AttnUnit un = attn_unit<D>(args, t);
      const int nkv_w = w == 0 ? un.nkv0 : un.nkv1;
      const int nkv_max = un.nkv1;
      if (!mbar_wait(q_full, static_cast<uint32_t>(units) & 1u, abort_flag)) {
        failed = true;
        break;
      }
      tc_fence_after();
      // after this thread's last S of the unit, the Q tiles may reload (when it completes)
      auto q_release = [&](int j) {
        if (j == nkv_w - 1) {
          if (lane == 0) tc_commit(q_empty);
          __syncwarp();
        }
      };
      if (!issue_s(kt, g)) {
        failed = true;
        break;
      }
      q_release(0);
      if (lane == 0) tc_commit(&k_empty[kt % NS]);
      __syncwarp();
      for (int j = 0; j < nkv_max && !failed; ++j) {
        if (j + 1 < nkv_max) {
          const uint32_t kn = kt + j + 1;
          if (j + 1 < nkv_w) {
            if (!issue_s(kn, g + j + 1)) failed = true;
            if (!failed) q_release(j + 1);
          } else if (!mbar_wait(&k_full[kn % NS], (kn / NS) & 1u, abort_flag)) {
            failed = true;
          }
          if (!failed && lane == 0) tc_commit(&k_empty[kn % NS]);
          __syncwarp();
        }
        if (!failed) {
          if (j < nkv_w) {
            // the unit's first P V overwrites O_w: the previous unit's O_w must be read out
            if (j == 0 && units > 0 && !mbar_wait(&o_free[w], static_cast<uint32_t>(units - 1) & 1u, abort_flag))
              failed = true;
            if (!failed && !issue_pv(vt + j, g + j, j == 0)) failed = true;
          } else if (!mbar_wait(&v_full[(vt + j) % NV], ((vt + j) / NV) & 1u, abort_flag)) {
            failed = true;
          }
        }
        if (!failed && lane == 0) tc_commit(&v_empty[(vt + j) % NV]);
        __syncwarp();
      }
      kt += nkv_max;
      vt += nkv_max;
      g += nkv_w;
    }
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
        tc_commit(&drain[w]);
      }
      __syncwarp();
      (void)mbar_wait(&drain[w], 0u, nullptr);
    }
  }  // warp 3: nothing to do
  } else {
    warpgroup_reg_alloc<kAttnSoftmaxRegs>();
    // -------------------------------------------------------------- softmax / entropy / output
    // Warpgroup w owns query tile w of the CTA: thread (quarter, lane) one whole row,
    // row = quarter * 32 + lane (its TMEM lane).  Per key tile: scores from TMEM into
    // registers with the reference's fp16 roundings, causal / length mask, the row max;
    // the reference point m of the exponentials moves only when the max grows by more
    // than 2^8 (then O_w in TMEM, l and t are rescaled once), so most tiles touch O not at
    // all; P = 2^(x log2 e - m) as fp16 into shared memory for the P V UMMA.
    const int w = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem_base + Cfg::kTmemS + w * KT + lane_off;
    const uint32_t t_o = tmem_base + Cfg::kTmemO + w * D + lane_off;
    constexpr float kLog2eF = 1.4426950408889634f;
    constexpr float kRescale = 8.f;  // log2 of the largest p allowed before m moves
    const float2 sc2 = make_float2(args.scale, args.scale);
    const __half sch = __float2half_rn(args.scale);
    const bool scale_is_f16 = __half2float(sch) == args.scale;  // uniform for the kernel
    const uint32_t sch2 = static_cast<uint32_t>(__half_as_ushort(sch)) * 0x10001u;
    uint8_t* pbuf = sP + w * Cfg::kPBytes;
    bool failed = false;
    uint32_t gbase = 0;  // this query tile's key tiles of the earlier units (all barrier phases count them)
    int64_t tu;
    for (int64_t r = 0; !failed && (tu = attn_unit_index(r, nunits)) >= 0; ++r) {
    const AttnUnit un = attn_unit<D>(args, tu);
    const int nkv_w = w == 0 ? un.nkv0 : un.nkv1;
    const int64_t q = un.q0 + w * kAttnTile + row;
    const int64_t b = un.b, h = un.h, bh = un.bh;
    float m2 = -__builtin_huge_valf(), l = 0.f, t2 = 0.f;
    for (int j = 0; j < nkv_w; ++j) {
      const uint32_t gj = gbase + static_cast<uint32_t>(j);
      if (!mbar_wait_warp(&s_full[w], gj & 1u, abort_flag)) {
        failed = true;
        break;
      }
      tc_fence_after();
      const int key0 = j * KT;
      int lim = static_cast<int>(args.S - key0);  // keys this row may see: sequence end, causal limit
      if (args.causal) {
        const int64_t c = q - key0 + 1;
        lim = c < lim ? static_cast<int>(c) : lim;
      }
      lim = lim < 0 ? 0 : (lim > KT ? KT : lim);
      // the reference's fp16 scores: fp16 Q K^T, times the scale in fp32, fp16; keys
      // outside the limit get -65504 (the fp16 lowest the reference's additive mask
      // drives them to), whose probability is exactly 0
      __half2 xs[KT / 2];
#pragma unroll
      for (int c0 = 0; c0 < KT; c0 += 64) {  // two TMEM loads in flight per wait
        uint32_t ra[32], rb[32];
        __syncwarp();
        tmem_ld32(t_s + c0, ra);
        tmem_ld32(t_s + c0 + 32, rb);
        tmem_ld_wait(ra);
        regs_after_wait(rb);
        if (scale_is_f16) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            xs[c0 / 2 + i] = scaled_scores_f16(ra[2 * i], ra[2 * i + 1], sch2);
            xs[c0 / 2 + 16 + i] = scaled_scores_f16(rb[2 * i], rb[2 * i + 1], sch2);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            xs[c0 / 2 + i] = scaled_scores(ra[2 * i], ra[2 * i + 1], sc2);
            xs[c0 / 2 + 16 + i] = scaled_scores(rb[2 * i], rb[2 * i + 1], sc2);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[w]);  // S_w is in registers: the next S may land
      if (!__all_sync(0xffffffffu, lim >= KT)) {
        const __half neg = __ushort_as_half(kHalfLowest);
#pragma unroll
        for (int i = 0; i < KT / 2; ++i)
          xs[i] = __halves2half2(2 * i < lim ? __low2half(xs[i]) : neg, 2 * i + 1 < lim ? __high2half(xs[i]) : neg);
      }
      __half2 mx[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) mx[k] = xs[k];
#pragma unroll
      for (int i = 4; i < KT / 2; ++i) mx[i & 3] = __hmax2(mx[i & 3], xs[i]);
      const __half2 mxx = __hmax2(__hmax2(mx[0], mx[1]), __hmax2(mx[2], mx[3]));
      const float mt = fmaxf(__low2float(mxx), __high2float(mxx)) * kLog2eF;
      // the reference point: set by the first tile, moved when the max outgrows it by 2^8
      float alpha = 1.f;
      const float m_old = m2;
      if (j == 0) {
        m2 = mt;
      } else if (mt > m2 + kRescale) {
        alpha = ex2f(m2 - mt);
        m2 = mt;
      }
      const bool rescale = __any_sync(0xffffffffu, alpha != 1.f);
      if (j > 0) {
        // P_w V_{j-1} done: P_w may be rewritten and O_w is stable
        if (!mbar_wait_warp(&o_done[w], (gj - 1u) & 1u, abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
      }
      if (rescale) {
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld32(t_o + c0, r);
          tmem_ld_wait(r);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(t_o + c0, r);
        }
        tmem_st_wait();
        t2 = alpha * (t2 + l * (m_old - m2));
        l = alpha * l;
      }
      // p = 2^(x log2 e - m): masked keys give 2^(-94500 - m) = 0 and p (x - m) = 0
      float2 sp2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      float2 spt2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 lg2 = make_float2(kLog2eF, kLog2eF), negm = make_float2(-m2, -m2);
#pragma unroll
      for (int g = 0; g < KT / 8; ++g) {
        uint4 pk;
        uint32_t* wv = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 d2 = __ffma2_rn(__half22float2(xs[g * 4 + k]), lg2, negm);
          const float2 p = make_float2(ex2f(d2.x), ex2f(d2.y));
          sp2[k & 1] = __fadd2_rn(sp2[k & 1], p);
          spt2[k & 1] = __ffma2_rn(p, d2, spt2[k & 1]);
          wv[k] = pack_half2_rn(p.x, p.y);
        }
        *reinterpret_cast<uint4*>(pbuf + p_offset(row, g * 8)) = pk;
      }
      fence_proxy_async_smem();  // the P stores (and O's TMEM stores), visible to the tensor core
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[w]);
      // running statistics (base 2, relative to m): l = sum p, t2 = sum p (x - m)
      l += (sp2[0].x + sp2[0].y) + (sp2[1].x + sp2[1].y);
      t2 += (spt2[0].x + spt2[0].y) + (spt2[1].x + spt2[1].y);
    }
    if (!failed && !mbar_wait_warp(&o_done[w], (gbase + static_cast<uint32_t>(nkv_w) - 1u) & 1u, abort_flag))
      failed = true;
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
    } else {
      tc_fence_after();
      const float inv = 1.f / l;
      const bool store = q < args.S;
      __half* out = args.O + ((b * args.S + (store ? q : 0)) * args.Hq + h) * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld32(t_o + c0, r);
        tmem_ld_wait(r);
        if (store) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 pk;
            uint32_t* wv = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              wv[k] = pack_half2_rn(__uint_as_float(r[g * 8 + 2 * k]) * inv, __uint_as_float(r[g * 8 + 2 * k + 1]) * inv);
            *reinterpret_cast<uint4*>(out + c0 + g * 8) = pk;
          }
        }
      }
      if (store) args.H[bh * args.S + q] = 0.69314718055994531f * (__log2f(l) - t2 / l);
      if (store && args.ml != nullptr) args.ml[bh * args.S + q] = make_float2(m2, l);
      // O_w is read out: the next unit's first P V may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[w]);
    }
    gbase += static_cast<uint32_t>(nkv_w);
    }
    tc_fence_before();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

// ---------------------------------------------------------------------------------
// The reference's rounding of the probabilities, as a second pass over the keys.
//
// The reference takes the entropy of transformers' fp16 probabilities,
// -sum_j p_j ln(p_j + 1e-10) with p_j = fp16(softmax_fp32(s)_j) (EE/python/dispatch.py:
// 243-245).  Rounding p_j to fp16 needs the row's normaliser, which the flash kernel
// has only after its last key tile, so exact agreement takes a second pass: with each
// row's exponent reference m and sum l from the first pass (AttnArgs::ml), this kernel
// recomputes the fp16 scores S = Q K^T on the tensor core (the same tcgen05 MMAs and
// roundings as the first pass, no P V), forms q_j = 2^(x_j log2 e - m) / l -- the fp32
// softmax --, rounds it to fp16 and adds p ln(p + 1e-10) in fp32 as the reference does.
// Persistent like the flash kernel: one CTA per SM, 384 threads, taking the units
// (batch, query head, two 128-row query tiles) longest first in snake order:
//   warp 0     TMA producer: both Q tiles of a unit (once the unit before has issued its
//              last S MMA), K tiles of 128 keys into a 3-deep ring running across units;
//   warp 1     TMEM owner + single-thread UMMA issuer: S_w,j into one of two TMEM buffers
//              of query tile w (S of tile j + 1 is issued while tile j is reduced);
//   warps 4-11 warpgroup w = query tile w, one row per thread.
// Every wait is bounded; on expiry the CTA records the error word, drains and exits.
// ---------------------------------------------------------------------------------
template <int D>
struct ExactCfg {
  static constexpr int KT = 128;
  static constexpr int kKBlocks = D / 64;
  static constexpr int kQTileBytes = kKBlocks * kAttnTileBytes;
  static constexpr int kKBytes = kKBlocks * KT * 128;
  static constexpr int kKStages = 3;
  static constexpr int kBarrierBytes = 256;
  static constexpr size_t kSmem = 1024 + 2 * size_t(kQTileBytes) + kKStages * size_t(kKBytes) + kBarrierBytes;
  static_assert(kSmem <= 227 * 1024, "exact-entropy shared memory above the 227 KB per-CTA limit");
  static constexpr uint32_t kTmemCols = 512;  // 2 query tiles x 2 buffers x 128 key columns
};

__device__ __forceinline__ float lg2_approx_f(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_entropy_exact_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                                   const AttnArgs args) {
  using Cfg = ExactCfg<D>;
  constexpr int KT = Cfg::KT;
  constexpr int NS = Cfg::kKStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * Cfg::kQTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sK + NS * Cfg::kKBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;        // [NS]
  uint64_t* k_empty = bars + 1 + NS;  // [NS]
  uint64_t* s_full = bars + 1 + 2 * NS;  // [2 tiles][2 buffers] S ready (MMA commit)
  uint64_t* s_free = s_full + 4;         // [2][2] S read into registers (4 warps)
  uint64_t* drain = s_full + 8;
  uint64_t* q_empty = s_full + 9;  // the issuer's last S MMA of a unit done: Q may reload
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 10);
  static_assert((1 + 2 * NS + 10) * 8 + 8 <= Cfg::kBarrierBytes, "exact-entropy barrier region overflows");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  static_assert(Cfg::KT == AttnCfg<D>::KT, "the units of the flash kernel");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nunits = args.B * args.Hq * ((args.S + 2 * kAttnTile - 1) / (2 * kAttnTile));

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    mbar_init(drain, 1);
    mbar_init(q_empty, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
  }
  griddep_wait();  // Q, K and the first pass's row statistics come from earlier kernels
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // -------------------------------------------------------------- TMA producer
    bool failed = false;
    uint32_t k_issued = 0, k_par = 0, kt = 0;  // kt: K tiles loaded (all units)
    int q_loads = 0;
    int64_t t;
    for (int64_t r = 0; !failed && (t = attn_unit_index(r, nunits)) >= 0; ++r) {
      const AttnUnit un = attn_unit<D>(args, t);
      if (q_loads > 0 && !mbar_wait_warp(q_empty, static_cast<uint32_t>(q_loads - 1) & 1u, abort_flag)) {
        failed = true;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full, 2 * Cfg::kQTileBytes);
        for (int q = 0; q < 2; ++q)
          for (int kb = 0; kb < Cfg::kKBlocks; ++kb)
            tma_load_2d(sQ + q * Cfg::kQTileBytes + kb * kAttnTileBytes, &tm_q, q_full, kb * 64, un.q_row0 + q * kAttnTile);
      }
      ++q_loads;
      __syncwarp();
      for (int j = 0; j < un.nkv1; ++j, ++kt) {
        const int s = kt % NS;
        const uint32_t ph = (kt / NS) & 1u;
        if (!mbar_wait_warp(&k_empty[s], ph ^ 1u, abort_flag)) {
          failed = true;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&k_full[s], Cfg::kKBytes);
          for (int kb = 0; kb < Cfg::kKBlocks; ++kb)
            tma_load_2d(sK + s * Cfg::kKBytes + kb * (KT * 128), &tm_k, &k_full[s], kb * 64, un.k_row0 + j * KT);
        }
        k_issued |= 1u << s;
        k_par = (k_par & ~(1u << s)) | (ph << s);
        __syncwarp();
      }
    }
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
      if (q_loads > 0) (void)mbar_wait(q_full, static_cast<uint32_t>(q_loads - 1) & 1u, nullptr);
      for (int s = 0; s < NS; ++s)
        if (k_issued & (1u << s)) (void)mbar_wait(&k_full[s], (k_par >> s) & 1u, nullptr);
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- UMMA issuer
    // counters over all units of the CTA: kt the K tiles, g[w] the S tiles of query tile w
    // (its buffer g & 1, that buffer's use g >> 1)
    constexpr uint32_t idesc_s = make_idesc(1u, 0u, kAttnTile, KT);  // f32 <- f16 x f16, 128 x 128
    bool failed = false;
    uint32_t kt = 0, g[2] = {0u, 0u};
    int units = 0;
    int64_t t;
    for (int64_t r = 0; !failed && (t = attn_unit_index(r, nunits)) >= 0; ++r, ++units) {
    const AttnUnit un = attn_unit<D>(args, t);
    if (!mbar_wait(q_full, static_cast<uint32_t>(units) & 1u, abort_flag)) {
      failed = true;
      break;
    }
    tc_fence_after();
    for (int j = 0; j < un.nkv1 && !failed; ++j, ++kt) {
      const int s = kt % NS;
      if (!mbar_wait(&k_full[s], (kt / NS) & 1u, abort_flag)) {
        failed = true;
        break;
      }
      for (int w = 0; w < 2 && !failed; ++w) {
        if (j >= (w == 0 ? un.nkv0 : un.nkv1)) continue;
        const int buf = static_cast<int>(g[w] & 1u);
        const uint32_t use = g[w] >> 1;
        ++g[w];
        if (!mbar_wait(&s_free[2 * w + buf], (use & 1u) ^ 1u, abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t dst = tmem_base + static_cast<uint32_t>((2 * w + buf) * KT);
          for (int kb = 0; kb < Cfg::kKBlocks; ++kb) {
            const uint64_t da = sdesc_k_sw128(smem_u32(sQ + w * Cfg::kQTileBytes + kb * kAttnTileBytes));
            const uint64_t db = sdesc_k_sw128(smem_u32(sK + s * Cfg::kKBytes + kb * (KT * 128)));
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma<kKindF16>(dst, da + 2u * k, db + 2u * k, idesc_s, (kb == 0 && k == 0) ? 0u : 1u);
          }
          tc_commit(&s_full[2 * w + buf]);
        }
        __syncwarp();
      }
      if (!failed && lane == 0) tc_commit(&k_empty[s]);  // the stage is free once these MMAs are done
      __syncwarp();
    }
    // every S of the unit is issued: Q may reload once they complete
    if (!failed && lane == 0) tc_commit(q_empty);
    __syncwarp();
    }
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
        tc_commit(drain);
      }
      __syncwarp();
      (void)mbar_wait(drain, 0u, nullptr);
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- rows: the reference's entropy
    const int w = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    constexpr float kLog2eF = 1.4426950408889634f;
    const float2 sc2 = make_float2(args.scale, args.scale);
    const __half sch = __float2half_rn(args.scale);
    const bool scale_is_f16 = __half2float(sch) == args.scale;
    const uint32_t sch2 = static_cast<uint32_t>(__half_as_ushort(sch)) * 0x10001u;
    bool failed = false;
    uint32_t gbase = 0;  // this query tile's S tiles of the earlier units
    int64_t tu;
    for (int64_t r = 0; !failed && (tu = attn_unit_index(r, nunits)) >= 0; ++r) {
    const AttnUnit un = attn_unit<D>(args, tu);
    const int nkv_w = w == 0 ? un.nkv0 : un.nkv1;
    const int64_t q = un.q0 + w * kAttnTile + row;
    const int64_t bh = un.bh;
    const bool live = q < args.S;
    const float2 ml = live ? args.ml[bh * args.S + q] : make_float2(0.f, 1.f);
    const float inv_l = 1.f / ml.y;
    const float2 lg2 = make_float2(kLog2eF, kLog2eF), negm = make_float2(-ml.x, -ml.x);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < nkv_w; ++j) {
      const uint32_t gj = gbase + static_cast<uint32_t>(j);
      const int buf = static_cast<int>(gj & 1u);
      if (!mbar_wait_warp(&s_full[2 * w + buf], (gj >> 1) & 1u, abort_flag)) {
        failed = true;
        break;
      }
      tc_fence_after();
      const uint32_t t_s = tmem_base + static_cast<uint32_t>((2 * w + buf) * KT) + lane_off;
      const int key0 = j * KT;
      int lim = static_cast<int>(args.S - key0);
      if (args.causal) {
        const int64_t c = q - key0 + 1;
        lim = c < lim ? static_cast<int>(c) : lim;
      }
      lim = lim < 0 ? 0 : (lim > KT ? KT : lim);
      __half2 xs[KT / 2];
#pragma unroll
      for (int c0 = 0; c0 < KT; c0 += 64) {
        uint32_t ra[32], rb[32];
        __syncwarp();
        tmem_ld32(t_s + c0, ra);
        tmem_ld32(t_s + c0 + 32, rb);
        tmem_ld_wait(ra);
        regs_after_wait(rb);
        if (scale_is_f16) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            xs[c0 / 2 + i] = scaled_scores_f16(ra[2 * i], ra[2 * i + 1], sch2);
            xs[c0 / 2 + 16 + i] = scaled_scores_f16(rb[2 * i], rb[2 * i + 1], sch2);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            xs[c0 / 2 + i] = scaled_scores(ra[2 * i], ra[2 * i + 1], sc2);
            xs[c0 / 2 + 16 + i] = scaled_scores(rb[2 * i], rb[2 * i + 1], sc2);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[2 * w + buf]);  // the buffer may take S of tile j + 2
      if (!__all_sync(0xffffffffu, lim >= KT)) {
        const __half neg = __ushort_as_half(kHalfLowest);
#pragma unroll
        for (int i = 0; i < KT / 2; ++i)
          xs[i] = __halves2half2(2 * i < lim ? __low2half(xs[i]) : neg, 2 * i + 1 < lim ? __high2half(xs[i]) : neg);
      }
      // p = fp16(2^(x log2 e - m) / l): the reference's fp16 probability; then
      // p * log2(p + 1e-10) in fp32 (masked keys: p = 0 contributes 0)
#pragma unroll
      for (int i = 0; i < KT / 2; ++i) {
        const float2 d2 = __ffma2_rn(__half22float2(xs[i]), lg2, negm);
        const __half2 p16 = __floats2half2_rn(ex2f(d2.x) * inv_l, ex2f(d2.y) * inv_l);
        const float2 pf = __half22float2(p16);
        acc[(2 * i) & 3] = fmaf(pf.x, lg2_approx_f(pf.x + 1e-10f), acc[(2 * i) & 3]);
        acc[(2 * i + 1) & 3] = fmaf(pf.y, lg2_approx_f(pf.y + 1e-10f), acc[(2 * i + 1) & 3]);
      }
    }
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
    } else if (live) {
      args.H[bh * args.S + q] = -0.69314718055994531f * ((acc[0] + acc[1]) + (acc[2] + acc[3]));
    }
    gbase += static_cast<uint32_t>(nkv_w);
    }
    tc_fence_before();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace ee
