// ee_attention.cuh - causal flash attention with the online entropy of every query row,
// on tcgen05: the router input of the Llama block without materialising the
// [B, H, S, S] probabilities (the reference's transformers attention returns them and
// computes -sum p log(p + 1e-10) in torch, EE/python/dispatch.py:236-245).
//
// One CTA per (batch, query head, 128-query tile), 384 threads:
//   warp 0     TMA producer: Q once, then K and V^T tiles of 128 keys into 2-deep rings;
//   warp 1     TMEM owner + single-thread UMMA issuer: S_j = Q K_j^T (M 128, N 128) into
//              one of two 128-column TMEM buffers, O_j = P_j V_j (M 128, N d) into one of
//              two d-column buffers;
//   warps 2-3  idle (they complete the producer warpgroup, which hands its registers to
//              the softmax warpgroups);
//   warps 4-11 two warpgroups, one half row per thread (64 of the tile's 128 scores,
//              half of O's columns): scores from TMEM into registers with the
//              reference's fp16 roundings (fp16 Q K^T, times the scale, fp16), causal
//              mask, the row max shared with the other half through shared memory,
//              running sum and sum of p (x - max) in base 2, P = 2^(x - max) as fp16 into
//              shared memory in the UMMA SW128 K-major layout, then O += alpha * O_j from
//              TMEM in registers; at the end O / l and H = ln(l) - t / l.
// V is consumed transposed (V^T [d, keys] per head, written by transpose_v_kernel) so
// both UMMA operands of P V are K-major.  Every wait is bounded (2 s); on expiry the CTA
// records an error word, drains its own MMAs and TMA loads, frees TMEM and exits.
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
// warpgroup gives its share to the softmax warpgroups (96 + 2 x 200 <= 3 x 168)
constexpr int kAttnLaunchRegs = 168;
constexpr int kAttnProducerRegs = 96;
constexpr int kAttnSoftmaxRegs = 200;
static_assert(kAttnProducerRegs + 2 * kAttnSoftmaxRegs <= 3 * kAttnLaunchRegs, "register split above the launch budget");
constexpr int kAttnTileBytes = kAttnTile * 128;  // one 128-byte-wide swizzled box of 128 rows: 16 KB

template <int D>
struct AttnCfg {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static constexpr int kKBlocks = D / 64;                      // 128-byte column blocks of Q / K rows
  static constexpr int kQBytes = kKBlocks * kAttnTileBytes;    // Q tile
  static constexpr int kKBytes = kKBlocks * kAttnTileBytes;    // one K tile
  static constexpr int kVBytes = 2 * (D * 128);                // one V^T tile: D rows x 128 keys, 2 blocks
  static constexpr int kPBytes = 2 * kAttnTileBytes;           // one P tile: 128 rows x 128 keys
  static constexpr int kBarrierBytes = 256 + 2 * 128 * 4;  // barriers, then the row-max exchange
  static constexpr size_t kSmem = 1024 + size_t(kQBytes) + 2 * size_t(kKBytes) + 2 * size_t(kVBytes) +
                                  2 * size_t(kPBytes) + kBarrierBytes;
  static_assert(kSmem <= 227 * 1024, "attention shared memory above the 227 KB per-CTA limit");
  static constexpr uint32_t kTmemCols = 512;  // S: 2 x 128, O: 2 x D
};

struct AttnArgs {
  int64_t B, Hq, Hkv, S, S_pad;  // S_pad: V^T row length (keys), a multiple of 64
  float scale;                   // softmax scale (head_dim^-0.5)
  int causal;
  __half* O;                     // [B, S, Hq, D]
  float* H;                      // [B, Hq, S] entropy of each query row (nats)
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

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
    flash_attention_entropy_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                                   const __grid_constant__ CUtensorMap tm_vt, const AttnArgs args) {
  using Cfg = AttnCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Cfg::kQBytes;            // [2]
  uint8_t* sV = sK + 2 * Cfg::kKBytes;        // [2]
  uint8_t* sP = sV + 2 * Cfg::kVBytes;        // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * Cfg::kPBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* s_empty = bars + 11;  // [2]
  uint64_t* p_full = bars + 13;   // [2]
  uint64_t* p_empty = bars + 15;  // [2]
  uint64_t* o_full = bars + 17;   // [2]
  uint64_t* o_empty = bars + 19;  // [2]
  uint64_t* drain = bars + 21;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nqt = (args.S + kAttnTile - 1) / kAttnTile;
  const int qt = static_cast<int>(nqt - 1 - static_cast<int64_t>(blockIdx.x) % nqt);  // longest tiles first
  const int64_t bh = static_cast<int64_t>(blockIdx.x) / nqt;                           // b * Hq + h
  const int64_t b = bh / args.Hq, h = bh % args.Hq;
  const int64_t hk = h / (args.Hq / args.Hkv);
  const int nkv_all = static_cast<int>((args.S + kAttnTile - 1) / kAttnTile);
  const int nkv = args.causal ? (qt + 1 < nkv_all ? qt + 1 : nkv_all) : nkv_all;
  const int q_row0 = static_cast<int>(bh * args.S + static_cast<int64_t>(qt) * kAttnTile);  // row in Q [B*Hq*S, D]
  const int k_row0 = static_cast<int>((b * args.Hkv + hk) * args.S);                        // row in K [B*Hkv*S, D]
  const int v_row0 = static_cast<int>((b * args.Hkv + hk) * D);                             // row in V^T [B*Hkv*D, S_pad]

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 8);  // eight softmax warps
      mbar_init(&p_full[i], 8);
      mbar_init(&p_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_vt);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_wait();  // Q, K, V^T may come from the previous kernel in the stream
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_s = tmem_base;            // columns [0, 256): two S buffers
  const uint32_t tmem_o = tmem_base + 2 * 128;  // columns [256, 256 + 2 D): two O buffers
  // the register budgets change inside each role's branch: code after a join would be
  // compiled for the smaller budget
  if (warp < 4) {
  warpgroup_reg_dealloc<kAttnProducerRegs>();
  if (warp == 0) {
    // -------------------------------------------------------------- TMA producer
    bool failed = false;
    uint32_t k_issued = 0, v_issued = 0;  // bit i: slot i has received a load (for the abort drain)
    uint32_t k_par = 0, v_par = 0;        // bit i: phase parity of slot i's last load
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, Cfg::kQBytes);
      for (int kb = 0; kb < Cfg::kKBlocks; ++kb) tma_load_2d(sQ + kb * kAttnTileBytes, &tm_q, q_full, kb * 64, q_row0);
    }
    for (int j = 0; j < nkv && !failed; ++j) {
      const int s = j & 1;
      const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
      if (!mbar_wait(&k_empty[s], ph ^ 1u, abort_flag)) {
        failed = true;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&k_full[s], Cfg::kKBytes);
        for (int kb = 0; kb < Cfg::kKBlocks; ++kb)
          tma_load_2d(sK + s * Cfg::kKBytes + kb * kAttnTileBytes, &tm_k, &k_full[s], kb * 64, k_row0 + j * kAttnTile);
      }
      k_issued |= 1u << s;
      k_par = (k_par & ~(1u << s)) | (ph << s);
      if (!mbar_wait(&v_empty[s], ph ^ 1u, abort_flag)) {
        failed = true;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&v_full[s], Cfg::kVBytes);
        for (int kb = 0; kb < 2; ++kb)
          tma_load_2d(sV + s * Cfg::kVBytes + kb * (D * 128), &tm_vt, &v_full[s], j * kAttnTile + kb * 64, v_row0);
      }
      v_issued |= 1u << s;
      v_par = (v_par & ~(1u << s)) | (ph << s);
      __syncwarp();
    }
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
      // let the loads already issued land before the CTA can exit (bounded, no abort)
      (void)mbar_wait(q_full, 0u, nullptr);
      for (int s = 0; s < 2; ++s) {
        if (k_issued & (1u << s)) (void)mbar_wait(&k_full[s], (k_par >> s) & 1u, nullptr);
        if (v_issued & (1u << s)) (void)mbar_wait(&v_full[s], (v_par >> s) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- UMMA issuer
    constexpr uint32_t idesc_s = make_idesc(1u, 0u, kAttnTile, kAttnTile);  // f32 <- f16 x f16, 128 x 128
    constexpr uint32_t idesc_o = make_idesc(1u, 0u, kAttnTile, D);          // f32 <- f16 x f16, 128 x D
    bool failed = !mbar_wait(q_full, 0u, abort_flag);
    tc_fence_after();
    auto issue_s = [&](int j) -> bool {
      const int s = j & 1;
      const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
      if (!mbar_wait(&k_full[s], ph, abort_flag) || !mbar_wait<false>(&s_empty[s], ph ^ 1u, abort_flag)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t dst = tmem_s + s * 128;
        for (int kb = 0; kb < Cfg::kKBlocks; ++kb) {
          const uint64_t da = sdesc_k_sw128(smem_u32(sQ + kb * kAttnTileBytes));
          const uint64_t db = sdesc_k_sw128(smem_u32(sK + s * Cfg::kKBytes + kb * kAttnTileBytes));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma<kKindF16>(dst, da + 2u * k, db + 2u * k, idesc_s, (kb == 0 && k == 0) ? 0u : 1u);
        }
        tc_commit(&s_full[s]);
        tc_commit(&k_empty[s]);
      }
      __syncwarp();
      return true;
    };
    if (!failed) failed = !issue_s(0);
    if (!failed && nkv > 1) failed = !issue_s(1);
    for (int j = 0; j < nkv && !failed; ++j) {
      const int s = j & 1;
      const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
      if (!mbar_wait(&p_full[s], ph, abort_flag) || !mbar_wait(&v_full[s], ph, abort_flag) ||
          !mbar_wait(&o_empty[s], ph ^ 1u, abort_flag)) {
        failed = true;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t dst = tmem_o + s * D;
        for (int kb = 0; kb < 2; ++kb) {
          const uint64_t da = sdesc_k_sw128(smem_u32(sP + s * Cfg::kPBytes + kb * kAttnTileBytes));
          const uint64_t db = sdesc_k_sw128(smem_u32(sV + s * Cfg::kVBytes + kb * (D * 128)));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma<kKindF16>(dst, da + 2u * k, db + 2u * k, idesc_o, (kb == 0 && k == 0) ? 0u : 1u);
        }
        tc_commit(&o_full[s]);
        tc_commit(&p_empty[s]);
        tc_commit(&v_empty[s]);
      }
      __syncwarp();
      if (j + 2 < nkv && !issue_s(j + 2)) failed = true;
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
  }  // warps 2 and 3: nothing to do
  } else {
    warpgroup_reg_alloc<kAttnSoftmaxRegs>();
    // -------------------------------------------------------------- softmax / entropy / output
    // Two warpgroups: thread (half h, quarter q, lane) owns row q * 32 + lane, score
    // columns 64 h .. 64 h + 63 and output columns h * D / 2 ..; the row max is exchanged
    // through shared memory once per tile, the sums stay per half until the end.
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;
    const int row = quarter * 32 + lane;
    const int64_t q = static_cast<int64_t>(qt) * kAttnTile + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    constexpr float kLog2eF = 1.4426950408889634f;
    constexpr int kOH = D / 2;  // output columns per thread
    float* red = reinterpret_cast<float*>(bars + 32);  // [2 halves][128 rows]: row maxima, then sums
    float m2 = -__builtin_huge_valf(), l = 0.f, t2 = 0.f, alpha_prev = 0.f;
    float2 o[kOH / 2];  // output columns 2 i, 2 i + 1 of this thread's half
#pragma unroll
    for (int i = 0; i < kOH / 2; ++i) o[i] = make_float2(0.f, 0.f);
    bool failed = false;

    auto consume_o = [&](int j, float alpha) -> bool {
      const int s = j & 1;
      const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
      if (!mbar_wait_warp(&o_full[s], ph, abort_flag)) return false;
      tc_fence_after();
      const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
      for (int c = 0; c < kOH / 32; ++c) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld32(tmem_o + s * D + half * kOH + c * 32 + lane_off, r);
        tmem_ld_wait(r);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          o[c * 16 + i] = __ffma2_rn(o[c * 16 + i], a2, make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[s]);
      return true;
    };

    // Every softmax warp runs every iteration, failed or not: the named barriers below
    // need all eight warps each time (a warp that gave up skips only the work).
    for (int j = 0; j < nkv; ++j) {
      const int s = j & 1;
      const uint32_t ph = static_cast<uint32_t>(j >> 1) & 1u;
      if (!failed && !mbar_wait_warp(&s_full[s], ph, abort_flag)) failed = true;
      if (failed && lane == 0) *abort_flag = 1;  // every role of the CTA stops waiting
      const int key0 = j * kAttnTile + half * 64;
      // keys this thread may see: causal limit and the sequence end
      int lim = static_cast<int>(args.S - key0);
      if (args.causal) {
        const int64_t c = q - key0 + 1;
        lim = c < lim ? static_cast<int>(c) : lim;
      }
      lim = lim < 0 ? 0 : (lim > 64 ? 64 : lim);
      // the reference's fp16 scores: fp16 Q K^T, times the scale in fp32, fp16; a key
      // outside the causal / length limit gets -65504 (the fp16 lowest the reference's
      // additive mask drives it to), whose probability is exactly 0 -- two per register
      __half2 xs[32];
      __half2 mx2 = __half2half2(__ushort_as_half(kHalfLowest));
      if (!failed) {
        tc_fence_after();
        uint32_t ra[32], rb[32];
        __syncwarp();
        tmem_ld32(tmem_s + s * 128 + half * 64 + lane_off, ra);
        tmem_ld32(tmem_s + s * 128 + half * 64 + 32 + lane_off, rb);
        tmem_ld_wait(ra);
        regs_after_wait(rb);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[s]);  // the scores are in registers: S buffer free
        const float2 sc2 = make_float2(args.scale, args.scale);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          xs[i] = scaled_scores(ra[2 * i], ra[2 * i + 1], sc2);
          xs[16 + i] = scaled_scores(rb[2 * i], rb[2 * i + 1], sc2);
        }
        if (!__all_sync(0xffffffffu, lim >= 64)) {  // a tile on the diagonal or the sequence end
          const __half neg = __ushort_as_half(kHalfLowest);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            xs[i] = __halves2half2(2 * i < lim ? __low2half(xs[i]) : neg, 2 * i + 1 < lim ? __high2half(xs[i]) : neg);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) mx2 = __hmax2(mx2, xs[i]);
      }
      const float mx = fmaxf(__low2float(mx2), __high2float(mx2)) * kLog2eF;
      // exchange the half-row maxima (barrier 1: the eight softmax warps); the first
      // barrier keeps this tile's writes behind the partner's read of the previous tile
      asm volatile("bar.sync 1, 256;" ::: "memory");
      red[half * 128 + row] = mx;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      const float m_new = fmaxf(m2, fmaxf(mx, red[(half ^ 1) * 128 + row]));
      const float alpha = (m2 == -__builtin_huge_valf()) ? 0.f : ex2f(m2 - m_new);
      // P may overwrite buffer s once the P V of tile j - 2 has read it
      if (!failed && !mbar_wait_warp(&p_empty[s], ph ^ 1u, abort_flag)) failed = true;
      if (failed && lane == 0) *abort_flag = 1;
      if (!failed) {
        // p = 2^(x log2 e - m): masked keys give 2^(-94500 - m) = 0 and p (x - m) = 0
        float2 sp2 = make_float2(0.f, 0.f), spt2 = make_float2(0.f, 0.f);
        const float2 lg2 = make_float2(kLog2eF, kLog2eF), negm = make_float2(-m_new, -m_new);
        uint8_t* pbuf = sP + s * Cfg::kPBytes;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          uint4 pk;
          uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 d2 = __ffma2_rn(__half22float2(xs[g * 4 + k]), lg2, negm);
            const float2 p = make_float2(ex2f(d2.x), ex2f(d2.y));
            sp2 = __fadd2_rn(sp2, p);
            spt2 = __ffma2_rn(p, d2, spt2);
            w[k] = pack_half2_rn(p.x, p.y);
          }
          *reinterpret_cast<uint4*>(pbuf + p_offset(row, half * 64 + g * 8)) = pk;
        }
        fence_proxy_async_smem();  // the P stores, visible to the tensor core's operand reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[s]);
        const float sp = sp2.x + sp2.y, spt = spt2.x + spt2.y;
        // running statistics of this half (base 2): l = sum p, t2 = sum p (x - m)
        if (m2 == -__builtin_huge_valf()) {
          l = sp;
          t2 = spt;
        } else {
          t2 = alpha * (t2 + l * (m2 - m_new)) + spt;
          l = alpha * l + sp;
        }
        m2 = m_new;
        if (j > 0 && !consume_o(j - 1, alpha_prev)) failed = true;
      }
      alpha_prev = alpha;
    }
    if (!failed && nkv > 0 && !consume_o(nkv - 1, alpha_prev)) failed = true;
    if (failed) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
    }
    // the two halves' sums (every softmax thread reaches this barrier, failed or not)
    asm volatile("bar.sync 1, 256;" ::: "memory");
    red[half * 128 + row] = l;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float l_all = l + red[(half ^ 1) * 128 + row];
    asm volatile("bar.sync 1, 256;" ::: "memory");
    red[half * 128 + row] = t2;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float t2_all = t2 + red[(half ^ 1) * 128 + row];
    if (!failed && q < args.S) {
      const float inv = 1.f / l_all;
      __half* out = args.O + ((b * args.S + q) * args.Hq + h) * D + half * kOH;
#pragma unroll
      for (int g = 0; g < kOH / 8; ++g) {
        uint4 pk;
        __half* h8 = reinterpret_cast<__half*>(&pk);
#pragma unroll
        for (int k = 0; k < 8; k += 2) {
          const float2 v = o[(g * 8 + k) >> 1];
          h8[k] = __float2half_rn(v.x * inv);
          h8[k + 1] = __float2half_rn(v.y * inv);
        }
        *reinterpret_cast<uint4*>(out + g * 8) = pk;
      }
      if (half == 0) args.H[bh * args.S + q] = 0.69314718055994531f * (__log2f(l_all) - t2_all / l_all);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace ee
