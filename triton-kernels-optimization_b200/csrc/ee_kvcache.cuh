// ee_kvcache.cuh - entropy-tied KV-cache compression (the reference's listed next step,
// README "dynamic KV-Cache compression tied to the entropy metric"): every cached token
// keeps its keys and values at the precision of its entropy tier -- INT8 or FP8-e4m3
// codes with one fp32 scale per (token, KV head), or fp16 -- in two slot pools (8-bit and
// fp16) addressed through a per-sequence slot table, and the decode-step attention reads
// the mixed cache directly, so its HBM traffic shrinks with the 8-bit share.
//   * kv_append_kernel: one CTA per appended token: takes a slot in its tier's pool,
//     quantises the token's K and V rows per KV head (INT8: s = amax / 127, q = rn(x / s);
//     FP8: s = amax / 448, e4m3 = rn-satfinite(x / s)) or copies them (FP16);
//   * kv_decode_attention_kernel: one CTA per (sequence, KV head, token split): a producer
//     warp gathers the split's K / V rows through the slot table into a ring of
//     shared-memory stages with bulk copies, four consumer warps score the KV head's query
//     heads against them (+ the new token's own fp16 K / V) on the tensor core with an
//     online softmax and the row entropy, as partials (m, l, t, o);
//   * kv_decode_combine_kernel: merges the splits of each (sequence, query head).
// Included once, by ee_kernels.cu.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "ee_gemm.cuh"  // g_device_error
#include "ee_internal.h"
#include "ee_ptx.cuh"

namespace ee {

// e4m3 <-> float (PTX cvt with round-to-nearest-even and saturation to +-448)
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(hi), "f"(lo));
  return out;
}
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint16_t v) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(v));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

constexpr int kKvThreads = 128;

// one CTA per appended token (b, t): heads are spread over the four warps, a head's D
// values over the 32 lanes (D / 32 each)
template <int D>
__global__ void __launch_bounds__(kKvThreads) kv_append_kernel(const KvCacheArgs c, const __half* __restrict__ k_rows,
                                                               int64_t ldk, const __half* __restrict__ v_rows,
                                                               int64_t ldv, const int8_t* __restrict__ tier,
                                                               int64_t t_new) {
  griddep_wait();
  constexpr int E = D / 32;  // values per lane
  const int64_t tok = blockIdx.x;  // b * t_new + t
  const int64_t b = tok / t_new, t = tok - b * t_new;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int s_slot;
  const int tr = tier[tok] < 0 ? 0 : (tier[tok] > 2 ? 2 : tier[tok]);
  const int pool = tr == 2 ? 1 : 0;
  const int64_t pos = c.length[b] + t;
  if (threadIdx.x == 0) {
    int sl = -1;
    if (pos < c.max_tokens) {
      const uint32_t idx = atomicAdd(&c.pool_used[pool], 1u);
      if (idx < static_cast<uint32_t>(pool ? c.slots16 : c.slots8)) sl = static_cast<int>(idx);
    }
    if (sl < 0) {
      atomicOr(&g_device_error, kErrCapacity);  // the pool (or the sequence) is full
      if (pos < c.max_tokens) c.slot[b * c.max_tokens + pos] = -1;  // a hole the attention skips
    } else {
      c.slot[b * c.max_tokens + pos] = (tr << 28) | sl;
    }
    s_slot = sl;
  }
  __syncthreads();
  const int sl = s_slot;
  if (sl < 0) return;
  const __half* kr = k_rows + tok * ldk;
  const __half* vr = v_rows + tok * ldv;
  for (int h = warp; h < c.kv_heads; h += kKvThreads / 32) {
    for (int which = 0; which < 2; ++which) {
      const __half* src = (which == 0 ? kr : vr) + h * D + lane * E;
      float x[E];
#pragma unroll
      for (int e = 0; e < E; e += 2) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(src + e));
        x[e] = f.x;
        x[e + 1] = f.y;
      }
      const size_t off = (static_cast<size_t>(sl) * c.kv_heads + h) * D + lane * E;
      if (tr == 2) {
        __half* dst = static_cast<__half*>(which == 0 ? c.k16 : c.v16) + off;
#pragma unroll
        for (int e = 0; e < E; e += 2) *reinterpret_cast<__half2*>(dst + e) = *reinterpret_cast<const __half2*>(src + e);
        continue;
      }
      float amax = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) amax = fmaxf(amax, fabsf(x[e]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float s = amax > 0.f ? amax / (tr == 0 ? 127.f : 448.f) : 1.f;
      const float inv = 1.f / s;
      uint8_t* dst = (which == 0 ? c.k8 : c.v8) + off;
      if (tr == 0) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float q = fminf(fmaxf(rintf(x[e] * inv), -127.f), 127.f);
          dst[e] = static_cast<uint8_t>(static_cast<int8_t>(q));
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; e += 2) *reinterpret_cast<uint16_t*>(dst + e) = f32x2_to_e4m3x2(x[e] * inv, x[e + 1] * inv);
      }
      if (lane == 0) (which == 0 ? c.k_scale : c.v_scale)[static_cast<size_t>(sl) * c.kv_heads + h] = s;
    }
  }
}

// lengths grow once every token of the step is stored
__global__ void kv_commit_kernel(const KvCacheArgs c, int64_t t_new) {
  griddep_wait();
  const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b < c.batch) {
    const int64_t n = c.length[b] + t_new;
    c.length[b] = static_cast<int32_t>(n < c.max_tokens ? n : c.max_tokens);
  }
}

// Decode attention as a copy pipeline.  One CTA per (sequence, KV head, token split, group
// of up to eight query heads), 192 threads:
//   warps 0-1  producers: per ring stage of kKvTT = 32 tokens, gather the tokens' K and V
//              rows (D bytes for an 8-bit token, 2 D for fp16, none for a hole) through
//              the slot table with 16-byte asynchronous copies, four lanes per row, and
//              their tiers and 8-bit scales into the stage's metadata; the copies complete
//              on the stage's full barrier;
//   warps 2-5  consumers: warp w takes tokens 8 (w - 2) .. + 7 of every stage and runs the
//              query heads against them on the tensor core (mma.sync m16n8k16 / m16n8k8,
//              fp16 operands, fp32 accumulation; the heads are the M = 16 rows, the 8-bit
//              codes convert to fp16 exactly): S = Q K^T, then the online softmax per head
//              (m base 2, l, t = sum p (x - m)) on S's fragment, then O += (p * s_v) V.
//              The K scale and softmax scale multiply S in fp32.
// The bytes in flight sit in the ring (kKvStages stages), not in registers.  Every wait is
// bounded; on expiry the CTA records the error word, the producer waits (bounded) for its
// copies in flight and the CTA exits.
constexpr int kKvTT = 32;        // tokens per ring stage (eight per consumer warp)
constexpr int kKvStages = 5;     // ring depth
constexpr int kKvCWarps = 4;     // consumer warps
constexpr int kKvPWarps = 2;     // producer warps (16 rows of a stage each)
constexpr int kKvPipeThreads = 32 * (kKvPWarps + kKvCWarps);
constexpr int kKvCodeNone = -2;  // past the split's tokens
constexpr int kKvCodeNew = -3;   // the step's own token (its rows in k_new / v_new)

template <int D>
struct KvPipe {
  static constexpr int kRow = 2 * D;                      // bytes per row slot (an fp16 row)
  static constexpr int kRowsBytes = 2 * kKvTT * kRow;     // K rows, then V rows
  static constexpr int kMetaBytes = kKvTT * 16;           // per token: K scale, V scale, tier
  static constexpr int kStageBytes = kRowsBytes + kMetaBytes;
  static constexpr size_t kSmem = 128 /*alignment slack*/ + size_t(kKvStages) * kStageBytes + 2 * kKvStages * 8 + 16;
};

// a stage's K row j / V row j / metadata
template <int D>
__device__ __forceinline__ uint8_t* kv_row(uint8_t* ring, int s, bool v, int j) {
  return ring + s * KvPipe<D>::kStageBytes + (v ? kKvTT * KvPipe<D>::kRow : 0) + j * KvPipe<D>::kRow;
}
template <int D>
__device__ __forceinline__ int4* kv_meta(uint8_t* ring, int s) {
  return reinterpret_cast<int4*>(ring + s * KvPipe<D>::kStageBytes + KvPipe<D>::kRowsBytes);
}

// 16-byte asynchronous copy global -> shared (load/store path, no registers held), and the
// arrival on `bar` once every copy this thread issued so far has landed (the barrier's
// count includes it: noinc)
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// producer warp: the split's tokens [t0, t1) through the ring, nst stages; false if a wait
// gave up (the copies already issued have then landed or timed out).  Both producer warps
// read the stage's 32 slot codes (lane l: token l, a chunk of four stages ahead) and rank
// the tokens by tier; lane l of producer pw copies the rows of tokens 8 k + l / 4
// (k = 2 pw, 2 pw + 1) into their ranked ring rows, 16-byte chunks 4 q + l % 4 (the four
// lanes of a row move 64 contiguous bytes per instruction), and the row's first lane puts
// the tier into the stage's metadata and copies the token's 8-bit scales there.
constexpr int kKvChunk = 4;  // stages whose slot codes are read at once
template <int D>
__device__ __forceinline__ bool kv_produce(const KvCacheArgs& c, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                           const volatile int* abort, int64_t b, int h, int64_t len, int64_t t0,
                                           int64_t t1, int nst, const __half* kn, const __half* vn, int pw, int lane) {
  constexpr int K = 4 / kKvPWarps;  // row groups per producer warp
  const int part = lane & 3;
  // lane l reads the code of token l of each stage
  auto codes_of = [&](int ch, int (&code)[kKvChunk]) {
#pragma unroll
    for (int ii = 0; ii < kKvChunk; ++ii) {
      const int64_t t = t0 + static_cast<int64_t>(ch * kKvChunk + ii) * kKvTT + lane;
      code[ii] = t >= t1 ? kKvCodeNone : (t == len ? kKvCodeNew : c.slot[b * c.max_tokens + t]);  // -1: hole
    }
  };
  int code[kKvChunk];
  codes_of(0, code);
  uint32_t issued = 0, parity = 0;  // per stage: copies issued, parity of the last issue
  bool ok = true;
  const int nch = (nst + kKvChunk - 1) / kKvChunk;
  for (int ch = 0; ch < nch && ok; ++ch) {
    int ncode[kKvChunk];
    codes_of(ch + 1, ncode);  // the next chunk's codes, under this chunk's copies
#pragma unroll
    for (int ii = 0; ii < kKvChunk; ++ii) {
      const int i = ch * kKvChunk + ii;
      if (i >= nst) break;
      const int s = i % kKvStages;
      const uint32_t ph = static_cast<uint32_t>(i / kKvStages) & 1u;
      if (!mbar_wait_warp(&empty[s], ph ^ 1u, abort)) {
        ok = false;
        break;
      }
      int4* meta = kv_meta<D>(ring, s);
      // the stage's ring row of token `lane`: tokens grouped by tier (INT8, FP8, fp16, then
      // nothing), so that most consumer warps meet one tier (the attention does not
      // depend on the tokens' order)
      const int my_tier = code[ii] == kKvCodeNew ? 2 : (code[ii] >= 0 ? code[ii] >> 28 : 3);
      const uint32_t below = (1u << lane) - 1u;
      int dest = 0;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint32_t m = __ballot_sync(0xffffffffu, my_tier == v);
        if (my_tier > v) dest += __popc(m);
        if (my_tier == v) dest += __popc(m & below);
      }
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int tok = 8 * (K * pw + k) + (lane >> 2);  // the token whose rows this lane copies
        const int cd = __shfl_sync(0xffffffffu, code[ii], tok);
        const int r = __shfl_sync(0xffffffffu, dest, tok);
        const int tier = cd == kKvCodeNew ? 2 : (cd >= 0 ? cd >> 28 : -1);
        const size_t sl = static_cast<size_t>(cd & 0x0FFFFFFF);
        const size_t roff = (sl * c.kv_heads + h) * D * (tier == 2 ? 2 : 1);
        const uint8_t* kp = cd == kKvCodeNew ? reinterpret_cast<const uint8_t*>(kn + h * D)
                                             : (tier == 2 ? static_cast<const uint8_t*>(c.k16) : c.k8) + roff;
        const uint8_t* vp = cd == kKvCodeNew ? reinterpret_cast<const uint8_t*>(vn + h * D)
                                             : (tier == 2 ? static_cast<const uint8_t*>(c.v16) : c.v8) + roff;
        const int nchunk = tier < 0 ? 0 : (tier == 2 ? 2 * D / 16 : D / 16);
        uint8_t* kd = kv_row<D>(ring, s, false, r);
        uint8_t* vd = kv_row<D>(ring, s, true, r);
#pragma unroll
        for (int q = 0; q < 2 * D / 64; ++q) {
          const int chunk = 4 * q + part;
          if (chunk < nchunk) {
            cp_async_16(kd + 16 * chunk, kp + 16 * chunk);
            cp_async_16(vd + 16 * chunk, vp + 16 * chunk);
          }
        }
        if (part == 0) {
          int* mr = reinterpret_cast<int*>(&meta[r]);
          mr[2] = tier;
          if (tier == 0 || tier == 1) {
            const size_t si = sl * c.kv_heads + h;
            cp_async_4(mr, c.k_scale + si);
            cp_async_4(mr + 1, c.v_scale + si);
          } else {
            mr[0] = __float_as_int(1.f);
            mr[1] = __float_as_int(1.f);
          }
        }
      }
      cp_async_arrive_noinc(&full[s]);  // this lane's copies of the stage, when they land
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);  // publishes the tiers written above
      issued |= 1u << s;
      parity = (parity & ~(1u << s)) | (ph << s);
    }
#pragma unroll
    for (int ii = 0; ii < kKvChunk; ++ii) code[ii] = ncode[ii];
  }
  if (!ok) {  // wait (bounded) for the copies in flight
    for (int s = 0; s < kKvStages; ++s)
      if (issued & (1u << s)) (void)mbar_wait(&full[s], (parity >> s) & 1u, nullptr);
  }
  return ok;
}

// fp16 pairs from 8-bit codes, exactly: four int8 (one word) -> (c0, c1), (c2, c3) by the
// 1024-offset trick (fp16 1024 + u for the byte u = c + 128, minus 1152); two e4m3 (a half
// word) -> one pair by cvt
__device__ __forceinline__ void i8x4_to_h2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;
  const uint32_t a = __byte_perm(x, 0x64646464u, 0x5140);  // bytes x0, 0x64, x1, 0x64
  const uint32_t b = __byte_perm(x, 0x64646464u, 0x7362);  // bytes x2, 0x64, x3, 0x64
  const __half2 off = __halves2half2(__ushort_as_half(0x6480u), __ushort_as_half(0x6480u));  // 1152
  const __half2 ra = __hsub2(*reinterpret_cast<const __half2*>(&a), off);
  const __half2 rb = __hsub2(*reinterpret_cast<const __half2*>(&b), off);
  lo = *reinterpret_cast<const uint32_t*>(&ra);
  hi = *reinterpret_cast<const uint32_t*>(&rb);
}
__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint32_t v16) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(static_cast<uint16_t>(v16)));
  return h;
}

// n consecutive values of a ring row from byte offset `first` (in elements) as n / 2 fp16
// pairs; zero for a row that holds nothing (tier < 0)
template <int N>
__device__ __forceinline__ void kv_pairs(const uint8_t* row, int tier, int first, uint32_t (&h)[N / 2]) {
  if (tier < 0) {
#pragma unroll
    for (int i = 0; i < N / 2; ++i) h[i] = 0u;
    return;
  }
  if (tier == 2) {  // fp16: the pairs as stored
    const uint32_t a = smem_u32(row + 2 * first);
#pragma unroll
    for (int q = 0; q < N / 8; ++q)
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(h[4 * q]), "=r"(h[4 * q + 1]), "=r"(h[4 * q + 2]), "=r"(h[4 * q + 3])
                   : "r"(a + 16u * q));
    return;
  }
  uint32_t w[N / 4];
  const uint32_t a = smem_u32(row + first);
  if constexpr (N >= 16) {
#pragma unroll
    for (int q = 0; q < N / 16; ++q)
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(w[4 * q]), "=r"(w[4 * q + 1]), "=r"(w[4 * q + 2]), "=r"(w[4 * q + 3])
                   : "r"(a + 16u * q));
  } else {
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "r"(a));
  }
  if (tier == 0) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) i8x4_to_h2(w[i], h[2 * i], h[2 * i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      h[2 * i] = e4m3x2_to_h2(w[i] & 0xFFFFu);
      h[2 * i + 1] = e4m3x2_to_h2(w[i] >> 16);
    }
  }
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_1688(float (&d)[4], uint32_t a0, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(b0));
}

// Partial attention of query heads h * G + g0 .. + GC - 1 of KV head h over tokens [t0, t1)
// of sequence b (t == len: the new token's own fp16 K / V), as (m, l, t, o) per head.
// Fragment layout of a consumer lane (gq, q4) = (lane / 4, lane % 4): Q / S / P rows are
// heads (row gq real when gq < GC; rows 8..15 zero); the K operand of token gq is its row
// elements (D/4) q4 .. + D/4 - 1 in order (the MMA's k index is a fixed permutation of
// the head dimension, the same for Q); S columns 2 q4, 2 q4 + 1 are tokens; the V operand
// of P V block nb is dimension (D/8) gq + nb of tokens 2 q4, 2 q4 + 1, so O's columns
// 2 q4, 2 q4 + 1 of block nb are dimensions (D/8) (2 q4) + nb and (D/8) (2 q4 + 1) + nb.
template <int D, int G, int GC>
__global__ void __launch_bounds__(kKvPipeThreads) kv_decode_attention_kernel(const KvCacheArgs c,
                                                                             const __half* __restrict__ q, int64_t ldq,
                                                                             const __half* __restrict__ k_new,
                                                                             const __half* __restrict__ v_new,
                                                                             int64_t ld_new, float scale, int splits,
                                                                             float* __restrict__ part) {
  static_assert(GC >= 1 && GC <= 8, "at most eight query heads per CTA (the M = 16 rows, 8..15 unused)");
  constexpr int W = kKvCWarps;
  constexpr int NB = D / 8;  // P V blocks of eight output dimensions
  constexpr float kNegInf = -__builtin_huge_valf();
  extern __shared__ uint8_t kv_smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(kv_smem_raw) + 127) & ~uintptr_t(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kKvStages * KvPipe<D>::kStageBytes);
  uint64_t* empty = full + kKvStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kKvStages);
  const int b = blockIdx.x / c.kv_heads, h = blockIdx.x % c.kv_heads;
  const int split = blockIdx.y;
  const int g0 = blockIdx.z * GC;  // first query head of the group this CTA handles
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(&full[s], 33 * kKvPWarps);  // per producer warp: its 32 lanes' copies + its metadata arrival
      mbar_init(&empty[s], W);  // one arrival per consumer warp
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();
  const int64_t len = c.length[b];
  const int64_t total = len + 1;  // cached tokens and the new one
  const int64_t per = (total + splits - 1) / splits;
  const int64_t t0 = split * per, t1 = t0 + per < total ? t0 + per : total;
  const int nst = t1 > t0 ? static_cast<int>((t1 - t0 + kKvTT - 1) / kKvTT) : 0;
  __shared__ float s_mlt[W][GC][3];
  __shared__ float s_o[W][GC][D];
  if (warp < kKvPWarps) {
    if (!kv_produce<D>(c, ring, full, empty, abort_flag, b, h, len, t0, t1, nst, k_new + b * ld_new,
                       v_new + b * ld_new, warp, lane)) {
      if (lane == 0) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        *abort_flag = 1;
      }
    }
  } else {
    const int cw = warp - kKvPWarps;
    const int gq = lane >> 2, q4 = lane & 3;
    const bool row_real = gq < GC;
    constexpr float kLog2e = 1.4426950408889634f;
    const float sl2e = scale * kLog2e;
    // Q rows (fp16 as given), the MMA A operand: k-block kb is qa[2 kb], qa[2 kb + 1]
    uint32_t qa[D / 8];
    {
      const uint32_t* qp = reinterpret_cast<const uint32_t*>(
          q + b * ldq + (static_cast<int64_t>(h) * G + g0 + (row_real ? gq : 0)) * D + (D / 4) * q4);
#pragma unroll
      for (int i = 0; i < D / 8; ++i) qa[i] = row_real ? qp[i] : 0u;
    }
    float m = kNegInf, l = 0.f, tt = 0.f;  // row gq, over this lane's columns
    float o[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.f;
    for (int i = 0; i < nst; ++i) {
      const int s = i % kKvStages;
      if (!mbar_wait_warp(&full[s], static_cast<uint32_t>(i / kKvStages) & 1u, abort_flag)) {
        if (lane == 0) {
          atomicOr(&g_device_error, kErrWaitTimeout);
          *abort_flag = 1;
        }
        break;
      }
      const int j0 = 8 * cw;  // this warp's first token of the stage
      const int4* meta = kv_meta<D>(ring, s);
      const int4 mk = meta[j0 + gq], ma = meta[j0 + 2 * q4], mb = meta[j0 + 2 * q4 + 1];
      uint32_t kf[D / 8];  // K of token gq, elements (D/4) q4 ..
      kv_pairs<D / 4>(kv_row<D>(ring, s, false, j0 + gq), mk.z, (D / 4) * q4, kf);
      uint32_t va[D / 16], vb[D / 16];  // V of tokens 2 q4, 2 q4 + 1, dimensions (D/8) gq ..
      kv_pairs<D / 8>(kv_row<D>(ring, s, true, j0 + 2 * q4), ma.z, (D / 8) * gq, va);
      kv_pairs<D / 8>(kv_row<D>(ring, s, true, j0 + 2 * q4 + 1), mb.z, (D / 8) * gq, vb);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // the stage's rows are in registers
      // two independent accumulation chains over the k-blocks (even / odd), added after
      float sc[4] = {0.f, 0.f, 0.f, 0.f}, sd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kb = 0; kb < D / 16; kb += 2) {
        mma_16816(sc, qa[2 * kb], qa[2 * kb + 1], kf[2 * kb], kf[2 * kb + 1]);
        mma_16816(sd, qa[2 * kb + 2], qa[2 * kb + 3], kf[2 * kb + 2], kf[2 * kb + 3]);
      }
      sc[0] += sd[0];
      sc[1] += sd[1];
      // row gq, tokens 2 q4 and 2 q4 + 1: base-2 logits (K scale, softmax scale), holes -inf
      const float x0 = ma.z >= 0 ? sc[0] * (sl2e * __int_as_float(ma.x)) : kNegInf;
      const float x1 = mb.z >= 0 ? sc[1] * (sl2e * __int_as_float(mb.x)) : kNegInf;
      float mt = fmaxf(x0, x1);
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      if (mt > m) {
        if (m != kNegInf) {
          const float alpha = exp2f(m - mt);
          tt = alpha * (tt + l * (m - mt));
          l *= alpha;
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            o[nb][0] *= alpha;
            o[nb][1] *= alpha;
          }
        }
        m = mt;
      }
      const float p0 = x0 == kNegInf ? 0.f : exp2f(x0 - m);
      const float p1 = x1 == kNegInf ? 0.f : exp2f(x1 - m);
      l += p0 + p1;
      tt += (p0 > 0.f ? p0 * (x0 - m) : 0.f) + (p1 > 0.f ? p1 * (x1 - m) : 0.f);
      // P (V scale folded in) as the A operand of row gq, k = tokens 2 q4, 2 q4 + 1
      const __half2 ph = __floats2half2_rn(p0 * __int_as_float(ma.y), p1 * __int_as_float(mb.y));
      const uint32_t pa = *reinterpret_cast<const uint32_t*>(&ph);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        // tokens 2 q4, 2 q4 + 1 of dimension (D/8) gq + nb, interleaved
        const uint32_t bv = __byte_perm(va[nb >> 1], vb[nb >> 1], (nb & 1) ? 0x7632 : 0x5410);
        mma_1688(o[nb], pa, bv);
      }
    }
    // the row's statistics over its four lanes (m is the same in all four)
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    tt += __shfl_xor_sync(0xffffffffu, tt, 1);
    tt += __shfl_xor_sync(0xffffffffu, tt, 2);
    if (row_real) {
      if (q4 == 0) {
        s_mlt[cw][gq][0] = m;
        s_mlt[cw][gq][1] = l;
        s_mlt[cw][gq][2] = tt;
      }
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        s_o[cw][gq][(D / 8) * (2 * q4) + nb] = o[nb][0];
        s_o[cw][gq][(D / 8) * (2 * q4 + 1) + nb] = o[nb][1];
      }
    }
  }
  __syncthreads();
  // one record per (split, query head): m, l, t, o[D]
  const size_t rec = 3 + D;
  const int Hq = static_cast<int>(c.kv_heads) * G;
  for (int idx = threadIdx.x; idx < GC * (D + 1); idx += blockDim.x) {
    const int g = idx / (D + 1), col = idx % (D + 1);
    float M = kNegInf;
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, s_mlt[w][g][0]);
    float L = 0.f, T = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      const float mw = s_mlt[w][g][0];
      if (mw == kNegInf) continue;
      const float a = exp2f(mw - M);
      L += s_mlt[w][g][1] * a;
      T += (s_mlt[w][g][2] + s_mlt[w][g][1] * (mw - M)) * a;
      if (col < D) O += s_o[w][g][col] * a;
    }
    const int hq = h * G + g0 + g;
    float* dst = part + ((static_cast<size_t>(b) * Hq + hq) * splits + split) * rec;
    if (col == D) {
      dst[0] = M;
      dst[1] = L;
      dst[2] = T;
    } else {
      dst[3 + col] = O;
    }
  }
}

// out[b, hq, :] = O / L and H[b, hq] = ln L - T ln2 / L over the splits of (b, hq): the
// splits' weights 2^(m_s - M) are formed once in shared memory, then every thread sums
// its output column over the splits with independent loads
constexpr int kKvMaxSplits = 1024;
template <int D>
__global__ void __launch_bounds__(kKvThreads) kv_decode_combine_kernel(const float* __restrict__ part, int splits,
                                                                       __half* __restrict__ out, int64_t ldo,
                                                                       float* __restrict__ H, int Hq) {
  griddep_wait();
  __shared__ float s_w[kKvMaxSplits];
  __shared__ float s_red[2][kKvThreads / 32];
  __shared__ float s_M;
  const int bh = blockIdx.x;  // b * Hq + hq
  const size_t rec = 3 + D;
  const float* p = part + static_cast<size_t>(bh) * splits * rec;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float mx = -__builtin_huge_valf();
  for (int sp = threadIdx.x; sp < splits; sp += kKvThreads) mx = fmaxf(mx, p[sp * rec]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[0][warp] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = s_red[0][0];
    for (int w = 1; w < kKvThreads / 32; ++w) M = fmaxf(M, s_red[0][w]);
    s_M = M;
  }
  __syncthreads();
  const float M = s_M;
  float L = 0.f, T = 0.f;
  for (int sp = threadIdx.x; sp < splits; sp += kKvThreads) {
    const float ms = p[sp * rec];
    const float a = ms == -__builtin_huge_valf() ? 0.f : exp2f(ms - M);
    s_w[sp] = a;
    if (a != 0.f) {
      const float ls = p[sp * rec + 1];
      L += ls * a;
      T += (p[sp * rec + 2] + ls * (ms - M)) * a;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    L += __shfl_xor_sync(0xffffffffu, L, o);
    T += __shfl_xor_sync(0xffffffffu, T, o);
  }
  __syncthreads();
  if (lane == 0) {
    s_red[0][warp] = L;
    s_red[1][warp] = T;
  }
  __syncthreads();
  L = 0.f;
  T = 0.f;
#pragma unroll
  for (int w = 0; w < kKvThreads / 32; ++w) {
    L += s_red[0][w];
    T += s_red[1][w];
  }
  const int b = bh / Hq, hq = bh % Hq;
  for (int col = threadIdx.x; col < D; col += blockDim.x) {
    float O0 = 0.f, O1 = 0.f, O2 = 0.f, O3 = 0.f;
    int sp = 0;
    for (; sp + 4 <= splits; sp += 4) {
      O0 = fmaf(p[sp * rec + 3 + col], s_w[sp], O0);
      O1 = fmaf(p[(sp + 1) * rec + 3 + col], s_w[sp + 1], O1);
      O2 = fmaf(p[(sp + 2) * rec + 3 + col], s_w[sp + 2], O2);
      O3 = fmaf(p[(sp + 3) * rec + 3 + col], s_w[sp + 3], O3);
    }
    for (; sp < splits; ++sp) O0 = fmaf(p[sp * rec + 3 + col], s_w[sp], O0);
    out[b * ldo + static_cast<int64_t>(hq) * D + col] = __float2half_rn(((O0 + O1) + (O2 + O3)) / L);
  }
  if (threadIdx.x == 0 && H != nullptr) H[bh] = 0.69314718055994531f * (__log2f(L) - T / L);
}

}  // namespace ee
