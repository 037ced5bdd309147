// ee_kvcache.cuh - entropy-tied KV-cache compression (the reference's listed next step,
// README "dynamic KV-Cache compression tied to the entropy metric"): every cached token
// keeps its keys and values at the precision of its entropy tier -- INT8 or FP8-e4m3
// codes with one fp32 scale per (token, KV head), or fp16 -- in two slot pools (8-bit and
// fp16) addressed through a per-sequence slot table, and the decode-step attention reads
// the mixed cache directly, so its HBM traffic shrinks with the 8-bit share.
//   * kv_append_kernel: one CTA per appended token: takes a slot in its tier's pool,
//     quantises the token's K and V rows per KV head (INT8: s = amax / 127, q = rn(x / s);
//     FP8: s = amax / 448, e4m3 = rn-satfinite(x / s)) or copies them (FP16);
//   * kv_decode_attention_kernel: one CTA per (sequence, KV head, token split): the
//     query heads of the group against the split's cached tokens (+ the new token's own
//     fp16 K / V in the last split), softmax with the row entropy as partials (m, l, t, o);
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

// one cached (or the new) token's K or V row of head h as D floats, lane slice e0 .. e0+E
template <int D, int E>
__device__ __forceinline__ void kv_row(const KvCacheArgs& c, int code, int h, bool is_v, int e0, float* x) {
  const int tr = code >> 28, sl = code & 0x0FFFFFFF;
  const size_t off = (static_cast<size_t>(sl) * c.kv_heads + h) * D + e0;
  if (tr == 2) {
    const __half* p = static_cast<const __half*>(is_v ? c.v16 : c.k16) + off;
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(p + e));
      x[e] = f.x;
      x[e + 1] = f.y;
    }
    return;
  }
  const float s = (is_v ? c.v_scale : c.k_scale)[static_cast<size_t>(sl) * c.kv_heads + h];
  const uint8_t* p = (is_v ? c.v8 : c.k8) + off;
  if (tr == 0) {
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = static_cast<float>(static_cast<int8_t>(p[e])) * s;
  } else {
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const float2 f = e4m3x2_to_f32x2(*reinterpret_cast<const uint16_t*>(p + e));
      x[e] = f.x * s;
      x[e + 1] = f.y * s;
    }
  }
}

// Partial attention of the G query heads of KV head h over tokens [t0, t1) of sequence b
// (t == len: the new token's own fp16 K / V).  A warp takes a token at a time (lanes split
// D); per query head the warp keeps m (base 2), l, t = sum p (x - m) and o[D] (lane slice).
template <int D, int G>
__global__ void __launch_bounds__(kKvThreads) kv_decode_attention_kernel(const KvCacheArgs c,
                                                                         const __half* __restrict__ q, int64_t ldq,
                                                                         const __half* __restrict__ k_new,
                                                                         const __half* __restrict__ v_new,
                                                                         int64_t ld_new, float scale, int splits,
                                                                         float* __restrict__ part) {
  griddep_wait();
  constexpr int E = D / 32;
  constexpr int W = kKvThreads / 32;
  const int b = blockIdx.x / c.kv_heads, h = blockIdx.x % c.kv_heads;
  const int split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t len = c.length[b];
  const int64_t total = len + 1;  // cached tokens and the new one
  const int64_t per = (total + splits - 1) / splits;
  const int64_t t0 = split * per, t1 = t0 + per < total ? t0 + per : total;
  constexpr float kLog2e = 1.4426950408889634f;
  float qv[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const __half* qp = q + b * ldq + (static_cast<int64_t>(h) * G + g) * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(qp + e));
      qv[g][e] = f.x * scale * kLog2e;
      qv[g][e + 1] = f.y * scale * kLog2e;
    }
  }
  float m[G], l[G], tt[G], o[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -__builtin_huge_valf();
    l[g] = 0.f;
    tt[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) o[g][e] = 0.f;
  }
  // one token's K and V slices (the new token's from k_new / v_new); false for a hole
  auto load_token = [&](int64_t t, float* kx, float* vx) -> bool {
    if (t == len) {  // the new token, not in the cache yet
      const __half* kp = k_new + b * ld_new + h * D + lane * E;
      const __half* vp = v_new + b * ld_new + h * D + lane * E;
#pragma unroll
      for (int e = 0; e < E; e += 2) {
        const float2 fk = __half22float2(*reinterpret_cast<const __half2*>(kp + e));
        const float2 fv = __half22float2(*reinterpret_cast<const __half2*>(vp + e));
        kx[e] = fk.x;
        kx[e + 1] = fk.y;
        vx[e] = fv.x;
        vx[e + 1] = fv.y;
      }
      return true;
    }
    const int code = c.slot[static_cast<int64_t>(b) * c.max_tokens + t];
    if (code < 0) return false;  // a token its pool had no room for (warp-uniform)
    kv_row<D, E>(c, code, h, false, lane * E, kx);
    kv_row<D, E>(c, code, h, true, lane * E, vx);
    return true;
  };
  auto update = [&](const float* kx, const float* vx) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float sdot = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) sdot = fmaf(qv[g][e], kx[e], sdot);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sdot += __shfl_xor_sync(0xffffffffu, sdot, off);
      // sdot = score * log2 e; online update of m, l, t (base 2) and o
      if (sdot > m[g]) {
        if (m[g] != -__builtin_huge_valf()) {  // (the first token has nothing to rescale)
          const float alpha = exp2f(m[g] - sdot);
          tt[g] = alpha * (tt[g] + l[g] * (m[g] - sdot));
          l[g] *= alpha;
#pragma unroll
          for (int e = 0; e < E; ++e) o[g][e] *= alpha;
        }
        m[g] = sdot;
      }
      const float p = exp2f(sdot - m[g]);
      l[g] += p;
      tt[g] = fmaf(p, sdot - m[g], tt[g]);
#pragma unroll
      for (int e = 0; e < E; ++e) o[g][e] = fmaf(p, vx[e], o[g][e]);
    }
  };
  // two tokens per step: both tokens' slot and row loads are in flight before either is used
  for (int64_t t = t0 + warp; t < t1; t += 2 * W) {
    float ka[E], va[E], kb[E], vb[E];
    const bool oka = load_token(t, ka, va);
    const bool okb = t + W < t1 && load_token(t + W, kb, vb);
    if (oka) update(ka, va);
    if (okb) update(kb, vb);
  }
  // the W warps' partials -> one per (split, query head), through shared memory
  __shared__ float s_mlt[W][G][3];
  __shared__ float s_o[W][G][D];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      s_mlt[warp][g][0] = m[g];
      s_mlt[warp][g][1] = l[g];
      s_mlt[warp][g][2] = tt[g];
    }
#pragma unroll
    for (int e = 0; e < E; ++e) s_o[warp][g][lane * E + e] = o[g][e];
  }
  __syncthreads();
  // thread i merges query head g = i / (kKvThreads / G) ... one (g, column) pair at a time
  const size_t rec = 3 + D;  // m, l, t, o[D] per (sequence, query head, split)
  for (int idx = threadIdx.x; idx < G * (D + 1); idx += kKvThreads) {
    const int g = idx / (D + 1), col = idx % (D + 1);
    float M = -__builtin_huge_valf();
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, s_mlt[w][g][0]);
    float L = 0.f, T = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      const float mw = s_mlt[w][g][0];
      if (mw == -__builtin_huge_valf()) continue;
      const float a = exp2f(mw - M);
      L += s_mlt[w][g][1] * a;
      T += (s_mlt[w][g][2] + s_mlt[w][g][1] * (mw - M)) * a;
      if (col < D) O += s_o[w][g][col] * a;
    }
    float* dst = part + ((static_cast<size_t>(b) * c.kv_heads * G + static_cast<size_t>(h) * G + g) * splits + split) * rec;
    if (col == D) {
      dst[0] = M;
      dst[1] = L;
      dst[2] = T;
    } else {
      dst[3 + col] = O;
    }
  }
}

// out[b, hq, :] = O / L and H[b, hq] = ln L - T ln2 / L over the splits of (b, hq)
template <int D>
__global__ void __launch_bounds__(kKvThreads) kv_decode_combine_kernel(const float* __restrict__ part, int splits,
                                                                       __half* __restrict__ out, int64_t ldo,
                                                                       float* __restrict__ H, int Hq) {
  griddep_wait();
  const int bh = blockIdx.x;  // b * Hq + hq
  const size_t rec = 3 + D;
  const float* p = part + static_cast<size_t>(bh) * splits * rec;
  float M = -__builtin_huge_valf();
  for (int s = 0; s < splits; ++s) M = fmaxf(M, p[s * rec]);
  float L = 0.f, T = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float ms = p[s * rec];
    if (ms == -__builtin_huge_valf()) continue;
    const float a = exp2f(ms - M);
    L += p[s * rec + 1] * a;
    T += (p[s * rec + 2] + p[s * rec + 1] * (ms - M)) * a;
  }
  const int b = bh / Hq, hq = bh % Hq;
  for (int col = threadIdx.x; col < D; col += blockDim.x) {
    float O = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float ms = p[s * rec];
      if (ms == -__builtin_huge_valf()) continue;
      O += p[s * rec + 3 + col] * exp2f(ms - M);
    }
    out[b * ldo + static_cast<int64_t>(hq) * D + col] = __float2half_rn(O / L);
  }
  if (threadIdx.x == 0 && H != nullptr) H[bh] = 0.69314718055994531f * (__log2f(L) - T / L);
}

}  // namespace ee
