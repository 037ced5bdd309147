// ee_kvcache.cuh - entropy-tied KV-cache compression (the reference's listed next step,
// README "dynamic KV-Cache compression tied to the entropy metric"): every cached token
// keeps its keys and values at the precision of its entropy tier -- INT8 or FP8-e4m3
// codes with one fp32 scale per (token, KV head), or fp16 -- in two slot pools (8-bit and
// fp16) addressed through a per-sequence slot table, and the decode-step attention reads
// the mixed cache directly, so its HBM traffic shrinks with the 8-bit share.
//   * kv_append_kernel: one CTA per appended token: takes a slot in its tier's pool,
//     quantises the token's K and V rows per KV head (INT8: s = amax / 127, q = rn(x / s);
//     FP8: s = amax / 448, e4m3 = rn-satfinite(x / s)) or copies them (FP16);
//   * kv_decode_attention_kernel: one CTA per (sequence, KV head, token split, group of up
//     to four query heads): eight lanes per token, four tokens per warp step, the query
//     heads against the split's cached tokens (+ the new token's own fp16 K / V),
//     softmax with the row entropy as partials (m, l, t, o);
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

// Eight lanes per token: lane (grp, sl) = (lane / 8, lane % 8) holds elements
// sl * E8 .. sl * E8 + E8 - 1 (E8 = D / 8) of token grp's K and V rows, so a warp has four
// tokens' rows in flight per step (eight with the two-step unroll) and a dot product
// needs three shuffles inside the lane group.
template <int D>
struct KvSlice {
  static constexpr int E8 = D / 8;  // values per lane: 16 (D 128) or 8 (D 64)
};

// One token's K and V slices as loaded, before dequantisation: 16 (8-bit) or 32 (fp16)
// bytes of each per lane, the tier and the two scales.  Loading a step's rows into these
// registers one step ahead of its arithmetic keeps two steps of loads in flight per warp.
// (A deeper ring of cp.async copies through shared memory measured slower: 471 against
// 380 us at 16 x 8192 tokens; the kernel's 200+ registers per thread, two CTAs per SM,
// limit it more than the depth of its prefetch.)
struct KvRaw {
  uint4 k[2], v[2];
  float ks, vs;
  int tier;  // 0 INT8, 1 FP8, 2 fp16 (the new token too), -1 nothing (hole / out of range)
};

template <int D>
__device__ __forceinline__ void kv_load(const KvCacheArgs& c, int code, bool is_new, const __half* kn,
                                        const __half* vn, int h, int e0, KvRaw& r) {
  constexpr int E8 = KvSlice<D>::E8;
  if (is_new) {
    const __half* kp = kn + h * D + e0;
    const __half* vp = vn + h * D + e0;
    r.k[0] = *reinterpret_cast<const uint4*>(kp);
    r.v[0] = *reinterpret_cast<const uint4*>(vp);
    if constexpr (E8 == 16) {
      r.k[1] = *reinterpret_cast<const uint4*>(kp + 8);
      r.v[1] = *reinterpret_cast<const uint4*>(vp + 8);
    }
    r.tier = 2;
    return;
  }
  if (code < 0) {
    r.tier = -1;
    return;
  }
  const int tr = code >> 28, sl = code & 0x0FFFFFFF;
  const size_t off = (static_cast<size_t>(sl) * c.kv_heads + h) * D + e0;
  r.tier = tr;
  if (tr == 2) {
    const __half* kp = static_cast<const __half*>(c.k16) + off;
    const __half* vp = static_cast<const __half*>(c.v16) + off;
    r.k[0] = *reinterpret_cast<const uint4*>(kp);
    r.v[0] = *reinterpret_cast<const uint4*>(vp);
    if constexpr (E8 == 16) {
      r.k[1] = *reinterpret_cast<const uint4*>(kp + 8);
      r.v[1] = *reinterpret_cast<const uint4*>(vp + 8);
    }
    return;
  }
  const size_t si = static_cast<size_t>(sl) * c.kv_heads + h;
  r.ks = c.k_scale[si];
  r.vs = c.v_scale[si];
  if constexpr (E8 == 16) {
    r.k[0] = *reinterpret_cast<const uint4*>(c.k8 + off);
    r.v[0] = *reinterpret_cast<const uint4*>(c.v8 + off);
  } else {
    const uint2 ku = *reinterpret_cast<const uint2*>(c.k8 + off);
    const uint2 vu = *reinterpret_cast<const uint2*>(c.v8 + off);
    r.k[0] = make_uint4(ku.x, ku.y, 0u, 0u);
    r.v[0] = make_uint4(vu.x, vu.y, 0u, 0u);
  }
}

// the E8 floats of a loaded slice (is_v: the V slice)
template <int D>
__device__ __forceinline__ void kv_dequant(const KvRaw& r, bool is_v, float* x) {
  constexpr int E8 = KvSlice<D>::E8;
  const uint4* u = is_v ? r.v : r.k;
  if (r.tier == 2) {
#pragma unroll
    for (int q = 0; q < E8 / 8; ++q) {
      const __half2* hp = reinterpret_cast<const __half2*>(&u[q]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(hp[i]);
        x[8 * q + 2 * i] = f.x;
        x[8 * q + 2 * i + 1] = f.y;
      }
    }
    return;
  }
  const float s = is_v ? r.vs : r.ks;
  const uint32_t w[4] = {u[0].x, u[0].y, u[0].z, u[0].w};
  if (r.tier == 0) {
#pragma unroll
    for (int i = 0; i < E8 / 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) x[4 * i + j] = static_cast<float>(static_cast<int8_t>(w[i] >> (8 * j))) * s;
  } else {
#pragma unroll
    for (int i = 0; i < E8 / 4; ++i) {
      const float2 lo = e4m3x2_to_f32x2(static_cast<uint16_t>(w[i] & 0xFFFFu));
      const float2 hi = e4m3x2_to_f32x2(static_cast<uint16_t>(w[i] >> 16));
      x[4 * i] = lo.x * s;
      x[4 * i + 1] = lo.y * s;
      x[4 * i + 2] = hi.x * s;
      x[4 * i + 3] = hi.y * s;
    }
  }
}

// Partial attention of query heads h * G + g0 .. + GC - 1 of KV head h over tokens [t0, t1)
// of sequence b (t == len: the new token's own fp16 K / V).  Per lane group (one token at
// a time) an online softmax per head: m (base 2), l, t = sum p (x - m) and the lane's
// slice of o; the four groups of a warp merge by shuffles, the warps through shared memory.
template <int D, int G, int GC>
__global__ void __launch_bounds__(kKvThreads) kv_decode_attention_kernel(const KvCacheArgs c,
                                                                         const __half* __restrict__ q, int64_t ldq,
                                                                         const __half* __restrict__ k_new,
                                                                         const __half* __restrict__ v_new,
                                                                         int64_t ld_new, float scale, int splits,
                                                                         float* __restrict__ part) {
  griddep_wait();
  constexpr int E8 = KvSlice<D>::E8;
  constexpr int W = kKvThreads / 32;
  constexpr float kNegInf = -__builtin_huge_valf();
  const int b = blockIdx.x / c.kv_heads, h = blockIdx.x % c.kv_heads;
  const int split = blockIdx.y;
  const int g0 = blockIdx.z * GC;  // first query head of the group this CTA handles
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 3, sl = lane & 7;
  const int e0 = sl * E8;
  const int64_t len = c.length[b];
  const int64_t total = len + 1;  // cached tokens and the new one
  const int64_t per = (total + splits - 1) / splits;
  const int64_t t0 = split * per, t1 = t0 + per < total ? t0 + per : total;
  constexpr float kLog2e = 1.4426950408889634f;
  float qv[GC][E8];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    const __half* qp = q + b * ldq + (static_cast<int64_t>(h) * G + g0 + g) * D + e0;
#pragma unroll
    for (int e = 0; e < E8; e += 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(qp + e));
      qv[g][e] = f.x * scale * kLog2e;
      qv[g][e + 1] = f.y * scale * kLog2e;
    }
  }
  float m[GC], l[GC], tt[GC], o[GC][E8];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    m[g] = kNegInf;
    l[g] = 0.f;
    tt[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E8; ++e) o[g][e] = 0.f;
  }
  const __half* kn = k_new + b * ld_new;
  const __half* vn = v_new + b * ld_new;
  // the warp's tokens: step i covers t = t0 + 4 * (warp + W * i) + grp; slot codes are read
  // two steps ahead and rows one step ahead of the arithmetic
  auto code_of = [&](int64_t t) -> int {
    if (t >= t1) return -1;
    if (t == len) return 0;  // the new token (its rows come from k_new / v_new)
    return c.slot[static_cast<int64_t>(b) * c.max_tokens + t];
  };
  const int64_t stride = 4 * W;
  int64_t tcur = t0 + 4 * warp + grp;
  int code_next = code_of(tcur + stride);
  KvRaw cur;
  kv_load<D>(c, code_of(tcur), tcur < t1 && tcur == len, kn, vn, h, e0, cur);
  if (tcur >= t1) cur.tier = -1;
  for (int64_t base = t0 + 4 * warp; base < t1; base += stride) {
    // next step's rows and the step after's codes, before this step's arithmetic
    const int64_t tn = tcur + stride;
    KvRaw nxt;
    kv_load<D>(c, code_next, tn < t1 && tn == len, kn, vn, h, e0, nxt);
    if (tn >= t1) nxt.tier = -1;
    code_next = code_of(tn + stride);
    const bool valid = cur.tier >= 0;
    float kx[E8], vx[E8];
    if (valid) {
      kv_dequant<D>(cur, false, kx);
      kv_dequant<D>(cur, true, vx);
    } else {
#pragma unroll
      for (int e = 0; e < E8; ++e) kx[e] = vx[e] = 0.f;
    }
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      float sdot = 0.f;
#pragma unroll
      for (int e = 0; e < E8; ++e) sdot = fmaf(qv[g][e], kx[e], sdot);
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 4);
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 2);
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
      if (!valid) continue;
      if (sdot > m[g]) {
        if (m[g] != kNegInf) {
          const float alpha = exp2f(m[g] - sdot);
          tt[g] = alpha * (tt[g] + l[g] * (m[g] - sdot));
          l[g] *= alpha;
#pragma unroll
          for (int e = 0; e < E8; ++e) o[g][e] *= alpha;
        }
        m[g] = sdot;
      }
      const float p = exp2f(sdot - m[g]);
      l[g] += p;
      tt[g] = fmaf(p, sdot - m[g], tt[g]);
#pragma unroll
      for (int e = 0; e < E8; ++e) o[g][e] = fmaf(p, vx[e], o[g][e]);
    }
    cur = nxt;
    tcur = tn;
  }
  // merge the warp's four token groups (lanes sl, sl + 8, sl + 16, sl + 24)
#pragma unroll
  for (int off = 8; off <= 16; off <<= 1) {
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[g], off);
      const float lo = __shfl_xor_sync(0xffffffffu, l[g], off);
      const float to = __shfl_xor_sync(0xffffffffu, tt[g], off);
      const float M = fmaxf(m[g], mo);
      const float a = m[g] == kNegInf ? 0.f : exp2f(m[g] - M);
      const float bb = mo == kNegInf ? 0.f : exp2f(mo - M);
      const float tn = (m[g] == kNegInf ? 0.f : a * (tt[g] + l[g] * (m[g] - M))) +
                       (mo == kNegInf ? 0.f : bb * (to + lo * (mo - M)));
      l[g] = l[g] * a + lo * bb;
      tt[g] = tn;
#pragma unroll
      for (int e = 0; e < E8; ++e) {
        const float oo = __shfl_xor_sync(0xffffffffu, o[g][e], off);
        o[g][e] = o[g][e] * a + oo * bb;
      }
      m[g] = M;
    }
  }
  // the W warps' partials -> one per (split, query head), through shared memory
  __shared__ float s_mlt[W][GC][3];
  __shared__ float s_o[W][GC][D];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    if (lane == 0) {
      s_mlt[warp][g][0] = m[g];
      s_mlt[warp][g][1] = l[g];
      s_mlt[warp][g][2] = tt[g];
    }
    if (grp == 0) {
#pragma unroll
      for (int e = 0; e < E8; ++e) s_o[warp][g][e0 + e] = o[g][e];
    }
  }
  __syncthreads();
  const size_t rec = 3 + D;  // m, l, t, o[D] per (sequence, query head, split)
  const int Hq = static_cast<int>(c.kv_heads) * G;
  for (int idx = threadIdx.x; idx < GC * (D + 1); idx += kKvThreads) {
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
