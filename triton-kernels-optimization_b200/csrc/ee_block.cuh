// ee_block.cuh - the elementwise work of the Llama decoder block around the routed
// linears and the attention, one pass each (the reference runs them as chains of torch
// kernels: EE/python/dispatch.py:166-210 with transformers' LlamaRMSNorm,
// apply_rotary_pos_emb and the residual adds):
//   * add_rmsnorm_kernel: s = fp16(residual + x) (optional, also stored), then
//     y = fp16(w * fp16(fp32(s) * rsqrt(mean(fp32(s)^2) + eps)));
//   * rope_layout_kernel: q / k rows of the projections -> rotary embedding with the
//     fp16 roundings of (q * cos) + (rotate_half(q) * sin) -> the [B, H, S, D] layouts the
//     flash-attention kernel reads;
//   * transpose_v_kernel: V from any [B, S, Hkv, D]-strided layout -> V^T [B*Hkv, D, S_pad].
// Included once, by ee_kernels.cu.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "ee_internal.h"
#include "ee_ptx.cuh"

namespace ee {

// ----------------------------------------------------------------------------------
// residual add + RMSNorm.  TPR threads per row (a multiple of 32, 256-thread blocks),
// NV 16-byte vectors per thread: rows up to TPR * NV * 8 columns, kept in registers.
// ----------------------------------------------------------------------------------
constexpr int kNormThreads = 256;

template <int TPR>
__device__ __forceinline__ float norm_group_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if constexpr (TPR > 32) {
    constexpr int WPR = TPR / 32;
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    const int g0 = (w / WPR) * WPR;
    float r = 0.f;
#pragma unroll
    for (int i = 0; i < WPR; ++i) r += red[g0 + i];
    v = r;
  }
  return v;
}

template <int TPR, int NV>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(const AddNormArgs a) {
  griddep_wait();  // the inputs may come from the previous kernel in the stream
  griddep_launch_dependents();
  constexpr int RPB = kNormThreads / TPR;
  __shared__ float red[kNormThreads / 32];
  const int g = threadIdx.x / TPR, lt = threadIdx.x % TPR;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * RPB + g;
  const bool ok = row < a.M;
  const int d = a.d;
  uint4 u[NV];
  float ss = 0.f;
  const __half* xr = a.x + (ok ? row : 0) * a.ldx;
  const __half* rr = a.res ? a.res + (ok ? row : 0) * a.ldr : nullptr;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int e0 = (lt + i * TPR) * 8;
    const bool in = ok && e0 < d;
    uint4 v = in ? __ldcs(reinterpret_cast<const uint4*>(xr + e0)) : make_uint4(0u, 0u, 0u, 0u);
    if (rr != nullptr && in) {  // s = fp16(residual + x): torch's half add
      const uint4 r = __ldcs(reinterpret_cast<const uint4*>(rr + e0));
      __half2* hv = reinterpret_cast<__half2*>(&v);
      const __half2* hr = reinterpret_cast<const __half2*>(&r);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 fx = __half22float2(hv[k]), fr = __half22float2(hr[k]);
        hv[k] = __floats2half2_rn(fr.x + fx.x, fr.y + fx.y);
      }
      if (a.sum_out) __stcs(reinterpret_cast<uint4*>(a.sum_out + row * a.lds + e0), v);
    }
    u[i] = v;
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(h[k]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  ss = norm_group_sum<TPR>(ss, red);
  // torch: mean = sum * (1 / d); rsqrt(mean + eps); fp32 product rounded to fp16; times w
  const float r = rsqrtf(ss * (1.f / static_cast<float>(d)) + a.eps);
  if (!ok) return;
  __half* yr = a.y + row * a.ldy;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int e0 = (lt + i * TPR) * 8;
    if (e0 < d) {
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(a.w + e0));
      const __half2* h = reinterpret_cast<const __half2*>(&u[i]);
      const __half2* hw = reinterpret_cast<const __half2*>(&wv);
      uint4 o;
      __half2* ho = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h[k]);
        const float2 n = __half22float2(__floats2half2_rn(f.x * r, f.y * r));
        const float2 w = __half22float2(hw[k]);
        ho[k] = __floats2half2_rn(w.x * n.x, w.y * n.y);
      }
      __stcs(reinterpret_cast<uint4*>(yr + e0), o);
    }
  }
}

// ----------------------------------------------------------------------------------
// rotary embedding + head layout.  One 256-thread block per token (b, s): thread t
// takes 16-byte vectors t, t + 256, ... of the token's q row (Hq heads of D) and then of
// its k row (Hkv heads): element j of a head becomes
//   fp16( fp16(x_j * cos_j) + fp16(rot_j * sin_j) ),  rot_j = -x_{j+D/2} (j < D/2), x_{j-D/2}
// -- transformers' (q * cos) + (rotate_half(q) * sin) on fp16 tensors, each product and
// the sum rounded to fp16 -- and is stored at [b, h, s, j] of Q / K (the flash kernel's
// row-major [B*H*S, D] operands).
// ----------------------------------------------------------------------------------
__device__ __forceinline__ uint4 rope_vec(const uint4& x, const uint4& partner, bool low_half, const uint4& c,
                                          const uint4& sn) {
  const __half2* hx = reinterpret_cast<const __half2*>(&x);
  const __half2* hp = reinterpret_cast<const __half2*>(&partner);
  const __half2* hc = reinterpret_cast<const __half2*>(&c);
  const __half2* hs = reinterpret_cast<const __half2*>(&sn);
  uint4 o;
  __half2* ho = reinterpret_cast<__half2*>(&o);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 fx = __half22float2(hx[k]), fp = __half22float2(hp[k]);
    const float2 fc = __half22float2(hc[k]), fs = __half22float2(hs[k]);
    const float2 rot = low_half ? make_float2(-fp.x, -fp.y) : fp;  // negation is exact
    const float2 a = __half22float2(__floats2half2_rn(fx.x * fc.x, fx.y * fc.y));
    const float2 b = __half22float2(__floats2half2_rn(rot.x * fs.x, rot.y * fs.y));
    ho[k] = __floats2half2_rn(a.x + b.x, a.y + b.y);
  }
  return o;
}

template <int D>
__global__ void __launch_bounds__(256) rope_layout_kernel(const RopeArgs a) {
  griddep_wait();  // the projections come from the previous kernels in the stream
  griddep_launch_dependents();
  constexpr int VPH = D / 8;  // 16-byte vectors per head
  const int64_t tok = blockIdx.x;  // b * S + s
  const int64_t b = tok / a.S, s = tok % a.S;
  const __half* cs = a.cos + tok * a.ld_cs;
  const __half* sn = a.sin + tok * a.ld_cs;
  const int nq = a.Hq * VPH, nk = a.Hkv * VPH;
  for (int v = threadIdx.x; v < nq + nk; v += 256) {
    const bool is_q = v < nq;
    const int vv = is_q ? v : v - nq;
    const int h = vv / VPH, j0 = (vv % VPH) * 8;
    const __half* src = is_q ? a.q + tok * a.ldq + h * D : a.k + tok * a.ldk + h * D;
    const bool low = j0 < D / 2;
    const uint4 x = *reinterpret_cast<const uint4*>(src + j0);
    const uint4 p = *reinterpret_cast<const uint4*>(src + (low ? j0 + D / 2 : j0 - D / 2));
    const uint4 c = __ldg(reinterpret_cast<const uint4*>(cs + j0));
    const uint4 sv = __ldg(reinterpret_cast<const uint4*>(sn + j0));
    const uint4 o = rope_vec(x, p, low, c, sv);
    const int64_t H = is_q ? a.Hq : a.Hkv;
    __half* dst = (is_q ? a.q_out : a.k_out) + (((b * H + h) * a.S + s) * D + j0);
    *reinterpret_cast<uint4*>(dst) = o;
  }
}

// ----------------------------------------------------------------------------------
// V -> V^T [B*Hkv, D, S_pad] (zero past S): the P V operand, K-major.  V element
// (b, h, s, c) sits at V + b * sb + h * sh + s * ss + c, so both a contiguous
// [B, Hkv, S, D] tensor and the v projection's [B, S, Hkv * D] rows are read in place.
// ----------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) transpose_v_kernel(const __half* __restrict__ V, int64_t Hkv, int64_t S,
                                                          int64_t S_pad, int64_t sb, int64_t sh, int64_t ss,
                                                          __half* __restrict__ VT) {
  __shared__ __half tile[32][D + 2];
  const int64_t head = blockIdx.y;  // b * Hkv + h
  const int64_t b = head / Hkv, h = head % Hkv;
  const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32;
  griddep_wait();
  const __half* vb = V + b * sb + h * sh;
  for (int i = threadIdx.x; i < 32 * D; i += 256) {
    const int r = i / D, c = i % D;
    const int64_t k = k0 + r;
    tile[r][c] = k < S ? vb[k * ss + c] : __float2half(0.f);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 32 * D; i += 256) {
    const int c = i / 32, r = i % 32;
    const int64_t k = k0 + r;
    if (k < S_pad) VT[(head * D + c) * S_pad + k] = tile[r][c];
  }
}

// ----------------------------------------------------------------------------------
// Router inputs of the decoder block from the attention's row entropies H [B, Hq, S]:
//   * head_mean_kernel: per query position the mean over the heads,
//     out[b * S + s] = (sum_h H[b, h, s]) / Hq, heads added in ascending order -- the
//     per-token entropy that routes that token's rows;
//   * batch_max_fill_kernel: every one of M positions gets max_b Hb[b] (the per-batch
//     means, B of them), so routing those values puts all rows in the tier the
//     reference's dispatcher picks from the batch max (EE/python/dispatch.py:63-79).
// ----------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) head_mean_kernel(const float* __restrict__ H, int64_t B, int64_t Hq,
                                                        int64_t S, float* __restrict__ out) {
  griddep_wait();  // the row entropies come from the previous kernel in the stream
  griddep_launch_dependents();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;  // b * S + s
  if (i >= B * S) return;
  const int64_t b = i / S, s = i - b * S;
  const float* h = H + b * Hq * S + s;
  float acc = 0.f;
  for (int64_t k = 0; k < Hq; ++k) acc += h[k * S];
  out[i] = __fdiv_rn(acc, static_cast<float>(Hq));
}

__global__ void __launch_bounds__(256) batch_max_fill_kernel(const float* __restrict__ Hb, int64_t B,
                                                             float* __restrict__ out, int64_t M) {
  griddep_wait();
  griddep_launch_dependents();
  float m = Hb[0];
  for (int64_t b = 1; b < B; ++b) m = fmaxf(m, Hb[b]);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < M; i += static_cast<int64_t>(gridDim.x) * 256)
    out[i] = m;
}

// out[i] = v for i < M (the router input of rows that must all take one tier, e.g. +inf:
// FP16 for the first layer's projections, which have no earlier entropy)
__global__ void __launch_bounds__(256) fill_value_kernel(float* __restrict__ out, int64_t M, float v) {
  griddep_wait();
  griddep_launch_dependents();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < M; i += static_cast<int64_t>(gridDim.x) * 256)
    out[i] = v;
}

}  // namespace ee
