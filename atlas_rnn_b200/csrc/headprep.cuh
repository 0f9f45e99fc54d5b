// Head preparation of the memory cells in one pass: the projection output
// t [B, T, H * d] (row-major, heads side by side) is split into heads, optionally
// RMS-normalised per head with a learned gain (MultiheadRMSNorm, rnn_memory.py:139-147:
// y = x / max(||x|| d^-1/2, 1e-8) * gamma[h]), cast, and written as
// o [B * H, T, Dp] with zero columns d .. Dp-1 (Dp = 128 feeds the tensor-core
// kernels with 64-wide heads zero-padded).
// Backward: dt (the same split, transposed back) and d gamma [H, d]:
//   m = max(s n, 1e-8), n = ||x||, s = d^-1/2
//   dx_j = g_j gamma_j / m - x_j (sum_i g_i gamma_i x_i) / (s n^3)   (m > 1e-8)
//   dx_j = g_j gamma_j / 1e-8                                         (clamped)
//   d gamma_j = sum over rows of g_j x_j / m
// A warp owns one row (b, t, h) at a time, each lane kHpPer = d / 32 elements
// (d = 32, 64, 96 or 128); a CTA takes one head h and kHpRows consecutive (b, t)
// rows, so d gamma is summed in registers, across the CTA's warps in shared
// memory, and added with one atomic per element and CTA.
#pragma once
#include "common.cuh"

namespace atlas {

constexpr int kHpWarps = 8;
constexpr int kHpRows = 128;  // (b, t) rows per CTA

template <class T>
__device__ __forceinline__ float hp_ld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float hp_ld<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float hp_ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
__device__ __forceinline__ void hp_st(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void hp_st(__nv_bfloat16* p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// grid (H, ceil(B * T / kHpRows)), kHpWarps * 32 threads
template <int PER, class I, class O>
__global__ void __launch_bounds__(kHpWarps * 32) k_head_prep_fwd(const I* t, const float* gamma, O* o, int64_t BT,
                                                                 int64_t T, int H, int Dp) {
  constexpr int d = PER * 32;
  const int h = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float s = rsqrtf((float)d);
  float gm[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) gm[i] = gamma ? gamma[h * d + lane + 32 * i] : 1.f;
  const int64_t r0 = (int64_t)blockIdx.y * kHpRows;
  for (int64_t r = r0 + warp; r < r0 + kHpRows && r < BT; r += kHpWarps) {
    const int64_t b = r / T, tt = r - b * T;
    const I* src = t + (r * H + h) * d;
    float x[PER], ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      x[i] = hp_ld(src, lane + 32 * i);
      ss += x[i] * x[i];
    }
    float scale = 1.f;
    if (gamma) scale = 1.f / fmaxf(sqrtf(warp_sum(ss)) * s, 1e-8f);
    O* dst = o + ((b * H + h) * T + tt) * Dp;
#pragma unroll
    for (int i = 0; i < PER; ++i) hp_st(dst, lane + 32 * i, x[i] * scale * gm[i]);
    for (int c = d + lane; c < Dp; c += 32) hp_st(dst, c, 0.f);
  }
}

template <int PER, class I, class O>
__global__ void __launch_bounds__(kHpWarps * 32) k_head_prep_bwd(const I* t, const float* gamma, const O* g,
                                                                 I* dt, float* dgamma, int64_t BT, int64_t T, int H,
                                                                 int Dp) {
  constexpr int d = PER * 32;
  __shared__ float red[kHpWarps][d];
  const int h = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float s = rsqrtf((float)d);
  float gm[PER], dg[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    gm[i] = gamma ? gamma[h * d + lane + 32 * i] : 1.f;
    dg[i] = 0.f;
  }
  const int64_t r0 = (int64_t)blockIdx.y * kHpRows;
  for (int64_t r = r0 + warp; r < r0 + kHpRows && r < BT; r += kHpWarps) {
    const int64_t b = r / T, tt = r - b * T;
    const I* src = t + (r * H + h) * d;
    const O* gsrc = g + ((b * H + h) * T + tt) * Dp;
    float x[PER], gy[PER], ss = 0.f, dot = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      x[i] = hp_ld(src, lane + 32 * i);
      gy[i] = hp_ld(gsrc, lane + 32 * i);
      ss += x[i] * x[i];
      dot += gy[i] * gm[i] * x[i];
    }
    I* dst = dt + (r * H + h) * d;
    if (!gamma) {
#pragma unroll
      for (int i = 0; i < PER; ++i) hp_st(dst, lane + 32 * i, gy[i]);
      continue;
    }
    const float n = sqrtf(warp_sum(ss)), m = n * s;
    dot = warp_sum(dot);
    const bool clamped = !(m > 1e-8f);
    const float inv = 1.f / (clamped ? 1e-8f : m);
    const float corr = clamped ? 0.f : dot / (s * n * n * n);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      hp_st(dst, lane + 32 * i, gy[i] * gm[i] * inv - x[i] * corr);
      dg[i] += gy[i] * x[i] * inv;
    }
  }
  if (!dgamma) return;
#pragma unroll
  for (int i = 0; i < PER; ++i) red[warp][lane + 32 * i] = dg[i];
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += kHpWarps * 32) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kHpWarps; ++w) v += red[w][c];
    atomicAdd(&dgamma[h * d + c], v);
  }
}

}  // namespace atlas
