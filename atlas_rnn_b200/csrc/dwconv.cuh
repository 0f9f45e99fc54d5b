// The q/k/v depthwise convolutions of the memory cells (rnn_memory.py:196-202,
// 334-340: Conv1d(dim, dim, K, padding=K//2, groups=dim, bias=False) applied to
// x^T, of which the first T outputs are used) as one pass over x in its own
// [B, T, C] layout, for all three weights at once:
//   y_m[b, t, c] = sum_j w_m[c, j] x[b, t + j - K/2, c]   (zero outside 0..T-1), m = q, k, v.
// Backward, in one pass as well:
//   dx[b, s, c]  = sum_m sum_j w_m[c, j] dy_m[b, s - j + K/2, c]   (dy zero outside 0..T-1)
//   dw_m[c, j]   = sum_{b,t} dy_m[b, t, c] x[b, t + j - K/2, c]
// A thread owns one channel and a run of kConvRun steps of one sequence, walking
// it with the K-tap window in registers; threads of a warp take consecutive
// channels, so every load and store of a warp is one contiguous row segment.
// The weight gradients are summed over the run in registers and added with one
// atomic per tap, weight and thread. HBM-bound: the forward reads x once (plus
// K - 1 halo steps per run) and writes three outputs.
#pragma once
#include "common.cuh"

namespace atlas {

constexpr int kConvThreads = 256;  // channels per CTA
constexpr int kConvRun = 256;      // steps per thread
constexpr int kConvMaxK = 8;

template <class T>
__device__ __forceinline__ float cv_ld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float cv_ld<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float cv_ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
__device__ __forceinline__ void cv_st(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void cv_st(__nv_bfloat16* p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }

// grid (ceil(C / kConvThreads), ceil(T / kConvRun), B)
template <int K, class X, class Y>
__global__ void __launch_bounds__(kConvThreads) k_dwconv3_fwd(const X* x, const float* wq, const float* wk,
                                                              const float* wv, Y* yq, Y* yk, Y* yv, int64_t T,
                                                              int64_t C) {
  constexpr int P = K / 2;
  const int64_t c = (int64_t)blockIdx.x * kConvThreads + threadIdx.x;
  if (c >= C) return;
  const int64_t b = blockIdx.z, t0 = (int64_t)blockIdx.y * kConvRun;
  const int64_t t1 = t0 + kConvRun < T ? t0 + kConvRun : T;
  float w[3][K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    w[0][j] = wq[c * K + j];
    w[1][j] = wk[c * K + j];
    w[2][j] = wv[c * K + j];
  }
  const X* xb = x + b * T * C + c;
  const int64_t ob = b * T * C + c;
  // win[j] = x[t + j - P] for the current t
  float win[K];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    const int64_t s = t0 + j - P;
    win[j] = (s >= 0 && s < T) ? cv_ld(xb, s * C) : 0.f;
  }
#pragma unroll 8  // loads of later steps issue ahead of the window shifts
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t s = t + K - 1 - P;
    win[K - 1] = s < T ? cv_ld(xb, s * C) : 0.f;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      a0 += w[0][j] * win[j];
      a1 += w[1][j] * win[j];
      a2 += w[2][j] * win[j];
    }
    cv_st(yq, ob + t * C, a0);
    cv_st(yk, ob + t * C, a1);
    cv_st(yv, ob + t * C, a2);
#pragma unroll
    for (int j = 0; j < K - 1; ++j) win[j] = win[j + 1];
  }
}

// dx and the three weight gradients (dw accumulated into zeroed fp32 [3][C][K]).
template <int K, class X, class Y>
__global__ void __launch_bounds__(kConvThreads) k_dwconv3_bwd(const X* x, const float* wq, const float* wk,
                                                              const float* wv, const Y* dq, const Y* dk,
                                                              const Y* dv, X* dx, float* dw, int64_t T,
                                                              int64_t C) {
  constexpr int P = K / 2;
  const int64_t c = (int64_t)blockIdx.x * kConvThreads + threadIdx.x;
  if (c >= C) return;
  const int64_t b = blockIdx.z, s0 = (int64_t)blockIdx.y * kConvRun;
  const int64_t s1 = s0 + kConvRun < T ? s0 + kConvRun : T;
  float w[3][K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    w[0][j] = wq[c * K + j];
    w[1][j] = wk[c * K + j];
    w[2][j] = wv[c * K + j];
  }
  const int64_t base = b * T * C + c;
  const X* xb = x + base;
  // dx[s] = sum_j w[j] dy[s - j + P]: window g[m][i] = dy_m[s + P - (K - 1) + i], i = 0..K-1
  float g[3][K];
  auto ldy = [&](int64_t t, float& a, float& bq, float& cv) {
    if (t >= 0 && t < T) {
      a = cv_ld(dq, base + t * C);
      bq = cv_ld(dk, base + t * C);
      cv = cv_ld(dv, base + t * C);
    } else {
      a = bq = cv = 0.f;
    }
  };
#pragma unroll
  for (int i = 0; i < K - 1; ++i) ldy(s0 + P - (K - 1) + i, g[0][i], g[1][i], g[2][i]);
  float acc[3][K];
#pragma unroll
  for (int m = 0; m < 3; ++m)
#pragma unroll
    for (int j = 0; j < K; ++j) acc[m][j] = 0.f;
#pragma unroll 8
  for (int64_t s = s0; s < s1; ++s) {
    ldy(s + P, g[0][K - 1], g[1][K - 1], g[2][K - 1]);
    const float xs = cv_ld(xb, s * C);
    float d = 0.f;
#pragma unroll
    for (int m = 0; m < 3; ++m)
#pragma unroll
      for (int j = 0; j < K; ++j) {
        // dy_m[s + P - j] sits at window index K - 1 - j
        const float gy = g[m][K - 1 - j];
        d += w[m][j] * gy;
        acc[m][j] += gy * xs;  // x[s] meets dy[t] at tap j with t + j - P = s
      }
    cv_st(dx, base + s * C, d);
#pragma unroll
    for (int m = 0; m < 3; ++m)
#pragma unroll
      for (int i = 0; i < K - 1; ++i) g[m][i] = g[m][i + 1];
  }
#pragma unroll
  for (int m = 0; m < 3; ++m)
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (acc[m][j] != 0.f) atomicAdd(&dw[((int64_t)m * C + c) * K + j], acc[m][j]);
}

}  // namespace atlas
