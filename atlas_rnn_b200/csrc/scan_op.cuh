// Scalar-gated scan over dim 1 of [B, T, D] (the third-party assoc_scan.AssocScan
// the reference calls at rnn_memory.py:189,363-379 and omega.py:315):
//   h_t = a[b,t] h_{t-1} + x[b,t,:],  h_0 = prev[b,:] (or 0),  outputs h_1..h_T,
// prev prepended when it is given and remove_prev is false.
// One thread per trailing element d (grid (ceil(D / 256), B)), sequential in t
// with the inputs of four steps loaded ahead; the backward runs the transposed
// recurrence from the last step down and reduces the gate gradient
// d a_t = sum_d g_t[d] h_{t-1}[d] by warp shuffles, shared memory across the
// CTA's warps every 32 steps, and one atomic per step and CTA.
#pragma once
#include "common.cuh"

namespace atlas {

constexpr int kScanOpThreads = 256;

template <class IO>
__device__ __forceinline__ float io_ld(const IO* p, int64_t i);
template <>
__device__ __forceinline__ float io_ld<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float io_ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
__device__ __forceinline__ void io_st(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void io_st(__nv_bfloat16* p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }

template <class IO>
__global__ void __launch_bounds__(kScanOpThreads) k_scan_op_fwd(const float* a, const IO* x, const float* prev,
                                                                IO* out, int64_t T, int64_t D, int off, int64_t b0) {
  const int64_t d = (int64_t)blockIdx.x * kScanOpThreads + threadIdx.x, b = b0 + blockIdx.y;
  if (d >= D) return;
  float h = prev ? prev[b * D + d] : 0.f;
  if (off) io_st(out, b * (T + 1) * D + d, h);
  const float* ab = a + b * T;
  const IO* xb = x + b * T * D + d;
  IO* ob = out + (b * (T + off) + off) * D + d;
  int64_t t = 0;
  for (; t + 4 <= T; t += 4) {
    float xv[4], av[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      xv[k] = io_ld(xb, (t + k) * D);
      av[k] = ab[t + k];
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      h = av[k] * h + xv[k];
      io_st(ob, (t + k) * D, h);
    }
  }
  for (; t < T; ++t) {
    h = ab[t] * h + io_ld(xb, t * D);
    io_st(ob, t * D, h);
  }
}

template <class IO>
__global__ void __launch_bounds__(kScanOpThreads) k_scan_op_bwd(const float* a, const IO* out, const float* prev,
                                                                const IO* dout, float* da, IO* dx, float* dprev,
                                                                int64_t T, int64_t D, int off, int64_t b0) {
  constexpr int kWarps = kScanOpThreads / 32, kTile = 32;
  __shared__ float part[kWarps][kTile];  // warp sums of d a_t for the last kTile steps
  const int64_t d = (int64_t)blockIdx.x * kScanOpThreads + threadIdx.x, b = b0 + blockIdx.y;
  const bool valid = d < D;  // every thread takes part in the shuffles and barriers
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* ab = a + b * T;
  const IO* ob = out + (b * (T + off) + off) * D + d;  // ob[t D] = h_{t+1}
  const IO* gb = dout + (b * (T + off) + off) * D + d;
  IO* xb = dx + b * T * D + d;
  const float h0 = valid && prev ? prev[b * D + d] : 0.f;
  float g = 0.f;
  auto step = [&](int64_t t, float up, float hp, float anext) {
    g = up + anext * g;
    if (valid) io_st(xb, t * D, g);
    float p = g * hp;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
    const int slot = (int)((T - 1 - t) % kTile);
    if (lane == 0) part[warp][slot] = p;
    if (slot == kTile - 1 || t == 0) {  // one atomic per step and CTA for the last (slot + 1) steps
      __syncthreads();
      if (threadIdx.x <= slot) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) sum += part[w][threadIdx.x];
        if (sum != 0.f) atomicAdd(&da[b * T + (t + slot - threadIdx.x)], sum);
      }
      __syncthreads();
    }
  };
  // h_t (the state step t reads) is out[t - 1] for t > 0 and prev for t = 0
  auto hprev = [&](int64_t t) { return !valid ? 0.f : (t > 0 ? io_ld(ob, (t - 1) * D) : h0); };
  int64_t t = T - 1;
  for (; t - 3 >= 0; t -= 4) {  // the inputs of four steps in flight before the dependent chain
    float up[4], hp[4], an[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      up[k] = valid ? io_ld(gb, (t - k) * D) : 0.f;
      hp[k] = hprev(t - k);
      an[k] = t - k + 1 < T ? ab[t - k + 1] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) step(t - k, up[k], hp[k], an[k]);
  }
  for (; t >= 0; --t) step(t, valid ? io_ld(gb, t * D) : 0.f, hprev(t), t + 1 < T ? ab[t + 1] : 0.f);
  if (valid && dprev) {
    float v = ab[0] * g;
    if (off) v += io_ld(dout, b * (T + 1) * D + d);
    dprev[b * D + d] = v;
  }
}

}  // namespace atlas
