// Scalar-gated scan over dim 1 of [B, T, D] (the third-party assoc_scan.AssocScan
// the reference calls at rnn_memory.py:189,363-379 and omega.py:315):
//   h_t = a[b,t] h_{t-1} + x[b,t,:],  h_0 = prev[b,:] (or 0),  outputs h_1..h_T,
// prev prepended when it is given and remove_prev is false.
// One thread per trailing element d (grid (ceil(D / 256), B)), sequential in t
// with the inputs of four steps loaded ahead; the backward runs the transposed
// recurrence from the last step down and reduces the gate gradient
// d a_t = sum_d g_t[d] h_{t-1}[d] by warp shuffles and one atomic per warp.
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
  const int64_t d = (int64_t)blockIdx.x * kScanOpThreads + threadIdx.x, b = b0 + blockIdx.y;
  const bool valid = d < D;  // every lane takes part in the shuffles
  const int lane = threadIdx.x & 31;
  const float* ab = a + b * T;
  const IO* ob = out + (b * (T + off) + off) * D + d;  // ob[t D] = h_{t+1}
  const IO* gb = dout + (b * (T + off) + off) * D + d;
  IO* xb = dx + b * T * D + d;
  const float h0 = valid && prev ? prev[b * D + d] : 0.f;
  float g = 0.f;
  for (int64_t t = T - 1; t >= 0; --t) {
    const float up = valid ? io_ld(gb, t * D) : 0.f;
    g = up + (t + 1 < T ? ab[t + 1] * g : 0.f);
    if (valid) io_st(xb, t * D, g);
    const float hp = !valid ? 0.f : (t > 0 ? io_ld(ob, (t - 1) * D) : h0);  // h_t, the state step t reads
    float p = g * hp;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
    if (lane == 0 && p != 0.f) atomicAdd(&da[b * T + t], p);
  }
  if (valid && dprev) {
    float v = ab[0] * g;
    if (off) v += io_ld(dout, b * (T + 1) * D + d);
    dprev[b * D + d] = v;
  }
}

}  // namespace atlas
