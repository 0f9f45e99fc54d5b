// The per-parameter update of the legacy OmegaNeuralMemory.store_memories
// (omega.py:262-315) in one pass over the [B, T, D] surprises (B = batch*heads,
// T = chunks, D = the parameter's elements):
//
//   m_t = beta_t m_{t-1} + s_t,   m_0 = last momentum          (omega.py:262-268)
//   g_t = u_t m_t                  (omega gate, per (b, t))      (omega.py:276-283)
//   w_t = sum_{j<e} g_{t-j},  g_{-1..-(e-1)} = the carried buffer (omega.py:285-298)
//   h_t = a_t h_{t-1} + w_t,      h_0 = last update, a_t = 1 - decay_t (omega.py:315)
//
// outputs h_0..h_T (prev kept, remove_prev=False), m_T (the next last momentum)
// and the new buffer (the last e-1 entries of [buffer; g]). Momentum and gate
// are optional. One thread per element d, sequential in t; the previous e-1
// window terms live in registers. The backward runs the transposed recurrences
// from t = T-1 down and reduces the per-(b, t) gradients of beta, u and a over
// the elements by warp shuffles and one atomic per warp and step.
#pragma once
#include "scan_op.cuh"

namespace atlas {

constexpr int kOmegaMaxWindow = 16;

struct OmegaStoreArgs {
  const float *beta, *u, *a;  // [B, T] (beta / u may be NULL)
  const void* s;              // [B, T, D] surprises (io)
  const float *m0, *buf, *h0; // [B, D], [B, e-1, D], [B, D] (may be NULL = zeros / no prev)
  void* out;                  // [B, T + off, D] io: h (h_0 first when h0 is given)
  float* m_all;               // [B, T, D] momentum sequence for the backward (or NULL)
  float *m_last, *buf_out;    // [B, D], [B, e-1, D]
  // backward
  const void* dout;           // [B, T + off, D] io
  const float *dm_last, *dbuf_out;  // may be NULL
  void* ds;                   // [B, T, D] io
  float *dbeta, *du, *da;     // [B, T] (zeroed by the caller's entry point)
  float *dm0, *dh0, *dbuf;    // [B, D], [B, D], [B, e-1, D] (may be NULL)
  int64_t B, T, D;
  int e, off;
};

template <class IO>
__global__ void __launch_bounds__(kScanOpThreads) k_omega_store_fwd(OmegaStoreArgs A) {
  const int64_t d = (int64_t)blockIdx.x * kScanOpThreads + threadIdx.x, b = blockIdx.y;
  if (d >= A.D) return;
  const int64_t T = A.T, D = A.D;
  const int e1 = A.e - 1;
  float hist[kOmegaMaxWindow];  // hist[0] = g_{t-1}, hist[1] = g_{t-2}, ...
#pragma unroll
  for (int j = 0; j < kOmegaMaxWindow; ++j) {
    const int i = e1 - 1 - j;  // buffer entry i is g_{i - (e-1)}
    hist[j] = (j < e1 && A.buf) ? A.buf[(b * e1 + i) * D + d] : 0.f;
  }
  float m = A.m0 ? A.m0[b * D + d] : 0.f;
  float h = A.h0 ? A.h0[b * D + d] : 0.f;
  const IO* sb = reinterpret_cast<const IO*>(A.s) + b * T * D + d;
  IO* ob = reinterpret_cast<IO*>(A.out) + b * (T + A.off) * D + d;
  if (A.off) io_st(ob, 0, h);
  for (int64_t t = 0; t < T; ++t) {
    const float sv = io_ld(sb, t * D);
    m = A.beta ? A.beta[b * T + t] * m + sv : sv;
    if (A.m_all) A.m_all[(b * T + t) * D + d] = m;
    const float g = A.u ? A.u[b * T + t] * m : m;
    float w = g;
#pragma unroll
    for (int j = 0; j < kOmegaMaxWindow; ++j) if (j < e1) w += hist[j];
#pragma unroll
    for (int j = kOmegaMaxWindow - 1; j > 0; --j) hist[j] = hist[j - 1];
    hist[0] = g;
    h = A.a[b * T + t] * h + w;
    io_st(ob, (t + A.off) * D, h);
  }
  if (A.m_last) A.m_last[b * D + d] = m;
  if (A.buf_out)
#pragma unroll
    for (int j = 0; j < kOmegaMaxWindow; ++j)
      if (j < e1) A.buf_out[(b * e1 + (e1 - 1 - j)) * D + d] = hist[j];
}

// Warp sum of v, added to *dst by lane 0 (skipped when the warp's sum is zero).
__device__ __forceinline__ void warp_atomic(float* dst, float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0 && v != 0.f) atomicAdd(dst, v);
}

template <class IO>
__global__ void __launch_bounds__(kScanOpThreads) k_omega_store_bwd(OmegaStoreArgs A) {
  const int64_t d = (int64_t)blockIdx.x * kScanOpThreads + threadIdx.x, b = blockIdx.y;
  const bool valid = d < A.D;  // every thread takes part in the shuffles
  const int64_t T = A.T, D = A.D, dd = valid ? d : 0;
  const int e1 = A.e - 1;
  const IO* ob = reinterpret_cast<const IO*>(A.out) + b * (T + A.off) * D + dd;   // ob[(t + off) D] = h_t
  const IO* gob = reinterpret_cast<const IO*>(A.dout) + b * (T + A.off) * D + dd;
  IO* dsb = reinterpret_cast<IO*>(A.ds) + b * T * D + dd;
  const float h0 = (valid && A.h0) ? A.h0[b * D + dd] : 0.f;
  const float m0 = (valid && A.m0) ? A.m0[b * D + dd] : 0.f;
  float fut[kOmegaMaxWindow];   // fut[j] = dw_{t+1+j}
  float bacc[kOmegaMaxWindow];  // d buffer entry i (the part from the windows)
#pragma unroll
  for (int j = 0; j < kOmegaMaxWindow; ++j) { fut[j] = 0.f; bacc[j] = 0.f; }
  float dh = 0.f, dm = 0.f;
  for (int64_t t = T - 1; t >= 0; --t) {
    const float anext = t + 1 < T ? A.a[b * T + t + 1] : 0.f;
    dh = (valid ? io_ld(gob, (t + A.off) * D) : 0.f) + anext * dh;
    const float hprev = !valid ? 0.f : (t > 0 ? io_ld(ob, (t - 1 + A.off) * D) : h0);
    warp_atomic(&A.da[b * T + t], dh * hprev);
    const float dw = dh;
    // window: g_t feeds w_t .. w_{t+e-1}; the new buffer holds g_t when t >= T - (e-1)
    float dg = dw;
#pragma unroll
    for (int j = 0; j < kOmegaMaxWindow; ++j) if (j < e1 && t + 1 + j < T) dg += fut[j];
    if (A.dbuf_out && valid && t + e1 >= T) dg += A.dbuf_out[(b * e1 + (t + e1 - T)) * D + dd];
#pragma unroll
    for (int j = kOmegaMaxWindow - 1; j > 0; --j) fut[j] = fut[j - 1];
    fut[0] = dw;
    // old buffer entry i (i < e-1) lies in the windows of w_0 .. w_i
#pragma unroll
    for (int i = 0; i < kOmegaMaxWindow; ++i) if (i < e1 && t <= i) bacc[i] += dw;
    const float mt = (valid && A.m_all) ? A.m_all[(b * T + t) * D + dd] : (valid ? io_ld(
        reinterpret_cast<const IO*>(A.s) + b * T * D + dd, t * D) : 0.f);
    float dmg = dg;
    if (A.u) {
      warp_atomic(&A.du[b * T + t], dg * mt);
      dmg = A.u[b * T + t] * dg;
    }
    if (A.beta) {
      const float bnext = t + 1 < T ? A.beta[b * T + t + 1] : 0.f;
      dm = dmg + bnext * dm + ((t == T - 1 && A.dm_last && valid) ? A.dm_last[b * D + dd] : 0.f);
      const float mprev = !valid ? 0.f : (t > 0 ? A.m_all[(b * T + t - 1) * D + dd] : m0);
      warp_atomic(&A.dbeta[b * T + t], dm * mprev);
      if (valid) io_st(dsb, t * D, dm);
    } else {
      if (valid) io_st(dsb, t * D, dmg);
    }
  }
  if (!valid) return;
  if (A.dm0) A.dm0[b * D + d] = A.beta ? A.beta[b * T] * dm : 0.f;
  if (A.dh0) A.dh0[b * D + d] = A.a[b * T] * dh + (A.off ? io_ld(reinterpret_cast<const IO*>(A.dout) + b * (T + 1) * D + d, 0) : 0.f);
  if (A.dbuf)
#pragma unroll
    for (int i = 0; i < kOmegaMaxWindow; ++i)
      if (i < e1) {
        float v = bacc[i];
        if (A.dbuf_out && i >= T) v += A.dbuf_out[(b * e1 + (i - T)) * D + d];
        A.dbuf[(b * e1 + i) * D + d] = v;
      }
}

}  // namespace atlas
