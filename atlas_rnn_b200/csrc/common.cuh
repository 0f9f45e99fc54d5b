// Shared device helpers for the memory-update kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "atlas_mem.h"

namespace atlas {

constexpr int kThreads = 256;  // every CTA of the SIMT path runs 256 threads

// Everything a kernel needs, passed by value (well under the 4 KB limit).
struct Params {
  // tensor-core path: TMA descriptors of the bf16 row-major [N, T, 128] operands
  // (q, k, dy, and the saved delta rows), viewed as 4-D (8 elements, T rows,
  // 16 column blocks, N units) so that a box of 8 rows lands in the
  // core-matrix tile layout; zero-filled outside each unit's rows
  alignas(64) CUtensorMap tm_q;
  alignas(64) CUtensorMap tm_k;
  alignas(64) CUtensorMap tm_dy;
  alignas(64) CUtensorMap tm_dl;
  // shape
  int N, T, dk, dphi, dv, e, fmode, fdeg, gmode, mom, bf, C, nch;
  // forward operands
  const void *k, *q, *v, *lr, *decay, *beta, *gate;
  const float *Sref, *S0, *Z0, *buf, *proj;
  void* y;
  float *S_end, *Z_end, *buf_out;
  // backward operands
  const void* dy;
  const float *dS_end, *dZ_end, *dbuf_out;
  void *dk_, *dq_, *dv_, *dlr, *ddecay, *dbeta, *dgate;
  float *dSref, *dS0, *dZ0, *dbuf;
  // saved workspace (forward -> backward)
  float *st;     // [N][nch][2][dv][dphi]: chunk deltas, then chunk-start S, Z
  float *delta;  // [N][T][dv]  delta_t = S_ref phi_t - v_t
  float *ST;     // [N][dv][dphi] unclamped S_T (clamp mask of the backward)
  float *cs;     // [N][nch][4] chunk transform scalars (a, b, c)
  float *phik, *phiq;  // [N][T][dphi] tensor feature map only
  unsigned char* projb;  // tensor feature map on tensor cores: Proj as dk + 1 bf16 tiles of dk x dphi
  int fm_bf16;           // stand-alone feature map: phi out / d phi in as bf16 (else fp32)
  // backward scratch
  float *adj;    // [N][nch][2][dv][dphi]: adjoint deltas, then adjoint at chunk end
  float *acs;    // [N][nch][4]
  float *dpsi;   // [N][T][dphi]
  float *ddel;   // [N][T][dv]
  float *dphiR;  // [N][T][dphi]
  float *hdd;    // [N][nch][e-1][dv]   halo partials of d delta
  float *hdp;    // [N][nch][e-1][dphi] halo partials of d phi
  float *du;     // [N][T]
  float *hdu;    // [N][nch][e-1]
  float *xq, *xf, *xs;  // Gram pieces of the tensor-core backward
  // tensor-core path: bf16 copies the chunk kernels read as raw 16-byte units
  __nv_bfloat16* dlb;   // [N][T][dv] delta (replaces `delta`)
  unsigned char* stb;   // [N][nch][2] 128x128 bf16 tiles of the chunk-start S, Z
  unsigned char* srb;   // [N] S_ref as a 128x128 bf16 operand tile
  unsigned char* adjb;  // [N][nch][2] 128x128 bf16 tiles of the adjoint at each chunk end
  int inc_bf16;         // chunk increments in `st` / `adj` are bf16 (tensor-core path)
  void* gt;             // [N][nch] 128x128 bf16 Gram blocks (core-matrix tile layout)
  __nv_bfloat16* ddb;   // [N][T][dv]   d delta of each chunk's own keys (bf16 hand-off to finalize)
  __nv_bfloat16* dpb;   // [N][T][dphi] d phi of each chunk's own keys (bf16 hand-off to finalize)
  __nv_bfloat16* dpsib; // [N][T][dphi] d psi (tensor-core path: keys part, then + state part)
  int apply_mask;
  // sequence-parallel segment outputs
  float *seg_coef, *seg_dS, *seg_dZ;
  // caller's device status word (NULL = none): bounded waits that ran out
  int* status;
};

__device__ __forceinline__ float ldio(const void* p, int64_t i, int bf) {
  return bf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
            : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void stio(void* p, int64_t i, float x, int bf) {
  if (bf) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else reinterpret_cast<float*>(p)[i] = x;
}

// Elementwise polynomial feature map phi(x) = sum_{i=1..g} x^i, evaluated in
// the reference's order (rnn_memory.py:117-123), and its derivative.
__device__ __forceinline__ float fmap_elem(float x, int mode, int deg) {
  if (mode != ATLAS_FMAP_ELEMENTWISE || deg <= 1) return x;
  float out = x, pw = x;
  for (int i = 2; i <= deg; ++i) { pw = pw * x; out = out + pw; }
  return out;
}
__device__ __forceinline__ float fmap_elem_grad(float x, int mode, int deg) {
  if (mode != ATLAS_FMAP_ELEMENTWISE || deg <= 1) return 1.f;
  float d = 1.f, pw = 1.f;
  for (int i = 2; i <= deg; ++i) { pw = pw * x; d += (float)i * pw; }
  return d;
}

// delta of row `row` (= n*T + t), component nn, from whichever copy is kept.
__device__ __forceinline__ float delta_at(const Params& P, int64_t row, int nn) {
  return P.dlb ? __bfloat162float(P.dlb[row * P.dv + nn]) : P.delta[row * P.dv + nn];
}

// phi of token `t` (key side if !isq), component m.
__device__ __forceinline__ float load_phi(const Params& P, int n, int t, int m, bool isq) {
  const int64_t row = (int64_t)n * P.T + t;
  if (P.fmode == ATLAS_FMAP_TENSOR) return (isq ? P.phiq : P.phik)[row * P.dphi + m];
  return fmap_elem(ldio(isq ? P.q : P.k, row * P.dk + m, P.bf), P.fmode, P.fdeg);
}

// ---------------------------------------------------------------------------
// Block GEMM on CUDA cores (fp32 FFMA), 256 threads, 64x64 output tiles,
// operands staged through shared memory in k-slices of 16.
//   out(m, n) = sum over segments s of sum_{k < s.K} s.A(m, k) * s.B(k, n)
// The epilogue epi(m, n, acc) is called once per output element by a thread
// that depends only on (M, N, m, n), so successive calls with equal (M, N)
// may read-modify-write the same element from the same thread without a
// barrier. Every thread of the CTA must call it. `stage` holds 2*16*68 floats.
// ---------------------------------------------------------------------------
template <class FA, class FB>
struct Seg {
  int K;
  FA A;
  FB B;
};
template <class FA, class FB>
__device__ __forceinline__ Seg<FA, FB> seg(int K, FA a, FB b) { return Seg<FA, FB>{K, a, b}; }

constexpr int kStageFloats = 2 * 16 * 68;

template <class S>
__device__ __forceinline__ void bgemm_run(const S& s, float (&acc)[4][4], int m0, int n0, int M,
                                          int N, float* As, float* Bs) {
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  for (int k0 = 0; k0 < s.K; k0 += 16) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int e = tid + kThreads * r;
      const int mm = e & 63, kk = e >> 6;
      const int k = k0 + kk;
      const int m = m0 + mm, n = n0 + mm;
      As[kk * 68 + mm] = (m < M && k < s.K) ? s.A(m, k) : 0.f;
      Bs[kk * 68 + mm] = (n < N && k < s.K) ? s.B(k, n) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk * 68 + ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk * 68 + tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
}

template <class Epi, class... S>
__device__ void bgemm(float* stage, int M, int N, Epi epi, const S&... segs) {
  float* As = stage;
  float* Bs = stage + 16 * 68;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  for (int m0 = 0; m0 < M; m0 += 64)
    for (int n0 = 0; n0 < N; n0 += 64) {
      float acc[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
      (bgemm_run(segs, acc, m0, n0, M, N, As, Bs), ...);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int m = m0 + ty + 16 * i, n = n0 + tx + 16 * j;
          if (m < M && n < N) epi(m, n, acc[i][j]);
        }
    }
}

// Block-wide sum; every thread gets the result. `red` holds 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (threadIdx.x < kThreads / 32) ? red[threadIdx.x] : 0.f;
  if (w == 0)
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

// Bump allocator over dynamic shared memory (floats).
// Phase clock for latency studies (built only with -DATLAS_PHASE_PROF): each
// mark() closes a phase at a block-wide barrier and adds its SM-clock cycles,
// summed over CTAs, to g_phase[slot]. Without the macro mark() is empty.
#ifdef ATLAS_PHASE_PROF
__device__ unsigned long long g_phase[64];
__device__ __forceinline__ long long sm_clock() {
  long long c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}
struct PhaseClock {
  long long t;
  __device__ PhaseClock() : t(sm_clock()) {}
  __device__ void mark(int slot) {
    __syncthreads();
    const long long now = sm_clock();
    if (threadIdx.x == 0) atomicAdd(&g_phase[slot], (unsigned long long)(now - t));
    t = now;
  }
  // cycles since the last mark, added by the calling thread (no barrier)
  __device__ void lap(int slot) { atomicAdd(&g_phase[slot], (unsigned long long)(sm_clock() - t)); }
};
#else
struct PhaseClock {
  __device__ void mark(int) {}
  __device__ void lap(int) {}
};
#endif

struct SmemAlloc {
  float* base;
  int off;
  __device__ float* take(int n) {
    float* p = base + off;
    off += (n + 3) & ~3;
    return p;
  }
};

}  // namespace atlas
