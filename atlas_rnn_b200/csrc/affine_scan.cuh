// Right-affine matrix scan, the drop-in of the reference's
// affine_associative_scan (affine_scan.py:36-160, composition rule :7-33):
//
//   H_t = H_{t-1} A_t + B_t,   H_{-1} = prev (or 0),   A_t [D, D], B_t, H_t [R, D]
//
// over t = 0 .. T-1 for N independent units, fp32. The reference composes the
// transforms in a log-depth tree ((A1, B1) o (A2, B2) = (A1 A2, B1 A2 + B2)),
// which costs O(T D^3) matrix products plus O(T) temporaries of [D, D]; the
// recurrence itself needs one [R, D] x [D, D] product per step, so this kernel
// runs it in order: one CTA per unit, H in shared memory, A_t staged by
// cp.async, each thread an 8 x 8 register tile of the product (FP32 FFMA; the
// results match the reference's fp32 arithmetic up to summation order).
//
// Backward (the transposed recurrence from the last step down):
//   G_t = dH_t + G_{t+1} A_{t+1}^T,  dA_t = H_{t-1}^T G_t,  dB_t = G_t,
//   d prev = dH_{-1} + G_0 A_0^T  (dH_{-1}: the gradient of the kept prev row).
#pragma once
#include "common.cuh"

namespace atlas {

constexpr int kAffThreads = 256;
constexpr int kAffMaxD = 128;

__device__ __forceinline__ void aff_cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void aff_wait() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  asm volatile("cp.async.wait_all;\n" ::: "memory");
}
// rows x cols fp32 (cols % 4 == 0) from global (row stride cols) into shared memory with row stride ld.
__device__ __forceinline__ void aff_load(float* dst, int ld, const float* src, int rows, int cols) {
  const int q = cols / 4;
  for (int u = threadIdx.x; u < rows * q; u += blockDim.x) aff_cp16(dst + (u / q) * ld + (u % q) * 4, src + u * 4);
}

// out[8x8 tile at (r0, c0)] = sum_k L(r, k) Rm(k, c) over k < K, for an R x C product.
template <class FL, class FR>
__device__ __forceinline__ void aff_tile(float (&acc)[8][8], int K, FL lhs, FR rhs) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int k = 0; k < K; ++k) {
    float a[8], b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = lhs(i, k);
#pragma unroll
    for (int j = 0; j < 8; ++j) b[j] = rhs(k, j);
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
  }
}

// Forward. A [N,T,D,D], B [N,T,R,D], prev [N,R,D] or NULL, out [N,T+off,R,D]
// (prev first when off = 1). Grid (N), kAffThreads threads; smem: A (D x D+4), H (R x D+4).
__global__ void __launch_bounds__(kAffThreads) k_affine_scan_fwd(const float* A, const float* B, const float* prev,
                                                                 float* out, int T, int R, int D, int off) {
  extern __shared__ float sm_aff[];
  const int ld = D + 4, n = blockIdx.x, tid = threadIdx.x;
  float* As = sm_aff;
  float* Hs = sm_aff + D * ld;
  const int rb = R / 8, cbk = D / 8, tiles = rb * cbk;
  const int r0 = (tid / cbk) * 8, c0 = (tid % cbk) * 8;
  const bool act = tid < tiles;
  for (int x = tid; x < R * D; x += kAffThreads) {
    const float v = prev ? prev[(int64_t)n * R * D + x] : 0.f;
    Hs[(x / D) * ld + x % D] = v;
    if (off) out[(int64_t)n * (T + 1) * R * D + x] = v;
  }
  for (int t = 0; t < T; ++t) {
    aff_load(As, ld, A + ((int64_t)n * T + t) * D * D, D, D);
    aff_wait();
    __syncthreads();
    float acc[8][8];
    if (act) aff_tile(acc, D, [&](int i, int k) { return Hs[(r0 + i) * ld + k]; },
                      [&](int k, int j) { return As[k * ld + c0 + j]; });
    __syncthreads();  // everyone has read H_{t-1} and A_t
    if (act) {
      const float* Bt = B + (((int64_t)n * T + t) * R) * D;
      float* Ot = out + (((int64_t)n * (T + off) + t + off) * R) * D;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = r0 + i;
        const float4 b0 = *reinterpret_cast<const float4*>(Bt + r * D + c0);
        const float4 b1 = *reinterpret_cast<const float4*>(Bt + r * D + c0 + 4);
        const float v[8] = {acc[i][0] + b0.x, acc[i][1] + b0.y, acc[i][2] + b0.z, acc[i][3] + b0.w,
                            acc[i][4] + b1.x, acc[i][5] + b1.y, acc[i][6] + b1.z, acc[i][7] + b1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) Hs[r * ld + c0 + j] = v[j];
        *reinterpret_cast<float4*>(Ot + r * D + c0) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(Ot + r * D + c0 + 4) = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
  }
}

// Backward. out: the forward output; dout its gradient (same layout). dA [N,T,D,D],
// dB [N,T,R,D], dprev [N,R,D] or NULL. Grid (N); smem: A (D x D+4), G (R x D+4), H (R x D+4).
__global__ void __launch_bounds__(kAffThreads) k_affine_scan_bwd(const float* A, const float* prev,
                                                                 const float* out, const float* dout, float* dA,
                                                                 float* dB, float* dprev, int T, int R, int D,
                                                                 int off) {
  extern __shared__ float sm_aff[];
  const int ld = D + 4, n = blockIdx.x, tid = threadIdx.x;
  float* As = sm_aff;
  float* Gs = As + D * ld;
  float* Hs = Gs + R * ld;
  const int rb = R / 8, cbk = D / 8;
  const bool actG = tid < rb * cbk, actA = tid < cbk * cbk;
  const int r0 = (tid / cbk) * 8, c0 = (tid % cbk) * 8;    // G tile
  const int k0 = (tid / cbk) * 8, j0 = (tid % cbk) * 8;    // dA tile
  for (int x = tid; x < R * D; x += kAffThreads) Gs[(x / D) * ld + x % D] = 0.f;
  const float* outn = out + (int64_t)n * (T + off) * R * D;
  const float* doutn = dout + (int64_t)n * (T + off) * R * D;
  for (int t = T - 1; t >= -1; --t) {
    // G_t = dH_t + G_{t+1} A_{t+1}^T  (t = -1: the gradient of prev)
    if (t + 1 < T) aff_load(As, ld, A + ((int64_t)n * T + t + 1) * D * D, D, D);
    aff_wait();
    __syncthreads();
    float acc[8][8];
    if (actG) {
      if (t + 1 < T)
        aff_tile(acc, D, [&](int i, int k) { return Gs[(r0 + i) * ld + k]; },
                 [&](int k, int j) { return As[(c0 + j) * ld + k]; });
      else
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    }
    __syncthreads();  // G_{t+1} and A_{t+1} read
    if (t < 0) {
      if (actG && dprev) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int r = r0 + i, c = c0 + j;
            dprev[((int64_t)n * R + r) * D + c] = acc[i][j] + (off ? doutn[r * D + c] : 0.f);
          }
      }
      break;
    }
    if (actG) {
      const float* dHt = doutn + (int64_t)(t + off) * R * D;
      float* dBt = dB + ((int64_t)n * T + t) * R * D;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int r = r0 + i, c = c0 + j;
          const float g = acc[i][j] + dHt[r * D + c];
          Gs[r * ld + c] = g;
          dBt[r * D + c] = g;
        }
    }
    // H_{t-1}: the previous output row block (prev, or zeros without prev)
    if (t > 0 || off) {
      aff_load(Hs, ld, outn + (int64_t)(t - 1 + off) * R * D, R, D);
    } else {
      for (int x = tid; x < R * D; x += kAffThreads)
        Hs[(x / D) * ld + x % D] = prev ? prev[(int64_t)n * R * D + x] : 0.f;
    }
    aff_wait();
    __syncthreads();
    if (actA) {  // dA_t = H_{t-1}^T G_t
      aff_tile(acc, R, [&](int i, int r) { return Hs[r * ld + k0 + i]; },
               [&](int r, int j) { return Gs[r * ld + j0 + j]; });
      float* dAt = dA + ((int64_t)n * T + t) * D * D;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        *reinterpret_cast<float4*>(dAt + (k0 + i) * D + j0) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        *reinterpret_cast<float4*>(dAt + (k0 + i) * D + j0 + 4) =
            make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
      }
    }
    __syncthreads();  // H and G read before the next step overwrites them
  }
}

}  // namespace atlas
