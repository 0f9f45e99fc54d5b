// Device self-check of the tensor-core building blocks: one 128 x N x K bf16
// GEMM through tcgen05 with operands in either major-ness, D = A * B^T
// (K-major B given as [N][K]) or A * B (MN-major B given as [K][N]).
#pragma once
#include <cuda_bf16.h>

#include "umma.cuh"

namespace atlas {

__global__ void __launch_bounds__(128) k_umma_selftest(const __nv_bfloat16* A, const __nv_bfloat16* B, float* D,
                                                       int N, int K, int a_mn, int b_mn, int* status) {
  constexpr int M = 128;
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* As = sm;                       // M*K bf16
  unsigned char* Bs = sm + M * K * 2;           // N*K bf16
  __shared__ uint64_t mbar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // operands -> core-matrix tiled layout
  for (int i = tid; i < M * K; i += 128) {
    int r, c, C;
    if (!a_mn) { r = i / K; c = i % K; C = K; }      // A[m][k]
    else { r = i / M; c = i % M; C = M; }            // A^T stored [k][m]
    *reinterpret_cast<__nv_bfloat16*>(As + umma::elem_off(r, c, C)) = A[i];
  }
  for (int i = tid; i < N * K; i += 128) {
    int r, c, C;
    if (!b_mn) { r = i / K; c = i % K; C = K; }      // B[n][k]
    else { r = i / N; c = i % N; C = N; }            // B stored [k][n]
    *reinterpret_cast<__nv_bfloat16*>(Bs + umma::elem_off(r, c, C)) = B[i];
  }
  umma::fence_async_smem();
  uint32_t ncols = 32;
  while ((int)ncols < N) ncols <<= 1;
  if (warp == 0) {
    umma::tmem_alloc(&tbase, ncols);
    umma::tmem_relinquish();
  }
  if (tid == 0) umma::mbar_init(&mbar, 1);
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  const uint32_t tm = tbase;
  if (tid == 0) {
    const uint32_t idesc = umma::make_idesc(M, N, a_mn, b_mn);
    const uint32_t a0 = umma::smem_u32(As), b0 = umma::smem_u32(Bs);
    for (int s = 0; s < K / 16; ++s) {
      const uint64_t ad = a_mn ? umma::desc_mnmajor(a0, M, s) : umma::desc_kmajor(a0, K, s);
      const uint64_t bd = b_mn ? umma::desc_mnmajor(b0, N, s) : umma::desc_kmajor(b0, K, s);
      umma::mma(tm, ad, bd, idesc, s > 0);
    }
    umma::commit(&mbar);
  }
  bool ok = umma::mbar_wait(&mbar, 0);
  if (!ok) {
    if (lane == 0) atomicExch(status, 1);
    umma::mbar_wait(&mbar, 0);  // bounded second wait for the MMAs in flight
  }
  umma::fence_after();
  if (ok) {
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      umma::tmem_ld16(tm + ((uint32_t)(warp * 32) << 16) + c0, v);
      umma::tmem_ld_wait();
      const int row = warp * 32 + lane;
#pragma unroll
      for (int j = 0; j < 16; ++j) D[row * N + c0 + j] = v[j];
    }
  }
  umma::fence_before();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tm, ncols);
}

}  // namespace atlas
