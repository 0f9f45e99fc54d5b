// Tensor feature map on tensor cores (tcgen05), the 'tensor' mode of
// PolynomialFeatureMap (rnn_memory.py:106-111,125-130):
//
//   phi(x) = [x ; vec(x x^T)] Proj,   x in R^dk, Proj in R^{(dk + dk^2) x dphi}
//
// The dk + dk^2 wide feature row is never written to memory. Its columns come
// in dk + 1 chunks of dk: chunk 0 is x itself, chunk a + 1 is x_a * x (the row
// a of the outer product). Each chunk of 128 tokens is generated into shared
// memory as a bf16 operand tile by the CTA's threads while the previous
// chunk's MMA runs; the matching dk rows of Proj (bf16, pre-tiled once per call
// by k_proj_tiles) arrive by bulk copy into a 3-stage ring. fp32 accumulation
// in TMEM over all dk + 1 chunks.
//
// Backward: d feature = d phi Proj^T is again produced chunk by chunk (M = 128
// tokens, N = dk, K = dphi) into two alternating TMEM accumulators; the
// epilogue of chunk a + 1 folds it into dx without storing it:
//   dx += d lin (chunk 0);  dx_a += <D_a, x>,  dx += x_a D_a  (chunk a + 1),
// the chain rule of x -> x_a x_b. Proj is a fixed buffer: no gradient.
#pragma once
#include "tc_common.cuh"

namespace atlas {
namespace tc {

constexpr int kFmT = 256;  // threads of the forward CTA (two warpgroups split the columns)
constexpr int kFbT = 128;  // threads of the backward CTA (one token row each)

// Shapes the tensor-core feature map handles: dk a multiple of 16 up to 64,
// dphi a multiple of 16 up to 256, bf16 io.
__host__ __device__ __forceinline__ bool fmap_tc_ok(int dk, int dphi, int bf) {
  return bf && dk >= 16 && dk <= 64 && dk % 16 == 0 && dphi >= 16 && dphi <= 256 && dphi % 16 == 0;
}
__host__ __device__ __forceinline__ int fm_chunk_bytes(int dk, int dphi) { return dk * dphi * 2; }
__host__ __device__ __forceinline__ int fm_a_bytes(int dk) { return kR * dk * 2; }
__host__ __device__ __forceinline__ int fm_x_stride(int dk) { return dk + 4; }  // padded fp32 rows: no bank conflicts
__host__ __device__ __forceinline__ size_t fm_fwd_smem(int dk, int dphi) {
  return 3 * (size_t)fm_chunk_bytes(dk, dphi) + 2 * (size_t)fm_a_bytes(dk) + 4 * (size_t)kR * fm_x_stride(dk);
}
__host__ __device__ __forceinline__ size_t fm_bwd_smem(int dk, int dphi) {
  return 3 * (size_t)fm_chunk_bytes(dk, dphi) + (size_t)kR * dphi * 2;
}
__host__ __device__ __forceinline__ uint32_t tmem_cols_for(int n) {
  uint32_t c = 32;
  while ((int)c < n) c <<= 1;
  return c;
}

// Proj [dk + dk^2, dphi] fp32 -> dk + 1 bf16 tiles of dk rows x dphi columns
// (core-matrix layout), chunk c holding rows [c dk, (c + 1) dk). Grid (dk + 1).
__global__ void __launch_bounds__(256) k_proj_tiles(Params P) {
  const int dk = P.dk, dphi = P.dphi, c = blockIdx.x, cpr = dphi / 8;
  unsigned char* dst = P.projb + (size_t)c * fm_chunk_bytes(dk, dphi);
  for (int u = threadIdx.x; u < dk * cpr; u += blockDim.x) {
    const int r = u / cpr, cb = u % cpr;
    float v[8];
    ld8f(P.proj + ((int64_t)c * dk + r) * dphi + cb * 8, v);
    *reinterpret_cast<uint4*>(dst + umma::unit_off(r, cb, dphi)) = pack_unit(v);
  }
}

// phi of 128 tokens of one unit for keys (blockIdx.z = 0) or queries (1), fp32
// out to P.phik / P.phiq. Grid (ceil(T / 128), N, 2), kFmT threads.
__global__ void __launch_bounds__(kFmT) k_fmap_fwd_tc(Params P) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const int dk = P.dk, dphi = P.dphi, n = blockIdx.y, isq = blockIdx.z, t0 = blockIdx.x * kR;
  const int TT = min(kR, P.T - t0), tid = threadIdx.x, nch = dk + 1, xs_ld = fm_x_stride(dk);
  const int cb_bytes = fm_chunk_bytes(dk, dphi), a_bytes = fm_a_bytes(dk);
  unsigned char* Bs = sm;                          // 3 stages of Proj chunks
  unsigned char* As = sm + 3 * cb_bytes;           // 2 stages of generated feature chunks
  float* xs = reinterpret_cast<float*>(As + 2 * a_bytes);  // [128][dk + 4] raw x
  __shared__ uint64_t bb[3], mb[2];
  __shared__ uint32_t tbase;
  const uint32_t ncols = tmem_cols_for(dphi);
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) umma::mbar_init(&bb[i], 1);
    for (int i = 0; i < 2; ++i) umma::mbar_init(&mb[i], 1);
    for (int c = 0; c < 2 && c < nch; ++c) {  // Proj chunks 0, 1 in flight
      mbar_expect_tx(&bb[c], cb_bytes);
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                       umma::smem_u32(Bs + c * cb_bytes)),
                   "l"(P.projb + (size_t)c * cb_bytes), "r"(cb_bytes), "r"(umma::smem_u32(&bb[c]))
                   : "memory");
      mbar_arrive(&bb[c]);
    }
  }
  if (tid < 32) {
    umma::tmem_alloc(&tbase, ncols);
    umma::tmem_relinquish();
  }
  const void* src = isq ? P.q : P.k;
  for (int x = tid; x < kR * dk; x += kFmT) {
    const int r = x / dk, c = x % dk;
    xs[r * xs_ld + c] = r < TT ? ldio(src, ((int64_t)n * P.T + t0 + r) * dk + c, P.bf) : 0.f;
  }
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  const uint32_t tm = tbase;
  const uint32_t idesc = umma::make_idesc(128, dphi, 0, 1);
  const int cpr = dk / 8, units = kR * cpr;
  bool ok = true;
  for (int c = 0; c < nch; ++c) {
    const int sa = c & 1, sb = c % 3;
    if (c >= 2) {  // MMA c - 2 done: A stage sa and B stage (c + 1) % 3 are free
      ok = umma::mbar_wait(&mb[sa], ((c >> 1) + 1) & 1) && ok;
      umma::fence_after();
      if (tid == 0 && c + 1 < nch) {
        const int s1 = (c + 1) % 3;
        mbar_expect_tx(&bb[s1], cb_bytes);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                umma::smem_u32(Bs + s1 * cb_bytes)),
            "l"(P.projb + (size_t)(c + 1) * cb_bytes), "r"(cb_bytes), "r"(umma::smem_u32(&bb[s1]))
            : "memory");
        mbar_arrive(&bb[s1]);
      }
    } else if (c == 1 && tid == 0 && nch > 2) {
      // stage 2 is untouched so far: chunk 2 can go in at once
      mbar_expect_tx(&bb[2], cb_bytes);
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                       umma::smem_u32(Bs + 2 * cb_bytes)),
                   "l"(P.projb + (size_t)2 * cb_bytes), "r"(cb_bytes), "r"(umma::smem_u32(&bb[2]))
                   : "memory");
      mbar_arrive(&bb[2]);
    }
    // feature chunk c: x itself (c = 0) or x_{c-1} * x
    unsigned char* A = As + sa * a_bytes;
    for (int u = tid; u < units; u += kFmT) {
      int r, cb;
      unit_rc(u, cpr, r, cb);
      const float* xr = xs + r * xs_ld;
      const float4 lo = *reinterpret_cast<const float4*>(xr + cb * 8);
      const float4 hi = *reinterpret_cast<const float4*>(xr + cb * 8 + 4);
      const float s = c == 0 ? 1.f : xr[c - 1];
      const float v[8] = {s * lo.x, s * lo.y, s * lo.z, s * lo.w, s * hi.x, s * hi.y, s * hi.z, s * hi.w};
      *reinterpret_cast<uint4*>(A + 16 * u) = pack_unit(v);
    }
    umma::fence_async_smem();
    umma::fence_before();
    __syncthreads();
    if (tid == 0) {
      // chunks 0, 1 and 2 were issued before their stage was waited on; later ones in the loop above
      ok = umma::mbar_wait(&bb[sb], (c / 3) & 1) && ok;
      umma::fence_after();
      const uint32_t a0 = umma::smem_u32(A), b0 = umma::smem_u32(Bs + sb * cb_bytes);
      for (int s = 0; s < dk / 16; ++s)
        umma::mma(tm, umma::desc_kmajor(a0, dk, s), umma::desc_mnmajor(b0, dphi, s), idesc, (c > 0 || s > 0) ? 1 : 0);
      umma::commit(&mb[sa]);
    }
  }
  // the last MMA (chunk nch - 1, stage (nch - 1) & 1)
  ok = umma::mbar_wait(&mb[(nch - 1) & 1], ((nch - 1) >> 1) & 1) && ok;
  umma::fence_after();
  if (__syncthreads_or(!ok)) {
    if (tid == 0 && P.status) atomicExch(P.status, kDevStatMmaTimeout);
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4).., warpgroup g columns [g dphi/2, (g+1) dphi/2)
    const int row = tid & 127, g = tid >> 7, half = dphi / 2;
    const int64_t off = ((int64_t)n * P.T + t0 + row) * dphi;
    float* dst = (isq ? P.phiq : P.phik) + off;
    __nv_bfloat16* dsth = reinterpret_cast<__nv_bfloat16*>(isq ? P.phiq : P.phik) + off;
    for (int c16 = g * half; c16 < (g + 1) * half; c16 += 16) {
      float a[16];
      umma::tmem_ld16(tm + ((uint32_t)((tid >> 5) & 3) * 32 << 16) + c16, a);
      umma::tmem_ld_wait();
      if (row < TT) {
        if (P.fm_bf16) st16bf(dsth + c16, a);
        else st16f(dst + c16, a);
      }
    }
  }
  umma::fence_before();
  __syncthreads();
  if (tid < 32) umma::tmem_dealloc(tm, ncols);
}

// dx of 128 tokens of one unit for keys (blockIdx.z = 0: d phi in P.dphiR, dk
// out) or queries (1: d psi in P.dpsi, dq out). Grid (ceil(T / 128), N, 2), kFbT threads.
__global__ void __launch_bounds__(kFbT) k_fmap_bwd_tc(Params P) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const int dk = P.dk, dphi = P.dphi, n = blockIdx.y, isq = blockIdx.z, t0 = blockIdx.x * kR;
  const int TT = min(kR, P.T - t0), tid = threadIdx.x, nch = dk + 1;
  void* out = isq ? P.dq_ : P.dk_;
  if (!out) return;
  const int cb_bytes = fm_chunk_bytes(dk, dphi);
  unsigned char* Bs = sm;                  // 3 stages of Proj chunks (used K-major: rows = dk, K = dphi)
  unsigned char* Ag = sm + 3 * cb_bytes;   // d phi tile [128 x dphi] bf16
  __shared__ uint64_t bb[3], mb[2];
  __shared__ uint32_t tbase;
  const uint32_t ncols = tmem_cols_for(2 * dk);
  auto issue_b = [&](int c) {
    const int s = c % 3;
    mbar_expect_tx(&bb[s], cb_bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                     umma::smem_u32(Bs + s * cb_bytes)),
                 "l"(P.projb + (size_t)c * cb_bytes), "r"(cb_bytes), "r"(umma::smem_u32(&bb[s]))
                 : "memory");
    mbar_arrive(&bb[s]);
  };
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) umma::mbar_init(&bb[i], 1);
    for (int i = 0; i < 2; ++i) umma::mbar_init(&mb[i], 1);
    for (int c = 0; c < 3 && c < nch; ++c) issue_b(c);
  }
  if (tid < 32) {
    umma::tmem_alloc(&tbase, ncols);
    umma::tmem_relinquish();
  }
  {  // d phi rows -> bf16 operand tile (rows past the unit's end are zero)
    const int64_t g0 = ((int64_t)n * P.T + t0) * dphi;
    const float* g = (isq ? P.dpsi : P.dphiR) + g0;
    const int cpr = dphi / 8;
    for (int u = tid; u < kR * cpr; u += kFbT) {
      int r, cb;
      unit_rc(u, cpr, r, cb);
      float v[8];
      if (r >= TT) zero8(v);
      else if (P.fm_bf16) ld8io(isq ? P.dpsi : P.dphiR, g0 + (int64_t)r * dphi + cb * 8, 1, v);
      else ld8f(g + (int64_t)r * dphi + cb * 8, v);
      *reinterpret_cast<uint4*>(Ag + 16 * u) = pack_unit(v);
    }
  }
  // this thread's token: x and dx in registers
  const int row = tid;
  float x[64], dx[64];
  const void* src = isq ? P.q : P.k;
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    x[i] = (i < dk && row < TT) ? ldio(src, ((int64_t)n * P.T + t0 + row) * dk + i, P.bf) : 0.f;
    dx[i] = 0.f;
  }
  umma::fence_async_smem();
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  const uint32_t tm = tbase;
  const uint32_t idesc = umma::make_idesc(128, dk, 0, 0);
  const uint32_t a0 = umma::smem_u32(Ag);
  const uint32_t lane = (uint32_t)((tid >> 5) & 3) * 32 << 16;
  auto issue_mma = [&](int c) {  // thread 0: accumulator c & 1 <- d phi Proj_c^T
    const int sb = c % 3;
    bool w = umma::mbar_wait(&bb[sb], (c / 3) & 1);
    umma::fence_after();
    const uint32_t b0 = umma::smem_u32(Bs + sb * cb_bytes);
    for (int s = 0; s < dphi / 16; ++s)
      umma::mma(tm + (c & 1) * dk, umma::desc_kmajor(a0, dphi, s), umma::desc_kmajor(b0, dphi, s), idesc,
                s > 0 ? 1 : 0);
    umma::commit(&mb[c & 1]);
    return w;
  };
  bool ok = true;
  if (tid == 0) ok = issue_mma(0) && ok;
  for (int c = 0; c < nch; ++c) {
    // accumulator c landed; the next chunk's MMA goes into the other accumulator meanwhile
    ok = umma::mbar_wait(&mb[c & 1], (c >> 1) & 1) && ok;
    umma::fence_after();
    if (tid == 0) {
      if (c + 1 < nch) ok = issue_mma(c + 1) && ok;  // its B stage was loaded two chunks ago
    }
    // fold chunk c into dx (columns in groups of 16)
    float xa = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) xa = (i == c - 1) ? x[i] : xa;
    float dot = 0.f;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      if (g * 16 >= dk) break;
      float a[16];
      umma::tmem_ld16(tm + lane + (c & 1) * dk + g * 16, a);
      umma::tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (c == 0) {
          dx[g * 16 + i] += a[i];
        } else {
          dot += a[i] * x[g * 16 + i];
          dx[g * 16 + i] += xa * a[i];
        }
      }
    }
    if (c > 0) {
#pragma unroll
      for (int i = 0; i < 64; ++i) if (i == c - 1) dx[i] += dot;
    }
    umma::fence_before();
    __syncthreads();  // accumulator c & 1 is read: MMA c + 2 may overwrite it; B stage c % 3 is free
    if (tid == 0 && c + 3 < nch) {
      // MMA c + 1 was issued above and reads stage (c + 1) % 3; stage c % 3 was read by MMA c (done)
      issue_b(c + 3);
    }
  }
  if (__syncthreads_or(!ok)) {
    if (tid == 0 && P.status) atomicExch(P.status, kDevStatMmaTimeout);
  } else if (row < TT) {
#pragma unroll
    for (int i = 0; i < 64; ++i)
      if (i < dk) stio(out, ((int64_t)n * P.T + t0 + row) * dk + i, dx[i], P.bf);
  }
  umma::fence_before();
  __syncthreads();
  if (tid < 32) umma::tmem_dealloc(tm, ncols);
}

}  // namespace tc
}  // namespace atlas
