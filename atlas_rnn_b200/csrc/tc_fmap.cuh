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

constexpr int kFmT = 256;  // threads of the forward and backward CTAs (two warpgroups)

// Shapes the tensor-core feature map handles: dk a multiple of 16 up to 64,
// dphi a multiple of 16 up to 256, bf16 io.
__host__ __device__ __forceinline__ bool fmap_tc_ok(int dk, int dphi, int bf) {
  return bf && dk >= 16 && dk <= 64 && dk % 16 == 0 && dphi >= 16 && dphi <= 256 && dphi % 16 == 0;
}
__host__ __device__ __forceinline__ int fm_chunk_bytes(int dk, int dphi) { return dk * dphi * 2; }
__host__ __device__ __forceinline__ int fm_a_bytes(int dk) { return kR * dk * 2; }
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

// Bulk copy of `bytes` (a multiple of 16) from global into shared memory on barrier `bar`
// (issuing thread; the barrier's arrival is the caller's).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  mbar_expect_tx(bar, bytes);
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   umma::smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(umma::smem_u32(bar))
               : "memory");
}

constexpr int kFmRows = 256;  // tokens per forward CTA: two 128-row MMAs share each Proj chunk
__host__ __device__ __forceinline__ int fm_xh_stride(int dk) { return dk + 8; }  // bf16 x rows, padded
__host__ __device__ __forceinline__ size_t fm_fwd_smem(int dk, int dphi) {
  return 3 * (size_t)fm_chunk_bytes(dk, dphi) + 4 * (size_t)fm_a_bytes(dk) + 2 * (size_t)kFmRows * fm_xh_stride(dk);
}
// Backward: G Proj chunks per MMA (N = G dk <= 128), two B stages of G chunks, the d phi tile.
__host__ __device__ __forceinline__ int fm_group(int dk) { return dk >= 48 ? 2 : 128 / dk; }
__host__ __device__ __forceinline__ size_t fm_bwd_smem(int dk, int dphi) {
  return 2 * (size_t)fm_group(dk) * fm_chunk_bytes(dk, dphi) + (size_t)kR * dphi * 2 + (size_t)kR * (dk + 8) * 2;
}

// phi of 256 tokens of one unit for keys (blockIdx.z = 0) or queries (1), out to
// P.phik / P.phiq (fp32, or bf16 with P.fm_bf16). Grid (ceil(T / 256), N, 2), kFmT threads.
// Per feature chunk c: both 128-token halves' operand tiles are generated (stage c & 1),
// then two MMAs (accumulators at TMEM columns 0 and 256) read the same Proj chunk
// (ring stage c % 3), so each Proj byte fetched from L2 serves 256 tokens.
__global__ void __launch_bounds__(kFmT) k_fmap_fwd_tc(Params P) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const int dk = P.dk, dphi = P.dphi, n = blockIdx.y, isq = blockIdx.z, t0 = blockIdx.x * kFmRows;
  const int TT = min(kFmRows, P.T - t0), tid = threadIdx.x, nch = dk + 1, xl = fm_xh_stride(dk);
  const int cb_bytes = fm_chunk_bytes(dk, dphi), a_bytes = fm_a_bytes(dk);
  unsigned char* Bs = sm;                                     // 3 stages of Proj chunks
  unsigned char* As = sm + 3 * cb_bytes;                      // 2 stages x 2 halves of feature chunks
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(As + 4 * a_bytes);  // [256][dk + 8] raw x
  __shared__ uint64_t bb[3], mb[2];
  __shared__ uint32_t tbase;
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) umma::mbar_init(&bb[i], 1);
    for (int i = 0; i < 2; ++i) umma::mbar_init(&mb[i], 1);
    for (int c = 0; c < 3 && c < nch; ++c) {  // Proj chunks 0..2 in flight
      bulk_g2s(Bs + c * cb_bytes, P.projb + (size_t)c * cb_bytes, cb_bytes, &bb[c]);
      mbar_arrive(&bb[c]);
    }
  }
  if (tid < 32) {
    umma::tmem_alloc(&tbase, 512);
    umma::tmem_relinquish();
  }
  {  // raw x rows (bf16; rows past the unit's end are zero)
    const int cpr = dk / 8;
    for (int u = tid; u < kFmRows * cpr; u += kFmT) {
      const int r = u / cpr, cb = u % cpr;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < TT) {
        if (P.bf) {
          v = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(isq ? P.q : P.k) +
                                              ((int64_t)n * P.T + t0 + r) * dk + cb * 8);
        } else {
          float f[8];
          ld8f(reinterpret_cast<const float*>(isq ? P.q : P.k) + ((int64_t)n * P.T + t0 + r) * dk + cb * 8, f);
          v = pack_unit(f);
        }
      }
      *reinterpret_cast<uint4*>(xs + r * xl + cb * 8) = v;
    }
  }
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  const uint32_t tm = tbase;
  const uint32_t idesc = umma::make_idesc(128, dphi, 0, 1);
  const int cpr = dk / 8, units = kR * cpr;
  // This thread's units of every feature chunk (the same for all chunks: 2 x 128 x cpr units over
  // kFmT threads = cpr <= 8 each): its raw x values stay in registers, the tile offset and the row
  // of the chunk's scalar x_{c-1} are fixed, so a chunk costs one shared load, a scale and a store per unit.
  uint4 xv[8];
  uint32_t aoff[8];
  int xrow[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    xv[k] = make_uint4(0u, 0u, 0u, 0u);
    aoff[k] = 0;
    xrow[k] = 0;
    if (k < cpr) {
      const int u = tid + k * kFmT, h = u >= units, uu = u - h * units;
      int r, cb;
      unit_rc(uu, cpr, r, cb);
      xrow[k] = (h * kR + r) * xl;
      xv[k] = *reinterpret_cast<const uint4*>(xs + xrow[k] + cb * 8);
      aoff[k] = (uint32_t)(h * a_bytes + 16 * uu);
    }
  }
  bool ok = true;
  for (int c = 0; c < nch; ++c) {
    const int sa = c & 1, sb = c % 3;
    if (c >= 2) {  // MMAs of chunk c - 2 done: A stage sa and B stage (c + 1) % 3 are free
      ok = umma::mbar_wait(&mb[sa], ((c >> 1) + 1) & 1) && ok;
      umma::fence_after();
      if (tid == 0 && c + 1 < nch) {
        const int s1 = (c + 1) % 3;
        bulk_g2s(Bs + s1 * cb_bytes, P.projb + (size_t)(c + 1) * cb_bytes, cb_bytes, &bb[s1]);
        mbar_arrive(&bb[s1]);
      }
    }
    // feature chunk c of both halves: x itself (c = 0) or x_{c-1} * x
    unsigned char* A = As + sa * 2 * a_bytes;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k >= cpr) break;
      if (c == 0) {
        *reinterpret_cast<uint4*>(A + aoff[k]) = xv[k];
      } else {
        const float s = __bfloat162float(xs[xrow[k] + c - 1]);
        const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xv[k]);
        __align__(16) __nv_bfloat162 o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 a = __bfloat1622float2(xh[i]);
          o[i] = __floats2bfloat162_rn(a.x * s, a.y * s);
        }
        *reinterpret_cast<uint4*>(A + aoff[k]) = *reinterpret_cast<uint4*>(o);
      }
    }
    umma::fence_async_smem();
    umma::fence_before();
    __syncthreads();
    if (tid == 0) {
      ok = umma::mbar_wait(&bb[sb], (c / 3) & 1) && ok;
      umma::fence_after();
      const uint32_t b0 = umma::smem_u32(Bs + sb * cb_bytes);
      for (int h = 0; h < 2; ++h) {
        const uint32_t a0 = umma::smem_u32(A + h * a_bytes);
        for (int s = 0; s < dk / 16; ++s)
          umma::mma(tm + h * 256, umma::desc_kmajor(a0, dk, s), umma::desc_mnmajor(b0, dphi, s), idesc,
                    (c > 0 || s > 0) ? 1 : 0);
      }
      umma::commit(&mb[sa]);
    }
  }
  ok = umma::mbar_wait(&mb[(nch - 1) & 1], ((nch - 1) >> 1) & 1) && ok;
  umma::fence_after();
  if (__syncthreads_or(!ok)) {
    if (tid == 0 && P.status) atomicExch(P.status, kDevStatMmaTimeout);
  } else {
    // warpgroup h stores the rows of half h (its warps read TMEM lanes 32 (w % 4)..)
    const int h = tid >> 7, row = h * kR + (tid & 127);
    const int64_t off = ((int64_t)n * P.T + t0 + row) * dphi;
    float* dst = (isq ? P.phiq : P.phik) + off;
    __nv_bfloat16* dsth = reinterpret_cast<__nv_bfloat16*>(isq ? P.phiq : P.phik) + off;
    const uint32_t lane = (uint32_t)((tid >> 5) & 3) * 32 << 16;
    for (int c16 = 0; c16 < dphi; c16 += 16) {
      float a[16];
      umma::tmem_ld16(tm + lane + h * 256 + c16, a);
      umma::tmem_ld_wait();
      if (row < TT) {
        if (P.fm_bf16) st16bf(dsth + c16, a);
        else st16f(dst + c16, a);
      }
    }
  }
  umma::fence_before();
  __syncthreads();
  if (tid < 32) umma::tmem_dealloc(tm, 512);
}

// dx of 128 tokens of one unit for keys (blockIdx.z = 0: d phi in P.dphiR, dk out) or
// queries (1: d psi in P.dpsi, dq out); d phi fp32, or bf16 with P.fm_bf16.
// Grid (ceil(T / 128), N, 2), kFmT threads. The feature chunks go G at a time
// (N = G dk columns per MMA, two alternating accumulators, B ring of two stages);
// warpgroup w folds chunks [w G/2, (w+1) G/2) of each group into its own copy of
// dx, and the two copies are summed at the end.
__global__ void __launch_bounds__(kFmT) k_fmap_bwd_tc(Params P) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const int dk = P.dk, dphi = P.dphi, n = blockIdx.y, isq = blockIdx.z, t0 = blockIdx.x * kR;
  const int TT = min(kR, P.T - t0), tid = threadIdx.x, nch = dk + 1;
  void* out = isq ? P.dq_ : P.dk_;
  if (!out) return;
  const int G = fm_group(dk), NG = G * dk, ngr = (nch + G - 1) / G;
  const int cb_bytes = fm_chunk_bytes(dk, dphi), gb_bytes = G * cb_bytes;
  unsigned char* Bs = sm;                  // 2 stages of G Proj chunks (K-major: rows = G dk, K = dphi)
  unsigned char* Ag = sm + 2 * gb_bytes;   // d phi tile [128 x dphi] bf16
  const int xl = fm_xh_stride(dk);
  __nv_bfloat16* xsh = reinterpret_cast<__nv_bfloat16*>(Ag + (size_t)kR * dphi * 2);  // [128][dk + 8] raw x
  constexpr uint32_t kDotCol = 256;       // TMEM columns 256 .. 256 + dk: the per-token dots
  __shared__ uint64_t bb[2], mb[2];
  __shared__ uint32_t tbase;
  // bytes of group g present in projb (the last group may hold fewer than G chunks)
  auto group_bytes = [&](int g) { return (uint32_t)(min(G, nch - g * G) * cb_bytes); };
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) { umma::mbar_init(&bb[i], 1); umma::mbar_init(&mb[i], 1); }
    for (int g = 0; g < 2 && g < ngr; ++g) {
      bulk_g2s(Bs + g * gb_bytes, P.projb + (size_t)g * gb_bytes, group_bytes(g), &bb[g]);
      mbar_arrive(&bb[g]);
    }
  }
  if (tid < 32) {
    umma::tmem_alloc(&tbase, 512);
    umma::tmem_relinquish();
  }
  {  // d phi rows -> bf16 operand tile (rows past the unit's end are zero)
    const int64_t g0 = ((int64_t)n * P.T + t0) * dphi;
    const void* gsrc = isq ? (const void*)P.dpsi : (const void*)P.dphiR;
    const int cpr = dphi / 8;
    for (int u = tid; u < kR * cpr; u += kFmT) {
      int r, cb;
      unit_rc(u, cpr, r, cb);
      float v[8];
      if (r >= TT) zero8(v);
      else if (P.fm_bf16) ld8io(gsrc, g0 + (int64_t)r * dphi + cb * 8, 1, v);
      else ld8f(reinterpret_cast<const float*>(gsrc) + g0 + (int64_t)r * dphi + cb * 8, v);
      *reinterpret_cast<uint4*>(Ag + 16 * u) = pack_unit(v);
    }
  }
  // this thread's token (row) and its warpgroup's chunks: x and a dx copy in registers
  const int row = tid & 127, wgp = tid >> 7, half = G / 2;
  float x[64], dx[64];
  {
    const void* src = isq ? P.q : P.k;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      x[i] = (i < dk && row < TT) ? ldio(src, ((int64_t)n * P.T + t0 + row) * dk + i, P.bf) : 0.f;
      dx[i] = 0.f;
      if (wgp == 0 && i < dk) xsh[row * xl + i] = __float2bfloat16_rn(x[i]);
    }
  }
  umma::fence_async_smem();
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  const uint32_t tm = tbase;
  const uint32_t idesc = umma::make_idesc(128, NG, 0, 0);
  const uint32_t a0 = umma::smem_u32(Ag);
  const uint32_t lane = (uint32_t)((tid >> 5) & 3) * 32 << 16;
  bool ok = true;
  auto issue_mma = [&](int g) {  // thread 0: accumulator g & 1 <- d phi [Proj chunks of group g]^T
    const int sb = g & 1;
    const bool w = umma::mbar_wait(&bb[sb], (g >> 1) & 1);
    umma::fence_after();
    const uint32_t b0 = umma::smem_u32(Bs + sb * gb_bytes);
    for (int s = 0; s < dphi / 16; ++s)
      umma::mma(tm + (g & 1) * 128, umma::desc_kmajor(a0, dphi, s), umma::desc_kmajor(b0, dphi, s), idesc,
                s > 0 ? 1 : 0);
    umma::commit(&mb[g & 1]);
    return w;
  };
  if (tid == 0) ok = issue_mma(0) && ok;
  for (int g = 0; g < ngr; ++g) {
    ok = umma::mbar_wait(&mb[g & 1], (g >> 1) & 1) && ok;  // accumulator of group g landed
    umma::fence_after();
    if (tid == 0) {
      // stage g & 1 was read by MMA g (done): group g + 2 goes in; MMA g + 1 reads the other stage
      if (g + 2 < ngr) {
        bulk_g2s(Bs + (g & 1) * gb_bytes, P.projb + (size_t)(g + 2) * gb_bytes, group_bytes(g + 2), &bb[g & 1]);
        mbar_arrive(&bb[g & 1]);
      }
      if (g + 1 < ngr) ok = issue_mma(g + 1) && ok;
    }
    for (int i = 0; i < half; ++i) {
      const int j = wgp * half + i, c = g * G + j;  // chunk of this warpgroup
      if (c >= nch) break;
      const float xa = c == 0 ? 0.f : __bfloat162float(xsh[row * xl + c - 1]);
      float dot = 0.f;
#pragma unroll
      for (int q16 = 0; q16 < 4; ++q16) {
        if (q16 * 16 >= dk) break;
        float a[16];
        umma::tmem_ld16(tm + lane + (g & 1) * 128 + j * dk + q16 * 16, a);
        umma::tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          if (c == 0) {
            dx[q16 * 16 + q] += a[q];
          } else {
            dot += a[q] * x[q16 * 16 + q];
            dx[q16 * 16 + q] += xa * a[q];
          }
        }
      }
      if (c > 0) umma::tmem_st1(tm + lane + kDotCol + c - 1, dot);  // dx_{c-1} += dot, folded in at the end
    }
    umma::fence_before();
    __syncthreads();  // accumulator g & 1 is read: MMA g + 2 may overwrite it
  }
  umma::tmem_st_wait();
  umma::fence_before();
  if (__syncthreads_or(!ok)) {
    if (tid == 0 && P.status) atomicExch(P.status, kDevStatMmaTimeout);
  } else {
    umma::fence_after();
    if (wgp == 0) {  // the dx_a += <D_a, x> terms of both warpgroups, kept in TMEM columns kDotCol + a
#pragma unroll
      for (int q16 = 0; q16 < 4; ++q16) {
        if (q16 * 16 >= dk) break;
        float a[16];
        umma::tmem_ld16(tm + lane + kDotCol + q16 * 16, a);
        umma::tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 16; ++q) dx[q16 * 16 + q] += a[q];
      }
    }
    // sum the two warpgroups' dx copies through shared memory (the B ring is no longer read)
    float* red = reinterpret_cast<float*>(sm);
    if (wgp == 1) {
#pragma unroll
      for (int q = 0; q < 64; ++q) red[q * kR + row] = dx[q];
    }
    __syncthreads();
    if (wgp == 0 && row < TT) {
#pragma unroll
      for (int q = 0; q < 64; ++q)
        if (q < dk) stio(out, ((int64_t)n * P.T + t0 + row) * dk + q, dx[q] + red[q * kR + row], P.bf);
    }
  }
  umma::fence_before();
  __syncthreads();
  if (tid < 32) umma::tmem_dealloc(tm, 512);
}

}  // namespace tc
}  // namespace atlas
