// Tensor-core (tcgen05) versions of the forward chunk kernels, bf16 operands
// with fp32 accumulation in TMEM. Same inputs, outputs and workspace layout
// as k_fwd_chunk / k_fwd_out (chunk_kernels.cuh).
#pragma once
#include "tc_common.cuh"

namespace atlas {
namespace tc {

// Floats of per-chunk context (gates) for a chunk length C and window e.
__host__ __device__ __forceinline__ int ctx_floats(int C, int e) {
  auto r4 = [](int n) { return (n + 3) & ~3; };
  return 3 * r4(C) + r4(C + e) + r4(C * e);
}

__device__ __forceinline__ void zero_tile(unsigned char* tile) {
  for (int u = threadIdx.x; u < kTileBytes / 16; u += blockDim.x)
    reinterpret_cast<uint4*>(tile)[u] = make_uint4(0u, 0u, 0u, 0u);
}
// Forward coefficients of key j token by token (the recurrence of fwd_coefs,
// chunk_kernels.cuh): emit(i, cS before token i, cZ before token i, cZ after
// token i). Key j has no coefficient before its first window token j - e + 1,
// receives window weights up to token j and then evolves homogeneously, so only
// tokens [max(0, j - e + 1), L) are emitted (the caller zero-fills the tile rows
// beforehand) and the weight lookup runs for at most e of them.
template <class F>
__device__ __forceinline__ void fwd_column_z(const Params& P, const Ctx& cx, int j, F emit) {
  const int L = cx.L;
  int i = max(0, j - (P.e - 1));
  const int wend = min(L, j + 1);
  float cs = 0.f, cz = 0.f;
  for (; i < wend; ++i) {
    const float czn = cx.be[i] * cz + wgt(P, cx, i, j);
    emit(i, cs, cz, czn);
    cz = czn;
    cs = cx.al[i] * cs - cx.et[i] * cz;
  }
  for (; i + 4 <= L; i += 4) {
    float al[4], et[4], be[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) { al[k] = cx.al[i + k]; et[k] = cx.et[i + k]; be[k] = cx.be[i + k]; }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float czn = be[k] * cz;
      emit(i + k, cs, cz, czn);
      cz = czn;
      cs = al[k] * cs - et[k] * cz;
    }
  }
  for (; i < L; ++i) {
    const float czn = cx.be[i] * cz;
    emit(i, cs, cz, czn);
    cz = czn;
    cs = cx.al[i] * cs - cx.et[i] * cz;
  }
}
// Adjoint coefficients of token q (the recurrence of adj_coefs, chunk_kernels.cuh):
// emit(i, eS_{i+1}[q], eZ_{i+1}[q]) for i descending. They vanish for rows
// i >= q, so only rows [0, q) are emitted (the caller zero-fills the tile).
// With es_end / ez_end given, the values after token 0 (eS_0[q], eZ_0[q]) are returned there.
template <class F>
__device__ __forceinline__ void adj_column_z(const Ctx& cx, int q, F emit, float* es_end = nullptr,
                                             float* ez_end = nullptr) {
  if (q >= cx.L) {
    if (es_end) *es_end = 0.f;
    if (ez_end) *ez_end = 0.f;
    return;
  }
  float es = 1.f, ez = -(q >= 1 ? cx.et[q - 1] : 0.f);  // after token q
  int i = q - 1;
  for (; i - 3 >= 0; i -= 4) {
    float al[4], be[4], etm[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      al[k] = cx.al[i - k];
      be[k] = cx.be[i - k];
      etm[k] = i - k >= 1 ? cx.et[i - k - 1] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      emit(i - k, es, ez);
      es = al[k] * es;
      ez = be[k] * ez - etm[k] * es;
    }
  }
  for (; i >= 0; --i) {
    emit(i, es, ez);
    const float etm = i >= 1 ? cx.et[i - 1] : 0.f;
    es = cx.al[i] * es;
    ez = cx.be[i] * ez - etm * es;
  }
  if (es_end) *es_end = es;
  if (ez_end) *ez_end = ez;
}

__device__ __forceinline__ void st_bf(unsigned char* tile, int r, int c, float v) {
  *reinterpret_cast<__nv_bfloat16*>(tile + umma::elem_off(r, c, kR)) = __float2bfloat16_rn(v);
}

// Key rows of phi into a tile (zero for p < 0 and rows >= K).
__device__ __forceinline__ void fill_keys_phi(const Params& P, const Ctx& cx, unsigned char* tile, int first = 0,
                                              int count = kT) {
  fill_tile(tile, kD, [&](int r, int c0, float(&v)[8]) {
    const int p = cx.kp0 + r;
    if (r < cx.K && p >= 0) phi8(P, cx.n, p, c0, false, v);
    else zero8(v);
  }, first, count);
}
// Token rows of psi (zero for rows >= L).
__device__ __forceinline__ void fill_rows_psi(const Params& P, const Ctx& cx, unsigned char* tile, int first = 0,
                                              int count = kT) {
  fill_tile(tile, kD, [&](int r, int c0, float(&v)[8]) {
    if (r < cx.L) phi8(P, cx.n, cx.t0 + r, c0, true, v);
    else zero8(v);
  }, first, count);
}
// Asynchronous forms: raw bf16 k / q rows (cp.async), then phi_xform() applies
// the elementwise feature map in place after async_wait() and a barrier. With
// the tensor feature map (fp32 phi buffers) the rows are converted synchronously.
__device__ __forceinline__ void async_keys_phi(const Params& P, const Ctx& cx, unsigned char* tile, int first = 0,
                                               int count = kT) {
  if (P.fmode == ATLAS_FMAP_TENSOR) { fill_keys_phi(P, cx, tile, first, count); return; }
  const __nv_bfloat16* k = reinterpret_cast<const __nv_bfloat16*>(P.k);
  async_rows(tile, [&](int r) -> const __nv_bfloat16* {
    const int p = cx.kp0 + r;
    return (r < cx.K && p >= 0) ? k + ((int64_t)cx.n * P.T + p) * P.dk : nullptr;
  }, P.k, first, count);
}
__device__ __forceinline__ void async_rows_psi(const Params& P, const Ctx& cx, unsigned char* tile, int first = 0,
                                               int count = kT) {
  if (P.fmode == ATLAS_FMAP_TENSOR) { fill_rows_psi(P, cx, tile, first, count); return; }
  const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(P.q);
  async_rows(tile, [&](int r) -> const __nv_bfloat16* {
    return r < cx.L ? q + ((int64_t)cx.n * P.T + cx.t0 + r) * P.dk : nullptr;
  }, P.q, first, count);
}
__device__ __forceinline__ void phi_xform(const Params& P, unsigned char* tile, int first = 0, int count = kT) {
  if (P.fmode != ATLAS_FMAP_ELEMENTWISE || P.fdeg <= 1) return;
  xform_rows(tile, kR, [&](int, float(&v)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = fmap_elem(v[i], P.fmode, P.fdeg);
  }, first, count);
}
// Rows of the bf16 delta buffer for the chunk's keys (zero for p < 0, rows >= K).
__device__ __forceinline__ void async_keys_delta(const Params& P, const Ctx& cx, unsigned char* tile, int first = 0,
                                                 int count = kT) {
  async_rows(tile, [&](int r) -> const __nv_bfloat16* {
    const int p = cx.kp0 + r;
    return (r < cx.K && p >= 0) ? P.dlb + ((int64_t)cx.n * P.T + p) * P.dv : nullptr;
  }, P.dlb, first, count);
}
// Token rows of dy (bf16; zero for rows >= L).
__device__ __forceinline__ void async_rows_dy(const Params& P, const Ctx& cx, unsigned char* tile, int first = 0,
                                              int count = kT) {
  const __nv_bfloat16* dy = reinterpret_cast<const __nv_bfloat16*>(P.dy);
  async_rows(tile, [&](int r) -> const __nv_bfloat16* {
    return r < cx.L ? dy + ((int64_t)cx.n * P.T + cx.t0 + r) * P.dv : nullptr;
  }, P.dy, first, count);
}
// TMA forms (call from every thread; thread 0 issues, the batch's barrier
// signals arrival). With the tensor feature map the fp32 phi rows are
// converted synchronously by all threads instead.
__device__ __forceinline__ void load_keys_phi(const Params& P, const Ctx& cx, unsigned char* tile, TmaBatch& b) {
  if (P.fmode == ATLAS_FMAP_TENSOR) { fill_keys_phi(P, cx, tile); return; }
  if (threadIdx.x == 0) tma_rows(&P.tm_k, tile, cx.n, cx.kp0, b.bar);
}
// Token rows of psi; rows >= L hold the next chunk's tokens until zero_rows_from(tile, L).
__device__ __forceinline__ void load_rows_psi(const Params& P, const Ctx& cx, unsigned char* tile, TmaBatch& b) {
  if (P.fmode == ATLAS_FMAP_TENSOR) { fill_rows_psi(P, cx, tile); return; }
  if (threadIdx.x == 0) tma_rows(&P.tm_q, tile, cx.n, cx.t0, b.bar);
}
__device__ __forceinline__ void load_keys_delta(const Params& P, const Ctx& cx, unsigned char* tile, TmaBatch& b) {
  if (threadIdx.x == 0) tma_rows(&P.tm_dl, tile, cx.n, cx.kp0, b.bar);
}
// Token rows of dy; rows >= L as for load_rows_psi.
__device__ __forceinline__ void load_rows_dy(const Params& P, const Ctx& cx, unsigned char* tile, TmaBatch& b) {
  if (threadIdx.x == 0) tma_rows(&P.tm_dy, tile, cx.n, cx.t0, b.bar);
}
__device__ __forceinline__ void load_tile(unsigned char* tile, const unsigned char* src, TmaBatch& b) {
  if (threadIdx.x == 0) tma_tile(tile, src, b.bar);
}

// Named barrier over warpgroups 1..kWG-1 (the loaders while warpgroup 0 is busy).
__device__ __forceinline__ void loaders_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kT - 128) : "memory"); }


// S_ref of every unit as one bf16 operand tile (core-matrix layout), once per
// call: the chunk kernels then copy it raw. Grid (N), 256 threads.
__global__ void __launch_bounds__(256) k_sref_tile(Params P) {
  const float* M = P.Sref + (int64_t)blockIdx.x * kD * kD;
  unsigned char* dst = P.srb + (int64_t)blockIdx.x * kTileBytes;
  for (int u = threadIdx.x; u < kTileBytes / 16; u += blockDim.x) {
    int r, cb;
    unit_rc(u, kD / 8, r, cb);
    float v[8];
    ld8f(M + r * kD + cb * 8, v);
    *reinterpret_cast<uint4*>(dst + 16 * u) = pack_unit(v);
  }
}

// ===========================================================================
// delta and the chunk increments (dS, dZ) on tensor cores.
//   delta[keys x d_v] = Phi[keys x d_phi] S_ref^T - V
//   dS[d_v x d_phi]   = (diag(cS_end) delta)^T Phi,  dZ likewise with cZ_end
// ===========================================================================
__global__ void __launch_bounds__(kT) k_fwd_chunk_tc(const __grid_constant__ Params P) {
  PhaseClock pc;
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* tPhi = sm;
  unsigned char* tSref = sm + kTileBytes;  // S_ref, later diag(cZ_end) delta
  unsigned char* tDS = sm + 2 * kTileBytes;
  unsigned char* tDZ = tSref;
  SmemAlloc sa{reinterpret_cast<float*>(sm + 3 * kTileBytes), 0};
  __shared__ uint64_t mbar, lbar;
  __shared__ uint32_t tbase;
  Ctx cx;
  ctx_geom(P, cx);
  TmaBatch ld{&lbar, 0};
  if (threadIdx.x == 0) tma_init(ld);
  load_keys_phi(P, cx, tPhi, ld);
  load_tile(tSref, P.srb + (int64_t)cx.n * kTileBytes, ld);
  if (threadIdx.x == 0) tma_commit(ld);
  load_ctx(P, sa, cx, kT);
  float* cSe = sa.take(kR);
  float* cZe = sa.take(kR);
  float* Asuf = sa.take(kR);
  float* Bsuf = sa.take(kR);
  float* Hs = sa.take(kR);
  const int n = cx.n, c = cx.c, K = cx.K, L = cx.L, tid = threadIdx.x, row = row_of(), wg = wg_of();
  Sync sy{&mbar, &tbase, 0, P.status};
  const uint32_t tm = tc_setup(sy, 256);  // (its barrier also publishes the gates)
  pc.mark(40);
  // End coefficients of key j from suffix sequences of the chunk (no per-key chain):
  //   cZ_end[j] = sum_m W(m, j) Bsuf[m],   Bsuf[m] = prod_{l > m} beta_l
  //   cS_end[j] = -sum_m W(m, j) H[m],     H[m] = Asuf[m] eta_m + beta_{m+1} H[m+1],
  // Asuf[m] = prod_{l > m} alpha_l, m over the key's window tokens only; the chunk
  // transform is (alpha_0 Asuf[0], -beta_0 H[0], beta_0 Bsuf[0]).
  if (tid < 32) {
    warp_affine_scan<false>(L, 1.f, [&](int m) { return m < L - 1 ? cx.al[m + 1] : 1.f; }, [](int) { return 0.f; },
                            [&](int m, float x) { Asuf[m] = x; });
    __syncwarp();
    warp_affine_scan<false>(L, 0.f, [&](int m) { return m < L - 1 ? cx.be[m + 1] : 0.f; },
                            [&](int m) { return Asuf[m] * cx.et[m]; }, [&](int m, float x) { Hs[m] = x; });
  } else if (tid < 64) {
    warp_affine_scan<false>(L, 1.f, [&](int m) { return m < L - 1 ? cx.be[m + 1] : 1.f; }, [](int) { return 0.f; },
                            [&](int m, float x) { Bsuf[m] = x; });
  }
  __syncthreads();
  if (wg == 0) {
    const int j = row;
    float cs = 0.f, cz = 0.f;
    for (int m = max(0, j - (P.e - 1)); m <= min(L - 1, j); ++m) {
      const float w = wgt(P, cx, m, j);
      cz += w * Bsuf[m];
      cs -= w * Hs[m];
    }
    cSe[j] = cs;
    cZe[j] = cz;
    if (j == 0) {
      float* o = P.cs + ((int64_t)n * P.nch + c) * 4;
      o[0] = cx.al[0] * Asuf[0]; o[1] = -cx.be[0] * Hs[0]; o[2] = cx.be[0] * Bsuf[0]; o[3] = 0.f;
    }
  }
  tma_wait(ld, P.status);
  __syncthreads();
  phi_xform(P, tPhi);
  pc.mark(41);
  smem_to_tc();
  if (tid == 0) mma_chain(tm, op(tPhi, kD, 0), op(tSref, kD, 0), kD / 16, kD, false);
  const int j = row, p = cx.kp0 + j;
  const bool valid = j < K && p >= 0;
  // this thread's half of the key's v row (bf16), fetched while the MMA runs
  uint4 vrow[kD / (8 * kWG)];
  if (valid) {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(P.v) +
                                                      ((int64_t)n * P.T + p) * P.dv + wg * (kD / kWG));
#pragma unroll
    for (int u = 0; u < kD / (8 * kWG); ++u) vrow[u] = src[u];
  }
  ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 256);
  pc.mark(42);
  {
    const float ws = cSe[j], wz = cZe[j];
#pragma unroll
    for (int h = 0; h < kCPW; ++h) {
      const int c16 = wg * kCPW + h;
      float a[16];
      umma::tmem_ld16(lane_addr(tm, c16 * 16), a);
      umma::tmem_ld_wait();
      if (valid) {
        const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&vrow[2 * h]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float2 f = __bfloat1622float2(hv[k]);
          a[2 * k] -= f.x;
          a[2 * k + 1] -= f.y;
        }
        if (p >= cx.t0) st16bf(P.dlb + ((int64_t)n * P.T + p) * P.dv + c16 * 16, a);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) a[i] = 0.f;
      }
      float s0[8], s1[8], z0[8], z1[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        s0[i] = ws * a[i]; s1[i] = ws * a[8 + i];
        z0[i] = wz * a[i]; z1[i] = wz * a[8 + i];
      }
      store_unit(tDS, j, 2 * c16, kD, s0);
      store_unit(tDS, j, 2 * c16 + 1, kD, s1);
      store_unit(tDZ, j, 2 * c16, kD, z0);
      store_unit(tDZ, j, 2 * c16 + 1, kD, z1);
    }
  }
  pc.mark(43);
  smem_to_tc();
  if (tid == 0) {
    mma_chain(tm + 128, op(tDS, kD, 1), op(tPhi, kD, 1), 8, kD, false);
    mma_chain(tm, op(tDZ, kD, 1), op(tPhi, kD, 1), 8, kD, false);  // over delta, already read
  }
  ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 256);
  pc.mark(44);
  {  // increments: row = state row nn
    const int64_t D2 = (int64_t)kD * kD;
    const float* bufn = buf_of(P, n, c);
    const int nb = bufn ? P.e - 1 : 0;
#pragma unroll
    for (int h = 0; h < kCPW; ++h) {
      const int c16 = wg * kCPW + h;
      float a[16], b[16];
      umma::tmem_ld16(lane_addr(tm, 128 + c16 * 16), a);
      umma::tmem_ld16(lane_addr(tm, c16 * 16), b);
      umma::tmem_ld_wait();
      for (int jb = 0; jb < nb; ++jb) {  // carried buffer entries of chunk 0 (dense)
        const float* bj = bufn + (int64_t)jb * D2 + (int64_t)row * kD + c16 * 16;
#pragma unroll
        for (int i = 0; i < 16; ++i) { a[i] += cSe[jb] * bj[i]; b[i] += cZe[jb] * bj[i]; }
      }
      __nv_bfloat16* db = reinterpret_cast<__nv_bfloat16*>(P.st) + ((int64_t)n * P.nch + c) * 2 * D2 + (int64_t)row * kD;
      st16bf(db + c16 * 16, a);
      st16bf(db + D2 + c16 * 16, b);
    }
  }
  tc_teardown(tm, 256);  pc.mark(45);

}

// ===========================================================================
// outputs y on tensor cores:
//   y = (cS o Psi Phi^T) delta + diag(sS) Psi S_in^T + diag(sZ) Psi Z_in^T
// (chunk 0 with a carried buffer adds its dense terms in k_fwd_buf_y).
// ===========================================================================
// Persistent: each CTA walks chunks it = blockIdx.x, + gridDim.x, ... (chunk
// fastest, then unit). The next chunk's operand tiles arrive by TMA while the
// current one finishes: Psi, Phi, S_in, Z_in as soon as the first MMAs have read
// them, delta once the last MMA has.
__global__ void __launch_bounds__(kT) k_fwd_out_tc(const __grid_constant__ Params P) {
  PhaseClock pc;
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* tPsi = sm;
  unsigned char* tPhi = sm + kTileBytes;
  unsigned char* tDl = sm + 2 * kTileBytes;
  unsigned char* tMs = sm + 3 * kTileBytes;
  unsigned char* tSin = sm + 4 * kTileBytes;
  unsigned char* tZin = sm + 5 * kTileBytes;
  __shared__ uint64_t mbar, lbarA, lbarB;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, row = row_of(), wg = wg_of();
  const int items = P.N * P.nch;
  const bool tens = P.fmode == ATLAS_FMAP_TENSOR;
  TmaBatch ldA{&lbarA, 0}, ldB{&lbarB, 0};
  // thread 0: operand loads of item `it` (Psi, Phi, S_in, Z_in on A; delta on B)
  auto issue_A = [&](int it) {
    Ctx g;
    ctx_at(P, g, it / P.nch, it % P.nch);
    if (!tens) {
      tma_rows(&P.tm_q, tPsi, g.n, g.t0, ldA.bar);
      tma_rows(&P.tm_k, tPhi, g.n, g.kp0, ldA.bar);
    }
    const unsigned char* Sin = P.stb + ((int64_t)g.n * P.nch + g.c) * 2 * kTileBytes;
    tma_tile(tSin, Sin, ldA.bar);
    tma_tile(tZin, Sin + kTileBytes, ldA.bar);
    tma_commit(ldA);
  };
  auto issue_B = [&](int it) {
    Ctx g;
    ctx_at(P, g, it / P.nch, it % P.nch);
    tma_rows(&P.tm_dl, tDl, g.n, g.kp0, ldB.bar);
    tma_commit(ldB);
  };
  if (tid == 0) {
    tma_init(ldA);
    tma_init(ldB);
    if ((int)blockIdx.x < items) {
      issue_A(blockIdx.x);
      issue_B(blockIdx.x);
    }
  }
  Sync sy{&mbar, &tbase, 0, P.status};
  GatePre gp;
  if ((int)blockIdx.x < items) gates_fetch(P, blockIdx.x / P.nch, blockIdx.x % P.nch, gp, kT);
  const uint32_t tm = tc_setup(sy);
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int nxt = it + gridDim.x;
    SmemAlloc sa{reinterpret_cast<float*>(sm + 6 * kTileBytes), 0};
    Ctx cx;
    ctx_at(P, cx, it / P.nch, it % P.nch);
    zero_tile(tMs);  // the last MMA of the previous chunk is done with it
    if (tens) {      // fp32 phi rows, converted here (no TMA)
      fill_rows_psi(P, cx, tPsi);
      fill_keys_phi(P, cx, tPhi);
    }
    gates_to_smem(P, sa, cx, gp, kT);
    if (nxt < items) gates_fetch(P, nxt / P.nch, nxt % P.nch, gp, kT);  // the next chunk's, in flight
    float* sSv = sa.take(kR + 1);
    float* sZv = sa.take(kR + 1);
    float* zZv = sa.take(kR + 1);
    const int n = cx.n, L = cx.L;
    __syncthreads();  // gates visible, tMs zero
    pc.mark(16);
    if (wg == 0) {  // column j = row of tMs: cS of key j before each token i (tile zero-filled)
      const int j = row;
      fwd_column_z(P, cx, j, [&](int i, float cs, float, float) { st_bf(tMs, i, j, cs); });
    } else if (wg == 1 && row < 32) {
      fwd_scalars_warp(cx, sSv, sZv, zZv);  // state-path scalars before token i
    }
    tma_wait(ldA, P.status);
    if (wg > 0) {
      zero_rows_from(tPsi, L, 128, kT - 128);
      loaders_sync();
      phi_xform(P, tPsi, 128, kT - 128);
      phi_xform(P, tPhi, 128, kT - 128);
    }
    pc.mark(17);
    smem_to_tc();
    if (tid == 0) {
      mma_chain(tm, op(tPsi, kD, 0), op(tPhi, kD, 0), kD / 16, kR, false);          // A2 = Psi Phi^T
      mma_chain(tm + 128, op(tPsi, kD, 0), op(tSin, kD, 0), kD / 16, kD, false);    // Psi S_in^T
      mma_chain(tm + 256, op(tPsi, kD, 0), op(tZin, kD, 0), kD / 16, kD, false);    // Psi Z_in^T
    }
    ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 512);
    if (tid == 0 && nxt < items) issue_A(nxt);  // Psi, Phi, S_in, Z_in are free
    pc.mark(19);
#pragma unroll
    for (int h = 0; h < kCPW; ++h) {  // Ms = cS o A2 (row `row`, this warpgroup's columns)
      const int c16 = wg * kCPW + h;
      float a[16], m0[8], m1[8];
      umma::tmem_ld16(lane_addr(tm, c16 * 16), a);
      umma::tmem_ld_wait();
      load_unit(tMs, row, 2 * c16, kR, m0);
      load_unit(tMs, row, 2 * c16 + 1, kR, m1);
#pragma unroll
      for (int i = 0; i < 8; ++i) { m0[i] *= a[i]; m1[i] *= a[8 + i]; }
      store_unit(tMs, row, 2 * c16, kR, m0);
      store_unit(tMs, row, 2 * c16 + 1, kR, m1);
    }
    pc.mark(20);
    if (tid == 0) tma_wait(ldB, P.status);  // delta, read only by the MMA thread 0 issues
    smem_to_tc();
    if (tid == 0) mma_chain(tm + 384, op(tMs, kR, 0), op(tDl, kD, 1), 8, kD, false);
    ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 512);
    if (tid == 0 && nxt < items) issue_B(nxt);  // delta is free
    pc.mark(21);
    {
      const int i = row;
      const float ss = i < L ? sSv[i] : 0.f, sz = i < L ? sZv[i] : 0.f;
#pragma unroll
      for (int h = 0; h < kCPW; ++h) {
        const int c16 = wg * kCPW + h;
        float yi[16], ps[16], pz[16];
        umma::tmem_ld16(lane_addr(tm, 384 + c16 * 16), yi);
        umma::tmem_ld16(lane_addr(tm, 128 + c16 * 16), ps);
        umma::tmem_ld16(lane_addr(tm, 256 + c16 * 16), pz);
        umma::tmem_ld_wait();
        if (i < L) {
#pragma unroll
          for (int k = 0; k < 16; ++k) yi[k] += ss * ps[k] + sz * pz[k];
          st16bf(reinterpret_cast<__nv_bfloat16*>(P.y) + ((int64_t)n * P.T + cx.t0 + i) * P.dv + c16 * 16, yi);
        }
      }
    }
    pc.mark(22);
    umma::fence_before();
    __syncthreads();  // TMEM read and sSv / sZv used before the next chunk rewrites them
    umma::fence_after();
  }
  tc_teardown(tm);
}

// Chunk 0 with a carried buffer: y_i += sum_jb cS_i[jb] Buf_jb psi_i (dense
// buffer entries) as one block GEMM over K = (e-1) d_phi on CUDA cores.
// Grid (column tiles of d_v, unit).
__global__ void __launch_bounds__(kThreads) k_fwd_buf_y(Params P) {
  extern __shared__ float smem[];
  SmemAlloc sa{smem, 0};
  Ctx cx;
  load_ctx(P, sa, cx, kThreads, 0);  // chunk 0 (blockIdx.x picks the column tile)
  const int L = cx.L, e1 = P.e - 1, dv = P.dv, dphi = P.dphi, n = cx.n, nn0 = blockIdx.x * 64;
  float* cSb = sa.take(L * e1);      // cS before token i for buffer key jb
  float* psi = sa.take(L * dphi);
  float* stage = sa.take(kStageFloats);
  __syncthreads();
  if ((int)threadIdx.x < e1) {
    const int j = threadIdx.x;
    float cs = 0.f, cz = 0.f;
    for (int i = 0; i < L; ++i) {
      cSb[i * e1 + j] = cs;
      cz = cx.be[i] * cz + wgt(P, cx, i, j);
      cs = cx.al[i] * cs - cx.et[i] * cz;
    }
  }
  for (int x = threadIdx.x; x < L * dphi; x += kThreads) psi[x] = load_phi(P, n, x / dphi, x % dphi, true);
  __syncthreads();
  const float* bufn = P.buf + (int64_t)n * e1 * dv * dphi;
  bgemm(stage, L, min(64, dv - nn0),
        [&](int i, int c, float acc) {
          const int64_t off = ((int64_t)n * P.T + i) * dv + nn0 + c;
          stio(P.y, off, ldio(P.y, off, P.bf) + acc, P.bf);
        },
        seg(e1 * dphi,
            [&](int i, int kk) {
              const int jb = kk / dphi;
              return cSb[i * e1 + jb] * psi[i * dphi + kk - jb * dphi];
            },
            [&](int kk, int c) {
              const int jb = kk / dphi;
              return bufn[((int64_t)jb * dv + nn0 + c) * dphi + kk - jb * dphi];
            }));
}

}  // namespace tc
}  // namespace atlas
