// Tensor-core (tcgen05) backward chunk kernels. Together they produce what
// k_bwd_chunk + k_bwd_grads (chunk_kernels.cuh) produce, split by operand set
// so that each kernel keeps at most six 32 KB operand tiles in shared memory:
//
//   k_bwd_chunk_tc        adjoint increments dShat, dZhat of a chunk   tiles dY*eS, dY*eZ, Psi
//   k_bwd_keys_tc         Phi F^T, delta F (Gram entries <F, R_j>,     tiles Phi, delta, F_S|Psi,
//                         d delta and d phi through F), then            F_Z|dY, cS|M3, M1
//                         A1 = dY delta^T, A2 = Psi Phi^T, the Gram
//                         block G = A1 o A2 and the intra-chunk terms
//   k_bwd_state_gates_tc  Psi S_in^T, dY S_in (and Z_in): the Gram     tiles Psi, dY, S_in, Z_in,
//                         entries <dy_q psi_q^T, S_in>, d psi, the      F_S, F_Z, then cS, G, cZ,
//                         four <F, S> dots; then d alpha, d eta,        eS+, eZ+
//                         d beta and the window-gate gradients as
//                         bilinear forms of the Gram matrix (W_e[i] =
//                         W_b[i + 1], so no cZ+ tile)
// Gram pieces travel between the two through the backward scratch:
//   xf[N][nch][128][2], G tiles [N][nch][32 KB].
#pragma once
#include "tc_fwd.cuh"

namespace atlas {
namespace tc {

__device__ __forceinline__ int64_t chunk_id(const Params& P, const Ctx& cx) { return (int64_t)cx.n * P.nch + cx.c; }


// Scalars of the adjoint transform of the chunk (rows r = 0..L) computed by one thread.
__device__ __forceinline__ void adj_scalars(const Ctx& cx, float* hS, float* hZS, float* hZZ) {
  const int L = cx.L;
  float hs = 1.f, hzs = -cx.et[L - 1], hzz = 1.f;
  hS[L] = hs; hZS[L] = hzs; hZZ[L] = hzz;
  for (int r = L - 1; r >= 0; --r) {
    const float eta = r >= 1 ? cx.et[r - 1] : 0.f;
    hs = cx.al[r] * hs;
    hzz = cx.be[r] * hzz;
    hzs = cx.be[r] * hzs - eta * hs;
    hS[r] = hs; hZS[r] = hzs; hZZ[r] = hzz;
  }
}

// ===========================================================================
// adjoint increments at the chunk input from the chunk's own dy:
//   dShat = dY^T diag(eS_0) Psi,  dZhat = dY^T diag(eZ_0) Psi
// ===========================================================================
__global__ void __launch_bounds__(kT) k_bwd_chunk_tc(const __grid_constant__ Params P) {
  PhaseClock pc;
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* tYS = sm;
  unsigned char* tYZ = sm + kTileBytes;
  unsigned char* tPsi = sm + 2 * kTileBytes;
  SmemAlloc sa{reinterpret_cast<float*>(sm + 3 * kTileBytes), 0};
  __shared__ uint64_t mbar, lbar;
  __shared__ uint32_t tbase;
  Ctx cx;
  ctx_geom(P, cx);
  TmaBatch ld{&lbar, 0};
  if (threadIdx.x == 0) tma_init(ld);
  load_rows_psi(P, cx, tPsi, ld);
  load_rows_dy(P, cx, tYS, ld);
  if (threadIdx.x == 0) tma_commit(ld);
  load_ctx(P, sa, cx, kT);
  float* eS0 = sa.take(kR + 1);
  float* eZ0 = sa.take(kR + 1);
  float* zZ = sa.take(kR + 1);
  float* hS = sa.take(kR + 1);
  float* hZS = sa.take(kR + 1);
  float* hZZ = sa.take(kR + 1);
  const int L = cx.L, tid = threadIdx.x, row = row_of(), wg = wg_of();
  Sync sy{&mbar, &tbase, 0, P.status};
  const uint32_t tm = tc_setup(sy, 256);
  pc.mark(48);
  // adjoint weights of token q at the chunk input: eS_0[q], eZ_0[q] equal the
  // forward state scalars sS[q], sZ[q] (the adjoint and forward recurrences are
  // transposes of each other); the chunk's adjoint transform is hS, hZS, hZZ at row 0
  if (tid < 32) {
    fwd_scalars_warp(cx, eS0, eZ0, zZ);
    if (tid == 0)
      for (int q = L; q < kR; ++q) { eS0[q] = 0.f; eZ0[q] = 0.f; }
  } else if (tid < 64) {
    adj_scalars_warp(cx, hS, hZS, hZZ);
    if (tid == 32) {
      float* o = P.acs + chunk_id(P, cx) * 4;
      o[0] = hS[0]; o[1] = hZS[0]; o[2] = hZZ[0]; o[3] = 0.f;
    }
  }
  tma_wait(ld, P.status);
  zero_rows_from(tPsi, L);
  zero_rows_from(tYS, L);
  __syncthreads();
  pc.mark(49);
  {  // dY rows scaled by eS0 (in place) and by eZ0 (into tYZ); psi feature map
    constexpr int kCpr = kD / 8;
    for (int u = tid; u < kR * kCpr; u += kT) {
      int r, cb;
      unit_rc(u, kCpr, r, cb);
      float v[8], z[8];
      unpack_unit(*reinterpret_cast<const uint4*>(tYS + 16 * u), v);
      const float a = eS0[r], b = eZ0[r];
#pragma unroll
      for (int k = 0; k < 8; ++k) { z[k] = b * v[k]; v[k] *= a; }
      *reinterpret_cast<uint4*>(tYS + 16 * u) = pack_unit(v);
      *reinterpret_cast<uint4*>(tYZ + 16 * u) = pack_unit(z);
    }
    phi_xform(P, tPsi);
  }
  pc.mark(50);
  smem_to_tc();
  if (tid == 0) {
    mma_chain(tm, op(tYS, kD, 1), op(tPsi, kD, 1), 8, kD, false);
    mma_chain(tm + 128, op(tYZ, kD, 1), op(tPsi, kD, 1), 8, kD, false);
  }
  ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 256);
  pc.mark(51);
  {
    const int64_t D2 = (int64_t)kD * kD;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(P.adj) + chunk_id(P, cx) * 2 * D2 + (int64_t)row * kD;
#pragma unroll
    for (int h = 0; h < kCPW; ++h) {
      const int c16 = wg * kCPW + h;
      float a[16], b[16];
      umma::tmem_ld16(lane_addr(tm, c16 * 16), a);
      umma::tmem_ld16(lane_addr(tm, 128 + c16 * 16), b);
      umma::tmem_ld_wait();
      st16bf(dst + c16 * 16, a);
      st16bf(dst + D2 + c16 * 16, b);
    }
  }
  tc_teardown(tm, 256);  pc.mark(52);

}

// Window-summed adjoint scalars of key j: wZS_j = sum_i W(i,j) hZS_{i+1}, wZZ likewise.
__device__ __forceinline__ void key_adj_weights(const Params& P, const Ctx& cx, int j, const float* hZS,
                                                const float* hZZ, float& a, float& b) {
  a = 0.f;
  b = 0.f;
  if (j >= cx.K) return;
  for (int i = max(0, j - P.e + 1); i <= min(cx.L - 1, j); ++i) {
    const float w = wgt(P, cx, i, j);
    a += w * hZS[i + 1];
    b += w * hZZ[i + 1];
  }
}

// ===========================================================================
// key-side backward in one pass:
//   phase 1  P1 = Phi F_S^T, P2 = Phi F_Z^T, Q1 = delta F_S, Q2 = delta F_Z
//            -> X[F][R_j]; d delta = wZS P1 + wZZ P2 and d phi = wZS Q1 + wZZ Q2 are
//            written back into TMEM (tcgen05.st) over P1 and Q1
//   phase 2  A1 = dY delta^T, A2 = Psi Phi^T -> G = A1 o A2 (scratch), M3 = cS o A1,
//            M1 = cS o A2
//   phase 3  d delta += M1 dY, d phi += M3^T Psi (accumulating in TMEM), I5 = M3 Phi
//   out      d delta, d phi written once (own keys / halo partials); d psi = I5 (bf16)
// The window-summed adjoint weight of key j for token q, sum_i W(i, j) eZ_{i+1}[q],
// equals the forward coefficient cS_q[j] (both are
// -sum_{n<q} prod_{l=n+1}^{q-1} alpha_l eta_n sum_{m<=n} prod_{l=m+1}^{n} beta_l W(m, j)),
// so one coefficient tile (cS, built by warpgroup 0 while the operand tiles
// arrive by cp.async) serves the adjoint weights as well, and M2 = wE o A1 = M3.
// ===========================================================================
__global__ void __launch_bounds__(kT) k_bwd_keys_tc(const __grid_constant__ Params P) {
  PhaseClock pc;
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* tPhi = sm;
  unsigned char* tDl = sm + kTileBytes;       // delta
  unsigned char* tFS = sm + 2 * kTileBytes;   // F_S, later Psi
  unsigned char* tFZ = sm + 3 * kTileBytes;   // F_Z, later dY
  unsigned char* tM3 = sm + 4 * kTileBytes;   // cS, later M3 (= M2)
  unsigned char* tM1 = sm + 5 * kTileBytes;   // M1
  SmemAlloc sa{reinterpret_cast<float*>(sm + 6 * kTileBytes), 0};
  __shared__ uint64_t mbar, lbar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, e = P.e, row = row_of(), wg = wg_of();
  const int items = P.N * P.nch;
  const bool tens = P.fmode == ATLAS_FMAP_TENSOR;
  TmaBatch ld{&lbar, 0};
  // thread 0: the first operand batch of item `it` (the adjoint tiles may go in earlier than the rows,
  // still on the same barrier phase); `rows` also commits the batch
  auto issue_adj = [&](int it) {
    const unsigned char* Fa = P.adjb + (int64_t)it * 2 * kTileBytes;  // item = n nch + c = chunk id
    tma_tile(tFS, Fa, ld.bar);
    tma_tile(tFZ, Fa + kTileBytes, ld.bar);
  };
  auto issue_rows = [&](int it) {
    Ctx g;
    ctx_at(P, g, it / P.nch, it % P.nch);
    if (!tens) tma_rows(&P.tm_k, tPhi, g.n, g.kp0, ld.bar);
    tma_rows(&P.tm_dl, tDl, g.n, g.kp0, ld.bar);
    tma_commit(ld);
  };
  if (tid == 0) {
    tma_init(ld);
    if ((int)blockIdx.x < items) {
      issue_adj(blockIdx.x);
      issue_rows(blockIdx.x);
    }
  }
  GatePre gp;
  if ((int)blockIdx.x < items) gates_fetch(P, blockIdx.x / P.nch, blockIdx.x % P.nch, gp, kT);
  Sync sy{&mbar, &tbase, 0, P.status};
  const uint32_t tm = tc_setup(sy);
  // Persistent: each CTA walks chunks it = blockIdx.x, + gridDim.x, ... (chunk fastest); the next
  // chunk's adjoint tiles load while this one's hand-offs are written, its key rows right after.
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
  const int nxt = it + gridDim.x;
  SmemAlloc sa{reinterpret_cast<float*>(sm + 6 * kTileBytes), 0};
  Ctx cx;
  ctx_at(P, cx, it / P.nch, it % P.nch);
  const int64_t cid = chunk_id(P, cx);
  if (tens) fill_keys_phi(P, cx, tPhi);
  gates_to_smem(P, sa, cx, gp, kT);
  if (nxt < items) gates_fetch(P, nxt / P.nch, nxt % P.nch, gp, kT);
  float* hS = sa.take(kR + 1);
  float* hZS = sa.take(kR + 1);
  float* hZZ = sa.take(kR + 1);
  float* part = sa.take(2 * kWG * kR);
  const int n = cx.n, K = cx.K, L = cx.L;
  zero_tile(tM3);
  __syncthreads();  // gates visible, tM3 zero
  pc.mark(0);
  if (wg == 0) {
    fwd_column_z(P, cx, row, [&](int i, float cs, float, float) { st_bf(tM3, i, row, cs); });
    if (row == 0) pc.lap(12);
  } else if (wg == 1 && row < 32) {
    adj_scalars_warp(cx, hS, hZS, hZZ);
  }
  tma_wait(ld, P.status);
  if (wg > 0) {
    loaders_sync();
    phi_xform(P, tPhi, 128, kT - 128);
    if (tid == 384) pc.lap(15);
  }
  pc.mark(1);
  smem_to_tc();
  if (tid == 0) {
    mma_chain(tm, op(tPhi, kD, 0), op(tFS, kD, 0), 8, kD, false);        // P1
    mma_chain(tm + 128, op(tPhi, kD, 0), op(tFZ, kD, 0), 8, kD, false);  // P2
    mma_chain(tm + 256, op(tDl, kD, 0), op(tFS, kD, 1), 8, kD, false);  // Q1
    mma_chain(tm + 384, op(tDl, kD, 0), op(tFZ, kD, 1), 8, kD, false);  // Q2
  }
  ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 512);
  pc.mark(4);
  load_rows_psi(P, cx, tFS, ld);  // F tiles are free once the phase-1 MMAs are done
  load_rows_dy(P, cx, tFZ, ld);
  if (threadIdx.x == 0) tma_commit(ld);
  {  // phase-1 epilogue, row j: X[F][R_j]; F parts of d delta / d phi back into TMEM
    const int j = row;
    float wzs, wzz;
    key_adj_weights(P, cx, j, hZS, hZZ, wzs, wzz);
    float xS = 0.f, xZ = 0.f;
    for (int h = 0; h < kCPW; ++h) {
      const int c16 = wg * kCPW + h;
      float p1[16], p2[16], q1[16], q2[16], dl[16];
      umma::tmem_ld16(lane_addr(tm, c16 * 16), p1);
      umma::tmem_ld16(lane_addr(tm, 128 + c16 * 16), p2);
      umma::tmem_ld16(lane_addr(tm, 256 + c16 * 16), q1);
      umma::tmem_ld16(lane_addr(tm, 384 + c16 * 16), q2);
      umma::tmem_ld_wait();
      load_unit(tDl, j, 2 * c16, kD, *reinterpret_cast<float(*)[8]>(dl));
      load_unit(tDl, j, 2 * c16 + 1, kD, *reinterpret_cast<float(*)[8]>(dl + 8));
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        xS += p1[i] * dl[i];
        xZ += p2[i] * dl[i];
        p1[i] = wzs * p1[i] + wzz * p2[i];
        q1[i] = wzs * q1[i] + wzz * q2[i];
      }
      umma::tmem_st16(lane_addr(tm, c16 * 16), p1);
      umma::tmem_st16(lane_addr(tm, 256 + c16 * 16), q1);
    }
    umma::tmem_st_wait();
    part[(wg * 2 + 0) * kR + j] = xS;
    part[(wg * 2 + 1) * kR + j] = xZ;
  }
  umma::fence_before();
  tma_wait(ld, P.status);
  zero_rows_from(tFS, L);
  zero_rows_from(tFZ, L);
  __syncthreads();  // psi / dY rows landed; P2 / Q2 columns are free
  if (wg == 0) {
    float a = 0.f, b = 0.f;
    for (int g = 0; g < kWG; ++g) { a += part[(2 * g) * kR + row]; b += part[(2 * g + 1) * kR + row]; }
    float* xf = P.xf + (cid * kR + row) * 2;
    xf[0] = row < K ? a : 0.f;
    xf[1] = row < K ? b : 0.f;
  }
  phi_xform(P, tFS);
  pc.mark(6);
  smem_to_tc();
  if (tid == 0) {
    mma_chain(tm + 128, op(tFZ, kD, 0), op(tDl, kD, 0), 8, kR, false);   // A1[q][j] = dY delta^T
    mma_chain(tm + 384, op(tFS, kD, 0), op(tPhi, kD, 0), 8, kR, false);  // A2[q][j] = Psi Phi^T
  }
  ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 512);
  pc.mark(7);
  {  // phase-2 epilogue, row q: G, M3 = cS o A1, M1 = cS o A2
    const int q = row;
    unsigned char* gdst = reinterpret_cast<unsigned char*>(P.gt) + cid * kTileBytes;
    for (int h4 = 0; h4 < kCPW; ++h4) {
      const int c16 = wg * kCPW + h4;
      float a1[16], a2[16];
      umma::tmem_ld16(lane_addr(tm, 128 + c16 * 16), a1);
      umma::tmem_ld16(lane_addr(tm, 384 + c16 * 16), a2);
      umma::tmem_ld_wait();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int cb = 2 * c16 + h;
        float g[8], c3[8], m1[8];
        load_unit(tM3, q, cb, kR, c3);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float x1 = a1[8 * h + k], x2 = a2[8 * h + k];
          g[k] = x1 * x2;
          m1[k] = c3[k] * x2;
          c3[k] *= x1;
        }
        store_unit(gdst, q, cb, kR, g);
        store_unit(tM3, q, cb, kR, c3);
        store_unit(tM1, q, cb, kR, m1);
      }
    }
  }
  pc.mark(8);
  smem_to_tc();
  if (tid == 0) {
    mma_chain(tm, op(tM1, kR, 1), op(tFZ, kD, 1), 8, kD, true);          // d delta += M1 dY
    mma_chain(tm + 256, op(tM3, kR, 1), op(tFS, kD, 1), 8, kD, true);    // d phi   += M2 Psi (M2 = M3)
    mma_chain(tm + 128, op(tM3, kR, 0), op(tPhi, kD, 1), 8, kD, false);  // I5 = M3 Phi
  }
  ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 512);
  if (tid == 0 && nxt < items) issue_adj(nxt);  // F_S / F_Z tiles (Psi, dY now) are read by no one any more
  pc.mark(9);
  {
    const int r = row, p = cx.kp0 + r;
    const bool own = r < K && p >= cx.t0, halo = r < K && p >= 0 && p < cx.t0;
    const int e1 = e > 1 ? e - 1 : 1;
    // own keys: bf16 hand-off to finalize; halo keys (of the previous chunk's tokens): fp32 partials
    // (the MMAs are done with every tile: own rows are staged in tPhi / tDl / tM1 and
    // leave row-contiguous below)
    float* ddh = P.hdd + (cid * e1 + (r < e - 1 ? r : 0)) * P.dv;
    float* dph = P.hdp + (cid * e1 + (r < e - 1 ? r : 0)) * P.dphi;
    for (int h = 0; h < kCPW; ++h) {
      const int c16 = wg * kCPW + h;
      float a[16], b[16], i5[16];
      umma::tmem_ld16(lane_addr(tm, c16 * 16), a);
      umma::tmem_ld16(lane_addr(tm, 256 + c16 * 16), b);
      umma::tmem_ld16(lane_addr(tm, 128 + c16 * 16), i5);
      umma::tmem_ld_wait();
      if (own) {
        stage16(tPhi, r, c16, a);
        stage16(tDl, r, c16, b);
      } else if (halo) {
        st16f(ddh + c16 * 16, a);
        st16f(dph + c16 * 16, b);
      }
      if (r < L) stage16(tM1, r, c16, i5);  // k_bwd_state_gates_tc adds the state part
    }
  }
  __syncthreads();
  {
    const int64_t base = (int64_t)n * P.T;
    auto own_row = [&](int r) { return r < K && cx.kp0 + r >= cx.t0; };
    store_rows_from_tile(tPhi, [&](int r) { return own_row(r) ? P.ddb + (base + cx.kp0 + r) * P.dv : nullptr; });
    store_rows_from_tile(tDl, [&](int r) { return own_row(r) ? P.dpb + (base + cx.kp0 + r) * P.dphi : nullptr; });
    store_rows_from_tile(tM1, [&](int r) { return r < L ? P.dpsib + (base + cx.t0 + r) * P.dphi : nullptr; });
  }
  pc.mark(10);
  umma::fence_async_smem();
  umma::fence_before();
  __syncthreads();  // the staged rows are written out; TMEM read
  umma::fence_after();
  if (tid == 0 && nxt < items) issue_rows(nxt);
  }
  tc_teardown(tm);
}

// ===========================================================================
// state side and gate gradients in one kernel.
//   state  G_S = Psi S_in^T, G_Z = Psi Z_in^T (-> X[D_q][S_in], X[D_q][Z_in]),
//          H_S = dY S_in, H_Z = dY Z_in (-> d psi = I5 + sS H_S + sZ H_Z; I5 from
//          k_bwd_keys_tc, which runs first; d psi leaves as bf16), and the four Gram
//          scalars <F_S|F_Z, S_in|Z_in> from the staged tiles while the MMAs run;
//   gates  d alpha, d eta, d beta and the window-gate gradients as bilinear forms
//          of the Gram matrix: W_a = C_S G^T, W_b = C_Z G^T (W_e = C_Z+ G^T is W_b
//          shifted by one row) and E_Z+ G on tensor cores, the F / S_in / Z_in rows and columns of the Gram
//          matrix folded in on CUDA cores.
// Once the state MMAs and the dots are done, five of the six tiles take the
// coefficient tiles of the gate gradients (warpgroups 0 and 1 build them)
// while warpgroups 2 and 3 run the state epilogue; the Gram block G then
// replaces dY. X[D_q][S_in|Z_in] and the four scalars stay on chip.
// ===========================================================================
constexpr int kGateParts = 10;
__device__ __forceinline__ void wg_sync(int id) {  // named barrier of one warpgroup
  asm volatile("bar.sync %0, 128;\n" ::"r"(id) : "memory");
}
__device__ __forceinline__ void pair_sync() {  // named barrier of warpgroups 2 and 3
  asm volatile("bar.sync 4, 256;\n" ::: "memory");
}
__global__ void __launch_bounds__(kT) k_bwd_state_gates_tc(const __grid_constant__ Params P) {
  PhaseClock pc;
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* tPsi = sm;
  unsigned char* tY = sm + kTileBytes;
  unsigned char* tSin = sm + 2 * kTileBytes;
  unsigned char* tZin = sm + 3 * kTileBytes;
  unsigned char* tFS = sm + 4 * kTileBytes;
  unsigned char* tFZ = sm + 5 * kTileBytes;
  unsigned char* tCS = tPsi;   // cS_i[j]      (state before token i)
  unsigned char* tG = tZin;    // Gram block (Z_in is free after the state MMAs)
  unsigned char* tCZp = tSin;  // cZ_i[j], rows 0..L (row L: after the last token)
  unsigned char* tES = tFS;    // eS_{i+1}[q]
  unsigned char* tEZ = tFZ;    // eZ_{i+1}[q]
  SmemAlloc sa{reinterpret_cast<float*>(sm + 6 * kTileBytes), 0};
  __shared__ uint64_t mbar, lbar;
  __shared__ uint32_t tbase;
  Ctx cx;
  ctx_geom(P, cx);
  const int64_t cid = chunk_id(P, cx);
  TmaBatch ld{&lbar, 0};
  if (threadIdx.x == 0) tma_init(ld);
  {  // every operand tile in flight before anything else
    const unsigned char* Sin = P.stb + cid * 2 * kTileBytes;
    const unsigned char* FS = P.adjb + cid * 2 * kTileBytes;
    load_rows_psi(P, cx, tPsi, ld);
    load_rows_dy(P, cx, tY, ld);
    load_tile(tSin, Sin, ld);
    load_tile(tZin, Sin + kTileBytes, ld);
    load_tile(tFS, FS, ld);
    load_tile(tFZ, FS + kTileBytes, ld);
    if (threadIdx.x == 0) tma_commit(ld);
  }
  load_ctx(P, sa, cx, kT);
  float* sS = sa.take(kR + 1);
  float* sZ = sa.take(kR + 1);
  float* zZ = sa.take(kR + 1);
  float* hS = sa.take(kR + 1);
  float* hZS = sa.take(kR + 1);
  float* hZZ = sa.take(kR + 1);
  float* xq = sa.take(2 * kR);
  float* xf = sa.take(2 * kR);
  float* xs = sa.take(4);
  float* duj = sa.take(kR);
  float* red = sa.take(4 * (kT / 32));
  float* part = sa.take(kGateParts * (kWG - 1) * kR);  // state: xq partials; gates: partial sums of warpgroups 1..
  float* sh0 = sa.take(2 * kR);                        // warpgroup 0's row-shifted gate sums
  const int n = cx.n, K = cx.K, L = cx.L, tid = threadIdx.x, e = P.e, row = row_of(), wg = wg_of();
  if (tid < 2 * kR / 4) cp16(xf + 4 * tid, P.xf + cid * 2 * kR + 4 * tid, true);
  if (tid < kR) duj[tid] = 0.f;
  Sync sy{&mbar, &tbase, 0, P.status};
  const uint32_t tm = tc_setup(sy);  // (its barrier also publishes the gates)
  pc.mark(32);
  if (tid < 32) fwd_scalars_warp(cx, sS, sZ, zZ);
  else if (tid < 64) adj_scalars_warp(cx, hS, hZS, hZZ);
  async_wait();  // xf
  tma_wait(ld, P.status);
  zero_rows_from(tPsi, L);
  zero_rows_from(tY, L);
  __syncthreads();
  phi_xform(P, tPsi);
  pc.mark(33);
  smem_to_tc();
  if (tid == 0) {
    mma_chain(tm, op(tPsi, kD, 0), op(tSin, kD, 0), 8, kD, false);
    mma_chain(tm + 128, op(tPsi, kD, 0), op(tZin, kD, 0), 8, kD, false);
    mma_chain(tm + 256, op(tY, kD, 0), op(tSin, kD, 1), 8, kD, false);
    mma_chain(tm + 384, op(tY, kD, 0), op(tZin, kD, 1), 8, kD, false);
  }
  {  // <F_S|F_Z, S_in|Z_in>: elementwise over the raw tiles (same layout for all four)
    float s00 = 0.f, s01 = 0.f, s10 = 0.f, s11 = 0.f;
    for (int u = tid; u < kTileBytes / 16; u += kT) {
      const uint4 a = reinterpret_cast<const uint4*>(tFS)[u], b = reinterpret_cast<const uint4*>(tFZ)[u];
      const uint4 c = reinterpret_cast<const uint4*>(tSin)[u], d = reinterpret_cast<const uint4*>(tZin)[u];
      const __nv_bfloat162* fa = reinterpret_cast<const __nv_bfloat162*>(&a);
      const __nv_bfloat162* fb = reinterpret_cast<const __nv_bfloat162*>(&b);
      const __nv_bfloat162* fc = reinterpret_cast<const __nv_bfloat162*>(&c);
      const __nv_bfloat162* fd = reinterpret_cast<const __nv_bfloat162*>(&d);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 fs = __bfloat1622float2(fa[k]), fz = __bfloat1622float2(fb[k]);
        const float2 si = __bfloat1622float2(fc[k]), zi = __bfloat1622float2(fd[k]);
        s00 += fs.x * si.x + fs.y * si.y;
        s01 += fs.x * zi.x + fs.y * zi.y;
        s10 += fz.x * si.x + fz.y * si.y;
        s11 += fz.x * zi.x + fz.y * zi.y;
      }
    }
    const float v[4] = {s00, s01, s10, s11};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float t = v[k];
      for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
      if ((tid & 31) == 0) red[k * (kT / 32) + (tid >> 5)] = t;
    }
  }
  // d psi part I5 of this thread's row for the state epilogue of warpgroups 2, 3
  // (column groups 4 (wg - 2) .. + 3), fetched while the MMAs run
  const int64_t grow = (int64_t)n * P.T + cx.t0 + row;
  uint4 i5v[4][2];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    i5v[h][0] = i5v[h][1] = make_uint4(0u, 0u, 0u, 0u);
    if (wg >= 2 && row < L) {
      const uint4* src = reinterpret_cast<const uint4*>(P.dpsib + grow * P.dphi + ((wg - 2) * 4 + h) * 16);
      i5v[h][0] = src[0];
      i5v[h][1] = src[1];
    }
  }
  ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 512);
  __syncthreads();  // the state MMAs and the dots are done with Psi, S_in, Z_in, F_S, F_Z
  pc.mark(34);
  if (wg == 0) {  // forward coefficients of key j (columns of tCS, tCZp)
    zero_tile_wg(tCS);
    zero_tile_wg(tCZp);
    wg_sync(2);
    const int j = row;
    fwd_column_z(P, cx, j, [&](int i, float cs, float cz, float czn) {
      st_bf(tCS, i, j, cs);
      st_bf(tCZp, i, j, cz);
      if (i == L - 1) st_bf(tCZp, L, j, czn);
    });
    if (row == 0) pc.lap(24);
  } else if (wg == 1) {  // adjoint coefficients of token q (columns of tES, tEZ): rows i <- eS_{i+1}, eZ_{i+1}
    zero_tile_wg(tES);
    zero_tile_wg(tEZ);
    wg_sync(3);
    const int q = row;
    adj_column_z(cx, q, [&](int i, float es, float ez) {
      st_bf(tES, i, q, es);
      st_bf(tEZ, i, q, ez);
    });
    if (row == 0) pc.lap(25);
  } else {  // state epilogue (warpgroups 2, 3): d psi, X[D_q][S_in|Z_in]; the Gram block arrives meanwhile
    if (tid == 256) {
      tma_tile(tG, reinterpret_cast<const unsigned char*>(P.gt) + cid * kTileBytes, ld.bar);
      tma_commit(ld);
    }
    const int q = row;
    float a = 0.f, b = 0.f;
    const float ss = q < L ? sS[q] : 0.f, sz = q < L ? sZ[q] : 0.f;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int c16 = (wg - 2) * 4 + h;
      float gs[16], gz[16], hs[16], hz[16], y0[8], y1[8];
      umma::tmem_ld16(lane_addr(tm, c16 * 16), gs);
      umma::tmem_ld16(lane_addr(tm, 128 + c16 * 16), gz);
      umma::tmem_ld16(lane_addr(tm, 256 + c16 * 16), hs);
      umma::tmem_ld16(lane_addr(tm, 384 + c16 * 16), hz);
      umma::tmem_ld_wait();
      if (q < L) {
        load_unit(tY, q, 2 * c16, kD, y0);
        load_unit(tY, q, 2 * c16 + 1, kD, y1);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          a += gs[i] * y0[i] + gs[8 + i] * y1[i];
          b += gz[i] * y0[i] + gz[8 + i] * y1[i];
        }
        float d[16], i0[8], i1[8];
        unpack_unit(i5v[h][0], i0);
        unpack_unit(i5v[h][1], i1);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          d[i] = ss * hs[i] + sz * hz[i] + i0[i];
          d[8 + i] = ss * hs[8 + i] + sz * hz[8 + i] + i1[i];
        }
        st16bf(P.dpsib + grow * P.dphi + c16 * 16, d);
      }
    }
    part[((wg - 2) * 2 + 0) * kR + q] = a;
    part[((wg - 2) * 2 + 1) * kR + q] = b;
    umma::fence_before();
    pair_sync();  // both halves of X[D_q] in part; dY no longer read
    if (wg == 2) {
      xq[2 * q] = q < L ? part[q] + part[2 * kR + q] : 0.f;
      xq[2 * q + 1] = q < L ? part[kR + q] + part[3 * kR + q] : 0.f;
    } else if (row < 4) {
      float t = 0.f;
      for (int w = 0; w < kT / 32; ++w) t += red[row * (kT / 32) + w];
      xs[row] = t;
    }
    if (tid == 256) pc.lap(26);
    tma_wait(ld, P.status);
    if (tid == 256) pc.lap(27);
  }
  if (tid == 0) tma_wait(ld, P.status);  // the Gram tile, before thread 0 issues the MMAs that read it
  pc.mark(35);
  smem_to_tc();  // coefficient tiles, G, xq, xs ready; the state accumulators are read
  if (tid == 0) {
    mma_chain(tm, op(tCS, kR, 0), op(tG, kR, 0), 8, kR, false);         // W_a[i][q]
    mma_chain(tm + 256, op(tCZp, kR, 0), op(tG, kR, 0), 8, kR, false);  // W_b[i][q]
    mma_chain(tm + 384, op(tEZ, kR, 0), op(tG, kR, 1), 8, kR, false);   // E_Z+ G [i][j]
  }
  ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 512);
  pc.mark(36);
  const int i = row;
  float acc[kGateParts];
#pragma unroll
  for (int k = 0; k < kGateParts; ++k) acc[k] = 0.f;
#pragma unroll
  for (int h4 = 0; h4 < kCPW; ++h4) {
    const int c16 = wg * kCPW + h4;
    float A[16], B[16];
    umma::tmem_ld16(lane_addr(tm, c16 * 16), A);
    umma::tmem_ld16(lane_addr(tm, 256 + c16 * 16), B);
    umma::tmem_ld_wait();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int cb = 2 * c16 + h;
      float cs8[8], czp8[8], es8[8], ez8[8], esm[8];
      load_unit(tCS, i, cb, kR, cs8);
      load_unit(tCZp, i, cb, kR, czp8);
      load_unit(tES, i, cb, kR, es8);
      load_unit(tEZ, i, cb, kR, ez8);
      load_unit(tES, i > 0 ? i - 1 : 0, cb, kR, esm);  // row i - 1, for the shifted W_e term
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int x = cb * 8 + k;  // key j (for c*) or token q (for e*)
        acc[0] += xf[2 * x] * cs8[k];        // F_S . cS_i
        acc[2] += xf[2 * x] * czp8[k];       // F_S . cZ_i
        acc[3] += xf[2 * x + 1] * czp8[k];   // F_Z . cZ_i
        acc[4] += xq[2 * x] * es8[k];        // eS_{i+1} . X[D][S_in]
        acc[5] += xq[2 * x + 1] * es8[k];    // eS_{i+1} . X[D][Z_in]
        acc[6] += xq[2 * x + 1] * ez8[k];    // eZ_{i+1} . X[D][Z_in]
        acc[7] += es8[k] * A[8 * h + k];
        acc[8] += esm[k] * B[8 * h + k];     // eS_i . W_b[i] = row i - 1's eS_{i'+1} . W_e[i']
        acc[9] += ez8[k] * B[8 * h + k];
      }
    }
  }
  // W_e[i] = W_b[i + 1] and cZ_{i+1} = cZ_i of row i + 1: the terms acc[1] = F_S . cZ_{i+1} and
  // acc[8] = eS_{i+1} . W_e[i] of row i are acc[2] and the shifted product of row i + 1.
  acc[1] = acc[2];
  if (i == 0) acc[8] = 0.f;
  if (wg >= 1) {
#pragma unroll
    for (int k = 0; k < kGateParts; ++k) part[((wg - 1) * kGateParts + k) * kR + i] = acc[k];
  } else {
    sh0[i] = acc[1];
    sh0[kR + i] = acc[8];
  }
  // window weights dW(i, j) = hZS_{i+1} X[F_S][R_j] + hZZ_{i+1} X[F_Z][R_j] + (E_Z+ G)[i][j]
  if (P.gmode != ATLAS_GATE_NONE) {
    const int rb = (threadIdx.x >> 5) & 3;  // this warp's rows [32 rb, 32 rb + 32)
#pragma unroll
    for (int h4 = 0; h4 < kCPW; ++h4) {
      const int c16 = wg * kCPW + h4;
      if (c16 * 16 + 15 < 32 * rb || c16 * 16 > 32 * rb + 31 + e - 1) continue;  // no window key here (warp-uniform)
      float W[16];
      umma::tmem_ld16(lane_addr(tm, 384 + c16 * 16), W);
      umma::tmem_ld_wait();
      if (i < L)
        for (int k = 0; k < 16; ++k) {
          const int j = c16 * 16 + k, jj = i - j + e - 1;
          if (j >= K || jj < 0 || jj >= e) continue;
          const float val = hZS[i + 1] * xf[2 * j] + hZZ[i + 1] * xf[2 * j + 1] + W[k];
          if (P.gmode == ATLAS_GATE_TOKEN) {
            if (cx.kp0 + j >= 0) atomicAdd(&duj[j], val);
          } else if (P.dgate) {
            stio(P.dgate, ((int64_t)n * P.T + cx.t0 + i) * e + jj, val, P.bf);
          }
        }
    }
  }
  __syncthreads();
  if (wg == 0 && i < L) {
    acc[1] = sh0[i + 1];
    acc[8] = sh0[kR + i + 1];
    for (int g = 1; g < kWG; ++g)
#pragma unroll
      for (int k = 0; k < kGateParts; ++k) acc[k] += part[((g - 1) * kGateParts + k) * kR + i + (k == 1 || k == 8 ? 1 : 0)];
    const float da = hS[i + 1] * (xs[0] * sS[i] + xs[1] * sZ[i] + acc[0]) + (acc[4] * sS[i] + acc[5] * sZ[i] + acc[7]);
    const float de = -(hS[i + 1] * (xs[1] * zZ[i + 1] + acc[1]) + (acc[5] * zZ[i + 1] + acc[8]));
    const float db = hZS[i + 1] * (xs[1] * zZ[i] + acc[2]) + hZZ[i + 1] * (xs[3] * zZ[i] + acc[3]) +
                     (acc[6] * zZ[i] + acc[9]);
    const int64_t r = (int64_t)n * P.T + cx.t0 + i;
    if (P.ddecay) stio(P.ddecay, r, da, P.bf);
    if (P.dlr) stio(P.dlr, r, de, P.bf);
    if (P.mom && P.dbeta) stio(P.dbeta, r, db, P.bf);
  }
  if (P.gmode == ATLAS_GATE_TOKEN && wg == 0) {
    const int j = row, p = cx.kp0 + j;
    if (j < K && p >= cx.t0) P.du[(int64_t)n * P.T + p] = duj[j];
    else if (j < K && p >= 0) P.hdu[cid * (e - 1) + j] = duj[j];
  }
  pc.mark(37);
  tc_teardown(tm);
}

// ===========================================================================
// chunk 0 with a carried omega buffer (dense entries Buf_jb, jb < e-1), after
// k_bwd_keys_tc and before k_bwd_state_gates_tc: the Gram columns of the buffer
// entries (X[F][Buf], G[q][Buf] = dy_q . Buf psi_q), their d psi terms, and the
// buffer's own gradient dBuf_jb = wZS F_S + wZZ F_Z + sum_q wE_jb[q] dy_q psi_q^T.
// Block GEMMs on CUDA cores, one CTA of kThreads per unit.
// ===========================================================================
__global__ void __launch_bounds__(kThreads) k_bwd_buf_tc(Params P) {
  extern __shared__ float smem[];
  SmemAlloc sa{smem, 0};
  Ctx cx;
  load_ctx(P, sa, cx, kThreads, 0);
  const int L = cx.L, e1 = P.e - 1, dv = P.dv, dphi = P.dphi, n = cx.n, tid = threadIdx.x;
  float* psi = sa.take(L * dphi);
  float* dy = sa.take(L * dv);
  float* cSb = sa.take(L * e1);   // cS_i[jb]
  float* wE = sa.take(e1 * L);    // wE_jb[q]
  float* gacc = sa.take(L * e1);  // G[q][jb]
  float* hS = sa.take(L + 1);
  float* hZS = sa.take(L + 1);
  float* hZZ = sa.take(L + 1);
  float* red = sa.take(32);
  float* stage = sa.take(kStageFloats);
  for (int x = tid; x < L * dphi; x += kThreads) psi[x] = load_phi(P, n, x / dphi, x % dphi, true);
  for (int x = tid; x < L * dv; x += kThreads) dy[x] = ldio(P.dy, (int64_t)n * P.T * dv + x, P.bf);
  for (int x = tid; x < e1 * L; x += kThreads) { wE[x] = 0.f; gacc[x] = 0.f; }
  __syncthreads();
  if (tid < e1) {
    const int j = tid;
    float cs = 0.f, cz = 0.f;
    for (int i = 0; i < L; ++i) {
      cSb[i * e1 + j] = cs;
      cz = cx.be[i] * cz + wgt(P, cx, i, j);
      cs = cx.al[i] * cs - cx.et[i] * cz;
    }
  }
  if (tid == kThreads - 1) adj_scalars(cx, hS, hZS, hZZ);
  if (tid < L) {  // column q of eZ; wE_jb[q] = sum_{i <= jb} W(i, jb) eZ_{i+1}[q]
    const int q = tid;
    float es = 0.f, ez = 0.f;
    for (int i = L - 1; i >= 0; --i) {
      for (int jb = i; jb < e1; ++jb) wE[jb * L + q] += wgt(P, cx, i, jb) * ez;
      const float eta = i >= 1 ? cx.et[i - 1] : 0.f;
      es = cx.al[i] * es + (q == i ? 1.f : 0.f);
      ez = cx.be[i] * ez - eta * es;
    }
  }
  __syncthreads();
  const int64_t D2 = (int64_t)dv * dphi;
  // adjoint at the end of chunk 0 of unit n (bf16 tiles)
  const unsigned char* FSt = P.adjb + (int64_t)n * P.nch * 2 * kTileBytes;
  const unsigned char* FZt = FSt + kTileBytes;
  const float* bufn = P.buf ? P.buf + (int64_t)n * e1 * D2 : nullptr;
  const int64_t cid = (int64_t)n * P.nch;
  if (bufn) {
    for (int jb = 0; jb < e1; ++jb) {
      const float* Bj = bufn + (int64_t)jb * D2;
      float s0 = 0.f, s1 = 0.f;
      for (int64_t x = tid; x < D2; x += kThreads) {
        const int r = (int)(x / dphi), c = (int)(x - (int64_t)r * dphi);
        s0 += bf_at(FSt, r, c) * Bj[x];
        s1 += bf_at(FZt, r, c) * Bj[x];
      }
      s0 = block_sum(s0, red);
      s1 = block_sum(s1, red);
      if (tid == 0) { P.xf[(cid * kR + jb) * 2] = s0; P.xf[(cid * kR + jb) * 2 + 1] = s1; }
    }
    // G[q][jb] = sum_nn dy_q[nn] (Buf_jb psi_q)[nn]
    bgemm(stage, L, e1 * dv,
          [&](int q, int c, float acc) { atomicAdd(&gacc[q * e1 + c / dv], acc * dy[q * dv + c % dv]); },
          seg(dphi, [&](int q, int m) { return psi[q * dphi + m]; },
              [&](int m, int c) { return bufn[(int64_t)c * dphi + m]; }));
    // d psi_i += sum_jb cS_i[jb] Buf_jb^T dy_i
    bgemm(stage, L, dphi,
          [&](int i, int m, float acc) {
            __nv_bfloat16* d = P.dpsib + ((int64_t)n * P.T + i) * dphi + m;
            *d = __float2bfloat16_rn(__bfloat162float(*d) + acc);
          },
          seg(e1 * dv,
              [&](int i, int kk) { return cSb[i * e1 + kk / dv] * dy[i * dv + kk % dv]; },
              [&](int kk, int m) { return bufn[(int64_t)kk * dphi + m]; }));
    __syncthreads();
    unsigned char* gt = reinterpret_cast<unsigned char*>(P.gt) + cid * kTileBytes;
    for (int x = tid; x < L * e1; x += kThreads) {
      const int q = x / e1, jb = x % e1;
      *reinterpret_cast<__nv_bfloat16*>(gt + umma::elem_off(q, jb, kR)) = __float2bfloat16_rn(gacc[x]);
    }
  }
  if (P.dbuf) {
    float* db = P.dbuf + (int64_t)n * e1 * D2;
    for (int jb = 0; jb < e1; ++jb) {
      float wzs = 0.f, wzz = 0.f;
      for (int i = 0; i <= min(L - 1, jb); ++i) {
        const float w = wgt(P, cx, i, jb);
        wzs += w * hZS[i + 1];
        wzz += w * hZZ[i + 1];
      }
      bgemm(stage, dv, dphi,
            [&](int nn, int m, float acc) {
              db[(int64_t)jb * D2 + (int64_t)nn * dphi + m] = acc + wzs * bf_at(FSt, nn, m) + wzz * bf_at(FZt, nn, m);
            },
            seg(L, [&](int nn, int q) { return wE[jb * L + q] * dy[q * dv + nn]; },
                [&](int q, int m) { return psi[q * dphi + m]; }));
    }
  }
}

// ===========================================================================
// per 128-token tile: fold in the halo partials of d delta / d phi / du, then
//   dv = -d delta,  d phi = d phi_window + d delta S_ref (tensor cores),
//   dk = d phi * fmap'(k), dq = d psi * fmap'(q)
// (tensor feature map: d phi is left in the scratch for its own backward).
// ===========================================================================
__global__ void __launch_bounds__(kT) k_bwd_finalize_tc(const __grid_constant__ Params P) {
  PhaseClock pc;
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* tDD = sm;               // d delta rows (bf16)
  unsigned char* tSR = sm + kTileBytes;  // S_ref
  __shared__ uint64_t mbar, lbar;
  __shared__ uint32_t tbase;
  const int n = blockIdx.y, p0 = blockIdx.x * kR, e = P.e, tid = threadIdx.x, row = row_of(), wg = wg_of();
  const int TT = min(kR, P.T - p0);
  TmaBatch ld{&lbar, 0};
  if (tid == 0) {
    tma_init(ld);
    tma_tile(tSR, P.srb + (int64_t)n * kTileBytes, ld.bar);
    tma_commit(ld);
  }
  Sync sy{&mbar, &tbase, 0, P.status};
  const uint32_t tm = tc_setup(sy, 128);
  const int e1 = e > 1 ? e - 1 : 1;
  // halo slot of token p in the next chunk (keys of chunk c+1 start at t0(c+1)-(e-1))
  auto halo = [&](int p) -> int64_t {
    const int c = p / P.C;
    if (e <= 1 || c + 1 >= P.nch) return -1;
    const int hs = (c + 1) * P.C - (e - 1);
    return p >= hs ? ((int64_t)n * P.nch + c + 1) * e1 + (p - hs) : -1;
  };
  fill_tile(tDD, kD, [&](int r, int c0, float(&v)[8]) {
    if (r >= TT) { zero8(v); return; }
    const int p = p0 + r;
    const int64_t gi = ((int64_t)n * P.T + p) * P.dv + c0;
    ld8io(P.ddb, gi, 1, v);
    const int64_t h = halo(p);
    if (h >= 0) {
      float a[8];
      ld8f(P.hdd + h * P.dv + c0, a);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] += a[k];
    }
    // final d delta (fp32, only for the dS_ref reduction) and dv = -d delta  (delta = pred - v, rnn_memory.py:660)
    if (P.dSref) {
      float4* dst = reinterpret_cast<float4*>(P.ddel + gi);
      dst[0] = make_float4(v[0], v[1], v[2], v[3]);
      dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (P.dv_) {
      __align__(16) __nv_bfloat162 hb[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) hb[k] = __floats2bfloat162_rn(-v[2 * k], -v[2 * k + 1]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(P.dv_) + gi) = *reinterpret_cast<uint4*>(hb);
    }
  }, 0, kT, /*rowmajor=*/true);
  pc.mark(56);
  if (tid == 0) tma_wait(ld, P.status);  // S_ref tile, read only by the MMA thread 0 issues
  smem_to_tc();
  if (tid == 0) mma_chain(tm, op(tDD, kD, 0), op(tSR, kD, 1), 8, kD, false);  // d delta S_ref
  // while the MMA runs: dq, and du in token-gate mode
  if (P.fmode != ATLAS_FMAP_TENSOR && P.dq_)
    for (int x = tid; x < TT * (P.dphi / 8); x += kT) {
      const int r = x / (P.dphi / 8), c0 = (x % (P.dphi / 8)) * 8;
      const int64_t gi = ((int64_t)n * P.T + p0 + r) * P.dphi + c0;
      float g[8], q[8];
      ld8io(P.dpsib, gi, 1, g);
      ld8io(P.q, gi, P.bf, q);
      __align__(16) __nv_bfloat162 hb[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        hb[k] = __floats2bfloat162_rn(g[2 * k] * fmap_elem_grad(q[2 * k], P.fmode, P.fdeg),
                                      g[2 * k + 1] * fmap_elem_grad(q[2 * k + 1], P.fmode, P.fdeg));
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(P.dq_) + gi) = *reinterpret_cast<uint4*>(hb);
    }
  if (P.fmode == ATLAS_FMAP_TENSOR && P.dq_)  // the feature-map backward reads d psi as fp32
    for (int x = tid; x < TT * (P.dphi / 8); x += kT) {
      const int r = x / (P.dphi / 8), c0 = (x % (P.dphi / 8)) * 8;
      const int64_t gi = ((int64_t)n * P.T + p0 + r) * P.dphi + c0;
      float g[8];
      ld8io(P.dpsib, gi, 1, g);
      float4* d = reinterpret_cast<float4*>(P.dpsi + gi);
      d[0] = make_float4(g[0], g[1], g[2], g[3]);
      d[1] = make_float4(g[4], g[5], g[6], g[7]);
    }
  if (P.gmode == ATLAS_GATE_TOKEN && P.dgate)
    for (int r = tid; r < TT; r += kT) {
      const int p = p0 + r;
      float d = P.du[(int64_t)n * P.T + p];
      const int64_t h = halo(p);
      if (h >= 0) d += P.hdu[h];
      stio(P.dgate, (int64_t)n * P.T + p, d, P.bf);
    }
  pc.mark(57);
  ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 128);
  pc.mark(58);
  {
    const int r = row, p = p0 + r;
    const int64_t h = r < TT ? halo(p) : -1;
#pragma unroll
    for (int h4 = 0; h4 < kCPW; ++h4) {
      const int c16 = wg * kCPW + h4;
      float a[16];
      umma::tmem_ld16(lane_addr(tm, c16 * 16), a);
      umma::tmem_ld_wait();
      if (r < TT) {
        const int64_t gi = ((int64_t)n * P.T + p) * P.dphi + c16 * 16;
        float w0[8], w1[8];
        ld8io(P.dpb, gi, 1, w0);
        ld8io(P.dpb, gi + 8, 1, w1);
#pragma unroll
        for (int k = 0; k < 8; ++k) { a[k] += w0[k]; a[8 + k] += w1[k]; }
        if (h >= 0) {
          ld8f(P.hdp + h * P.dphi + c16 * 16, w0);
          ld8f(P.hdp + h * P.dphi + c16 * 16 + 8, w1);
#pragma unroll
          for (int k = 0; k < 8; ++k) { a[k] += w0[k]; a[8 + k] += w1[k]; }
        }
        if (P.fmode == ATLAS_FMAP_TENSOR) {
          st16f(P.dphiR + gi, a);
        } else if (P.dk_) {
          float k0[8], k1[8];
          ld8io(P.k, gi, P.bf, k0);
          ld8io(P.k, gi + 8, P.bf, k1);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            a[k] *= fmap_elem_grad(k0[k], P.fmode, P.fdeg);
            a[8 + k] *= fmap_elem_grad(k1[k], P.fmode, P.fdeg);
          }
          st16bf(reinterpret_cast<__nv_bfloat16*>(P.dk_) + gi, a);
        }
      }
    }
  }
  tc_teardown(tm, 128);  pc.mark(59);

}

// ===========================================================================
// dS_ref = sum_t d delta_t phi_t^T  (delta = S_ref phi - v, rnn_memory.py:659):
// a reduction over the tokens of a unit on tensor cores. CTA (segment, unit)
// accumulates its 128-token tiles in TMEM, then adds into dS_ref (zeroed by
// the host) with vector atomics.
// ===========================================================================
__global__ void __launch_bounds__(kT) k_bwd_dsref_tc(Params P, int tiles_per_cta) {
  extern __shared__ __align__(1024) unsigned char sm[];
  unsigned char* tDD = sm;               // d delta rows (bf16), MN-major A: [M = d_v, K = tokens]
  unsigned char* tPh = sm + kTileBytes;  // phi rows,             MN-major B: [N = d_phi, K = tokens]
  __shared__ uint64_t mbar;
  __shared__ uint32_t tbase;
  const int n = blockIdx.y, tid = threadIdx.x, row = row_of(), wg = wg_of();
  const int ntiles = (P.T + kR - 1) / kR;
  const int tb = blockIdx.x * tiles_per_cta, te = min(ntiles, tb + tiles_per_cta);
  Sync sy{&mbar, &tbase, 0, P.status};
  const uint32_t tm = tc_setup(sy, 128);
  for (int t = tb; t < te; ++t) {
    const int p0 = t * kR, TT = min(kR, P.T - p0);
    fill_tile(tDD, kD, [&](int r, int c0, float(&v)[8]) {
      if (r < TT) ld8f(P.ddel + ((int64_t)n * P.T + p0 + r) * P.dv + c0, v);
      else zero8(v);
    });
    fill_tile(tPh, kD, [&](int r, int c0, float(&v)[8]) {
      if (r < TT) phi8(P, n, p0 + r, c0, false, v);
      else zero8(v);
    });
    smem_to_tc();
    if (tid == 0) mma_chain(tm, op(tDD, kD, 1), op(tPh, kD, 1), 8, kD, t > tb);
    ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, 128);  // the tiles are refilled next iteration
  }
  if (te > tb) {
    float* dst = P.dSref + ((int64_t)n * kD + row) * kD;
    for (int h = 0; h < kCPW; ++h) {
      const int c16 = wg * kCPW + h;
      float a[16];
      umma::tmem_ld16(lane_addr(tm, c16 * 16), a);
      umma::tmem_ld_wait();
#pragma unroll
      for (int k = 0; k < 16; k += 4)
        atomicAdd(reinterpret_cast<float4*>(dst + c16 * 16 + k), make_float4(a[k], a[k + 1], a[k + 2], a[k + 3]));
    }
  }
  tc_teardown(tm, 128);
}

}  // namespace tc
}  // namespace atlas
