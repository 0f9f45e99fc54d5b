// Chunked forward / backward kernels of the memory recurrence (fp32 FFMA path).
//
// Within a chunk of L tokens starting at t0 the state is an explicit linear
// combination of the chunk-start state and rank-1 window terms:
//   S_i = sS_i S_in + sZ_i Z_in + sum_j cS_i[j] R_j,   Z_i = zZ_i Z_in + sum_j cZ_i[j] R_j
// with R_j = delta_p phi_p^T for the K = L+e-1 keys p = t0-(e-1)+j (the e-1 halo
// keys before t0 feed the window; in chunk 0 they are the carried omega buffer).
// The scalar coefficients follow the reference recurrences Z_t = beta_t Z_{t-1}+g_t,
// S_t = alpha_t S_{t-1} - eta_t Z_t (rnn_memory.py:697-702) with the window weights
// W(t,p) of rnn_memory.py:666-681. The backward expands the adjoint the same way
// over {F_S, F_Z, dy_q psi_q^T}; every inner product the gate gradients need is an
// entry of the small Gram matrix X between the two bases.
#pragma once
#include "common.cuh"

namespace atlas {

struct Ctx {
  int n, c, t0, L, K, kp0;
  float *al, *et, *be, *u, *U;
};

// Geometry of the chunk (unit n = blockIdx.y, chunk c = blockIdx.x unless given).
__device__ __forceinline__ void ctx_geom(const Params& P, Ctx& cx, int chunk = -1) {
  cx.n = blockIdx.y;
  cx.c = chunk >= 0 ? chunk : blockIdx.x;
  cx.t0 = cx.c * P.C;
  cx.L = min(P.C, P.T - cx.t0);
  cx.K = cx.L + P.e - 1;
  cx.kp0 = cx.t0 - (P.e - 1);
}
// Geometry of chunk c of unit n (persistent kernels that walk several chunks).
__device__ __forceinline__ void ctx_at(const Params& P, Ctx& cx, int n, int c) {
  cx.n = n;
  cx.c = c;
  cx.t0 = c * P.C;
  cx.L = min(P.C, P.T - cx.t0);
  cx.K = cx.L + P.e - 1;
  cx.kp0 = cx.t0 - (P.e - 1);
}
__device__ __forceinline__ void load_ctx_gates(const Params& P, SmemAlloc& sa, Ctx& cx, int nthreads);
__device__ __forceinline__ void load_ctx(const Params& P, SmemAlloc& sa, Ctx& cx, int nthreads = kThreads,
                                         int chunk = -1) {
  ctx_geom(P, cx, chunk);
  load_ctx_gates(P, sa, cx, nthreads);
}
// The gates of the chunk cx already describes (ctx_geom / ctx_at) into shared memory.
__device__ __forceinline__ void load_ctx_gates(const Params& P, SmemAlloc& sa, Ctx& cx, int nthreads) {
  cx.al = sa.take(P.C);
  cx.et = sa.take(P.C);
  cx.be = sa.take(P.C);
  cx.u = sa.take(P.C + P.e);
  cx.U = sa.take(P.C * P.e);
  const int64_t row0 = (int64_t)cx.n * P.T + cx.t0;
  for (int i = threadIdx.x; i < cx.L; i += nthreads) {
    cx.al[i] = ldio(P.decay, row0 + i, P.bf);                   // alpha  (to_decay)
    cx.et[i] = ldio(P.lr, row0 + i, P.bf);                      // eta    (to_lr)
    cx.be[i] = P.mom ? ldio(P.beta, row0 + i, P.bf) : 0.f;      // beta   (to_momentum)
  }
  if (P.gmode == ATLAS_GATE_TOKEN)
    for (int j = threadIdx.x; j < cx.K; j += nthreads) {
      const int p = cx.kp0 + j;
      cx.u[j] = p >= 0 ? ldio(P.gate, (int64_t)cx.n * P.T + p, P.bf) : 1.f;
    }
  if (P.gmode == ATLAS_GATE_WINDOW)
    for (int x = threadIdx.x; x < cx.L * P.e; x += nthreads)
      cx.U[x] = ldio(P.gate, row0 * P.e + x, P.bf);
}

// Gates of one chunk held in registers by each of `nthreads` (>= 128) threads,
// loaded one chunk ahead in the persistent kernels so the global loads overlap
// the current chunk's work; gates_to_smem() then lays them out as load_ctx_gates does.
struct GatePre {
  float al, et, be, u, U[4];
};
__device__ __forceinline__ void gates_fetch(const Params& P, int n, int c, GatePre& g, int nthreads) {
  Ctx cx;
  ctx_at(P, cx, n, c);
  const int i = threadIdx.x;
  const int64_t row0 = (int64_t)n * P.T + cx.t0;
  g.al = g.et = g.be = 0.f;
  g.u = 1.f;
  if (i < cx.L) {
    g.al = ldio(P.decay, row0 + i, P.bf);
    g.et = ldio(P.lr, row0 + i, P.bf);
    g.be = P.mom ? ldio(P.beta, row0 + i, P.bf) : 0.f;
  }
  if (P.gmode == ATLAS_GATE_TOKEN && i < cx.K && cx.kp0 + i >= 0) g.u = ldio(P.gate, (int64_t)n * P.T + cx.kp0 + i, P.bf);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int x = i + k * nthreads;
    g.U[k] = (P.gmode == ATLAS_GATE_WINDOW && x < cx.L * P.e) ? ldio(P.gate, row0 * P.e + x, P.bf) : 0.f;
  }
}
__device__ __forceinline__ void gates_to_smem(const Params& P, SmemAlloc& sa, Ctx& cx, const GatePre& g,
                                              int nthreads) {
  cx.al = sa.take(P.C);
  cx.et = sa.take(P.C);
  cx.be = sa.take(P.C);
  cx.u = sa.take(P.C + P.e);
  cx.U = sa.take(P.C * P.e);
  const int i = threadIdx.x;
  if (i < cx.L) { cx.al[i] = g.al; cx.et[i] = g.et; cx.be[i] = g.be; }
  if (P.gmode == ATLAS_GATE_TOKEN && i < cx.K) cx.u[i] = g.u;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int x = i + k * nthreads;
    if (P.gmode == ATLAS_GATE_WINDOW && x < cx.L * P.e) cx.U[x] = g.U[k];
  }
}

// Weight of key j in g of local token i (0 outside the window). TOKEN mode: the
// per-token gate u_p (buffer entries are stored already gated, weight 1).
__device__ __forceinline__ float wgt(const Params& P, const Ctx& cx, int i, int j) {
  const int jj = i - j + P.e - 1;  // t - p
  if (jj < 0 || jj >= P.e) return 0.f;
  if (P.gmode == ATLAS_GATE_NONE) return 1.f;
  if (P.gmode == ATLAS_GATE_TOKEN) return cx.u[j];
  return cx.U[i * P.e + jj];
}

// Forward coefficients, rows r = 0..L (state after r tokens of the chunk).
__device__ __forceinline__ void fwd_coefs(const Params& P, const Ctx& cx, float* cS, float* cZ,
                                          float* sS, float* sZ, float* zZ) {
  const int j = threadIdx.x, K = cx.K;
  if (j < K) {
    float cs = 0.f, cz = 0.f;
    cS[j] = 0.f;
    cZ[j] = 0.f;
    for (int i = 0; i < cx.L; ++i) {
      cz = cx.be[i] * cz + wgt(P, cx, i, j);
      cs = cx.al[i] * cs - cx.et[i] * cz;
      cS[(i + 1) * K + j] = cs;
      cZ[(i + 1) * K + j] = cz;
    }
  } else if (j == K) {
    float s = 1.f, sz = 0.f, z = 1.f;
    sS[0] = s; sZ[0] = sz; zZ[0] = z;
    for (int i = 0; i < cx.L; ++i) {
      z = cx.be[i] * z;
      s = cx.al[i] * s;
      sz = cx.al[i] * sz - cx.et[i] * z;
      sS[i + 1] = s; sZ[i + 1] = sz; zZ[i + 1] = z;
    }
  }
}

// Adjoint coefficients, rows r = 0..L: the adjoint of the state after r tokens
// (r = L chunk end, r = 0 chunk input) as
//   Shat_r = hS_r F_S + sum_q eS_r[q] D_q,  Zhat_r = hZS_r F_S + hZZ_r F_Z + sum_q eZ_r[q] D_q
// with D_q = dy_q psi_q^T. Threads [tb, tb+L] do the work.
__device__ __forceinline__ void adj_coefs(const Params& P, const Ctx& cx, int tb, float* hS,
                                          float* hZS, float* hZZ, float* eS, float* eZ) {
  const int q = (int)threadIdx.x - tb, L = cx.L;
  if (q >= 0 && q < L) {
    float es = 0.f, ez = 0.f;
    eS[L * L + q] = 0.f;
    eZ[L * L + q] = 0.f;
    for (int r = L - 1; r >= 0; --r) {
      const float eta = r >= 1 ? cx.et[r - 1] : 0.f;
      es = cx.al[r] * es + (q == r ? 1.f : 0.f);
      ez = cx.be[r] * ez - eta * es;
      eS[r * L + q] = es;
      eZ[r * L + q] = ez;
    }
  } else if (q == L) {
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
}

// Key rows of phi (zero for p < 0) and of v or the saved delta.
__device__ __forceinline__ void load_keys_phi(const Params& P, const Ctx& cx, float* Phi) {
  for (int x = threadIdx.x; x < cx.K * P.dphi; x += kThreads) {
    const int j = x / P.dphi, m = x - j * P.dphi, p = cx.kp0 + j;
    Phi[x] = p >= 0 ? load_phi(P, cx.n, p, m, false) : 0.f;
  }
}
__device__ __forceinline__ void load_keys_delta(const Params& P, const Ctx& cx, float* Dl) {
  for (int x = threadIdx.x; x < cx.K * P.dv; x += kThreads) {
    const int j = x / P.dv, nn = x - j * P.dv, p = cx.kp0 + j;
    Dl[x] = p >= 0 ? P.delta[((int64_t)cx.n * P.T + p) * P.dv + nn] : 0.f;
  }
}
__device__ __forceinline__ void load_rows_psi(const Params& P, const Ctx& cx, float* Psi) {
  for (int x = threadIdx.x; x < cx.L * P.dphi; x += kThreads) {
    const int i = x / P.dphi, m = x - i * P.dphi;
    Psi[x] = load_phi(P, cx.n, cx.t0 + i, m, true);
  }
}
__device__ __forceinline__ void load_rows_dy(const Params& P, const Ctx& cx, float* dY) {
  const int64_t base = ((int64_t)cx.n * P.T + cx.t0) * P.dv;
  for (int x = threadIdx.x; x < cx.L * P.dv; x += kThreads) dY[x] = ldio(P.dy, base + x, P.bf);
}

__device__ __forceinline__ const float* buf_of(const Params& P, int n, int c) {
  return (c == 0 && P.buf) ? P.buf + (int64_t)n * (P.e - 1) * P.dv * P.dphi : nullptr;
}

// ===========================================================================
// F1: per chunk, delta = Phi S_ref^T - V for the keys, and the chunk's state
// increment from a zero chunk-start state (dS, dZ) plus its scalars.
// ===========================================================================
__global__ void __launch_bounds__(kThreads) k_fwd_chunk(Params P) {
  extern __shared__ float smem[];
  SmemAlloc sa{smem, 0};
  Ctx cx;
  load_ctx(P, sa, cx);
  const int K = cx.K, L = cx.L, dphi = P.dphi, dv = P.dv, n = cx.n, c = cx.c;
  float* Phi = sa.take(K * dphi);
  float* Dl = sa.take(K * dv);
  float* cS = sa.take((L + 1) * K);
  float* cZ = sa.take((L + 1) * K);
  float* sS = sa.take(L + 1);
  float* sZ = sa.take(L + 1);
  float* zZ = sa.take(L + 1);
  float* stage = sa.take(kStageFloats);
  load_keys_phi(P, cx, Phi);
  for (int x = threadIdx.x; x < K * dv; x += kThreads) {
    const int j = x / dv, nn = x - j * dv, p = cx.kp0 + j;
    Dl[x] = p >= 0 ? ldio(P.v, ((int64_t)n * P.T + p) * dv + nn, P.bf) : 0.f;
  }
  __syncthreads();
  const float* Sref = P.Sref + (int64_t)n * dv * dphi;
  // delta_p = S_ref phi_p - v_p  (rnn_memory.py:659-660)
  bgemm(stage, K, dv,
        [&](int j, int nn, float acc) {
          const int p = cx.kp0 + j;
          const float d = p >= 0 ? acc - Dl[j * dv + nn] : 0.f;
          Dl[j * dv + nn] = d;
          if (p >= cx.t0) P.delta[((int64_t)n * P.T + p) * dv + nn] = d;
        },
        seg(dphi, [&](int j, int m) { return Phi[j * dphi + m]; },
            [&](int m, int nn) { return Sref[nn * dphi + m]; }));
  fwd_coefs(P, cx, cS, cZ, sS, sZ, zZ);
  __syncthreads();
  const float* cSe = cS + L * K;
  const float* cZe = cZ + L * K;
  float* dst = P.st + ((int64_t)n * P.nch + c) * 2 * dv * dphi;
  const float* bufn = buf_of(P, n, c);
  const int nb = bufn ? P.e - 1 : 0;
  bgemm(stage, dv, dphi,
        [&](int nn, int m, float acc) {
          for (int jb = 0; jb < nb; ++jb) acc += cSe[jb] * bufn[((int64_t)jb * dv + nn) * dphi + m];
          dst[nn * dphi + m] = acc;
        },
        seg(K, [&](int nn, int j) { return Dl[j * dv + nn] * cSe[j]; },
            [&](int j, int m) { return Phi[j * dphi + m]; }));
  bgemm(stage, dv, dphi,
        [&](int nn, int m, float acc) {
          for (int jb = 0; jb < nb; ++jb) acc += cZe[jb] * bufn[((int64_t)jb * dv + nn) * dphi + m];
          dst[(int64_t)dv * dphi + nn * dphi + m] = acc;
        },
        seg(K, [&](int nn, int j) { return Dl[j * dv + nn] * cZe[j]; },
            [&](int j, int m) { return Phi[j * dphi + m]; }));
  if (threadIdx.x == 0) {
    float* s = P.cs + ((int64_t)n * P.nch + c) * 4;
    s[0] = sS[L]; s[1] = sZ[L]; s[2] = zZ[L]; s[3] = 0.f;
  }
}

// ===========================================================================
// F2: sequential scan over chunks. Each thread owns VEC consecutive state
// elements of one unit and walks the chunks with the increments of the next
// two chunks already in flight. Turns the chunk increments into chunk-start
// states in place; writes S_end / Z_end. dry = 1: start from zero, write
// nothing in place, emit the segment transform instead.
// ===========================================================================
template <int VEC>
struct VecT;
template <>
struct VecT<1> { using T = float; };
template <>
struct VecT<4> { using T = float4; };

__device__ __forceinline__ float axpby(float a, float x, float b, float y, float z) { return a * x + b * y + z; }
__device__ __forceinline__ float4 axpby(float a, float4 x, float b, float4 y, float4 z) {
  return make_float4(a * x.x + b * y.x + z.x, a * x.y + b * y.y + z.y, a * x.z + b * y.z + z.z,
                     a * x.w + b * y.w + z.w);
}
__device__ __forceinline__ float vzero(float) { return 0.f; }
__device__ __forceinline__ float4 vzero(float4) { return make_float4(0.f, 0.f, 0.f, 0.f); }

// Loads the per-chunk scalars of unit n into shared memory (nch float4).
__device__ __forceinline__ const float4* stage_chunk_scalars(const float* src, int n, int nch, float4* dst) {
  const float4* s4 = reinterpret_cast<const float4*>(src) + (int64_t)n * nch;
  for (int c = threadIdx.x; c < nch; c += kThreads) dst[c] = s4[c];
  __syncthreads();
  return dst;
}

// Writes 4 consecutive state elements (element offset e0 of a 128x128 state)
// as bf16 into the core-matrix tile layout used by the tensor-core kernels.
__device__ __forceinline__ void st4_tile(unsigned char* tile, int64_t e0, float4 v) {
  const int r = (int)(e0 >> 7), c = (int)(e0 & 127);
  const uint32_t off = (uint32_t)(((r >> 3) * 16 + (c >> 3)) * 128 + (r & 7) * 16 + (c & 7) * 2);
  __align__(8) __nv_bfloat162 h[2] = {__floats2bfloat162_rn(v.x, v.y), __floats2bfloat162_rn(v.z, v.w)};
  *reinterpret_cast<uint2*>(tile + off) = *reinterpret_cast<uint2*>(h);
}
__device__ __forceinline__ void st4_tile(unsigned char*, int64_t, float) {}

// Chunk increment i (in units of V) of a unit: fp32, or bf16 on the tensor-core path.
template <class V>
__device__ __forceinline__ V ld_inc(const V* f32, const __nv_bfloat16* b16, int64_t i);
template <>
__device__ __forceinline__ float ld_inc<float>(const float* f32, const __nv_bfloat16*, int64_t i) { return f32[i]; }
template <>
__device__ __forceinline__ float4 ld_inc<float4>(const float4* f32, const __nv_bfloat16* b16, int64_t i) {
  if (!b16) return f32[i];
  const uint2 u = *reinterpret_cast<const uint2*>(b16 + i * 4);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <int VEC>
__global__ void __launch_bounds__(kThreads) k_fwd_scan(Params P, int dry) {
  using V = typename VecT<VEC>::T;
  extern __shared__ float4 scs[];
  const int n = blockIdx.y, nch = P.nch;
  const int64_t D2 = (int64_t)P.dv * P.dphi, DV = D2 / VEC;
  const int64_t x = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const float4* cs = stage_chunk_scalars(P.cs, n, nch, scs);
  if (dry && blockIdx.x == 0 && threadIdx.x == 0) {
    float A = 1.f, B = 0.f, Cc = 1.f;
    for (int c = 0; c < nch; ++c) {
      B = cs[c].x * B + cs[c].y * Cc;
      A = cs[c].x * A;
      Cc = cs[c].z * Cc;
    }
    P.seg_coef[n * 3 + 0] = A; P.seg_coef[n * 3 + 1] = B; P.seg_coef[n * 3 + 2] = Cc;
  }
  if (x >= DV) return;
  V* __restrict__ st = reinterpret_cast<V*>(P.st) + (int64_t)n * nch * 2 * DV;
  const __nv_bfloat16* sb =
      P.inc_bf16 ? reinterpret_cast<const __nv_bfloat16*>(P.st) + (int64_t)n * nch * 2 * D2 : nullptr;
  auto ld = [&](int64_t i) { return ld_inc<V>(st, sb, i); };
  V S = dry ? vzero(V()) : reinterpret_cast<const V*>(P.S0)[n * DV + x];
  V Z = (dry || !P.Z0) ? vzero(V()) : reinterpret_cast<const V*>(P.Z0)[n * DV + x];
  V dS0 = ld(x), dZ0 = ld(DV + x);
  V dS1 = nch > 1 ? ld(2 * DV + x) : dS0, dZ1 = nch > 1 ? ld(3 * DV + x) : dZ0;
  for (int c = 0; c < nch; ++c) {
    V dS2 = dS1, dZ2 = dZ1;
    if (c + 2 < nch) { dS2 = ld((int64_t)(c + 2) * 2 * DV + x); dZ2 = ld((int64_t)(c + 2) * 2 * DV + DV + x); }
    if (!dry) {
      if (P.stb) {  // tensor-core path: bf16 tiles, the fp32 increments stay as they are
        unsigned char* t = P.stb + ((int64_t)n * nch + c) * 2 * 32768;
        st4_tile(t, x * VEC, S);
        st4_tile(t + 32768, x * VEC, Z);
      } else {
        st[(int64_t)c * 2 * DV + x] = S;
        st[(int64_t)c * 2 * DV + DV + x] = Z;
      }
    }
    const float4 k = cs[c];
    const V nS = axpby(k.x, S, k.y, Z, dS0);
    Z = axpby(k.z, Z, 0.f, Z, dZ0);
    S = nS;
    dS0 = dS1; dZ0 = dZ1; dS1 = dS2; dZ1 = dZ2;
  }
  const float* Sf = reinterpret_cast<const float*>(&S);
  const float* Zf = reinterpret_cast<const float*>(&Z);
  for (int v = 0; v < VEC; ++v) {
    const int64_t e = n * D2 + x * VEC + v;
    if (dry) {
      P.seg_dS[e] = Sf[v];
      P.seg_dZ[e] = Zf[v];
    } else {
      P.ST[e] = Sf[v];
      P.S_end[e] = fminf(fmaxf(Sf[v], -100.f), 100.f);  // rnn_memory.py:701
      if (P.Z_end) P.Z_end[e] = Zf[v];                  // rnn_memory.py:702
    }
  }
}

// ===========================================================================
// F3: outputs y_i = S_{i-1} psi_i (rnn_memory.py:712-717) from the chunk-start
// states and the intra-chunk terms.
// ===========================================================================
__global__ void __launch_bounds__(kThreads) k_fwd_out(Params P) {
  extern __shared__ float smem[];
  SmemAlloc sa{smem, 0};
  Ctx cx;
  load_ctx(P, sa, cx);
  const int K = cx.K, L = cx.L, dphi = P.dphi, dv = P.dv, n = cx.n, c = cx.c;
  float* Phi = sa.take(K * dphi);
  float* Dl = sa.take(K * dv);
  float* Psi = sa.take(L * dphi);
  float* Ms = sa.take(L * K);
  float* cS = sa.take((L + 1) * K);
  float* cZ = sa.take((L + 1) * K);
  float* sS = sa.take(L + 1);
  float* sZ = sa.take(L + 1);
  float* zZ = sa.take(L + 1);
  float* stage = sa.take(kStageFloats);
  load_keys_phi(P, cx, Phi);
  load_keys_delta(P, cx, Dl);
  load_rows_psi(P, cx, Psi);
  __syncthreads();
  fwd_coefs(P, cx, cS, cZ, sS, sZ, zZ);
  __syncthreads();
  // Ms[i][j] = cS_{i-1}[j] (psi_i . phi_j)
  bgemm(stage, L, K, [&](int i, int j, float acc) { Ms[i * K + j] = acc * cS[i * K + j]; },
        seg(dphi, [&](int i, int m) { return Psi[i * dphi + m]; },
            [&](int m, int j) { return Phi[j * dphi + m]; }));
  __syncthreads();
  const int64_t D2 = (int64_t)dv * dphi;
  const float* Sin = P.st + ((int64_t)n * P.nch + c) * 2 * D2;
  const float* Zin = Sin + D2;
  const float* bufn = buf_of(P, n, c);
  const int nbK = bufn ? (P.e - 1) * dphi : 0;
  const int64_t ybase = ((int64_t)n * P.T + cx.t0) * dv;
  bgemm(stage, L, dv, [&](int i, int nn, float acc) { stio(P.y, ybase + (int64_t)i * dv + nn, acc, P.bf); },
        seg(K, [&](int i, int j) { return Ms[i * K + j]; }, [&](int j, int nn) { return Dl[j * dv + nn]; }),
        seg(dphi, [&](int i, int m) { return sS[i] * Psi[i * dphi + m]; },
            [&](int m, int nn) { return Sin[nn * dphi + m]; }),
        seg(P.mom ? dphi : 0, [&](int i, int m) { return sZ[i] * Psi[i * dphi + m]; },
            [&](int m, int nn) { return Zin[nn * dphi + m]; }),
        seg(nbK,
            [&](int i, int kk) {
              const int jb = kk / dphi;
              return cS[i * K + jb] * Psi[i * dphi + (kk - jb * dphi)];
            },
            [&](int kk, int nn) {
              const int jb = kk / dphi;
              return bufn[((int64_t)jb * dv + nn) * dphi + (kk - jb * dphi)];
            }));
}

// New omega buffer: the last e-1 window terms (rnn_memory.py:684), gated in
// TOKEN mode as the reference stores them.
__global__ void __launch_bounds__(kThreads) k_buf_out(Params P) {
  const int m = blockIdx.x, n = blockIdx.y, e = P.e;
  const int p = P.T - (e - 1) + m;
  const int64_t D2 = (int64_t)P.dv * P.dphi;
  float* dst = P.buf_out + ((int64_t)n * (e - 1) + m) * D2;
  if (p < 0) {
    const float* src = P.buf ? P.buf + ((int64_t)n * (e - 1) + p + e - 1) * D2 : nullptr;
    for (int64_t x = threadIdx.x; x < D2; x += kThreads) dst[x] = src ? src[x] : 0.f;
    return;
  }
  const float w = P.gmode == ATLAS_GATE_TOKEN ? ldio(P.gate, (int64_t)n * P.T + p, P.bf) : 1.f;
  const int64_t drow = (int64_t)n * P.T + p;
  for (int64_t x = threadIdx.x; x < D2; x += kThreads) {
    const int nn = (int)(x / P.dphi), mm = (int)(x - (int64_t)nn * P.dphi);
    dst[x] = (delta_at(P, drow, nn) * load_phi(P, n, p, mm, false)) * w;
  }
}

// ===========================================================================
// B1: per chunk, the adjoint increment at the chunk input from the chunk's own
// dy (zero adjoint at the chunk end) and the adjoint transform scalars.
// ===========================================================================
__global__ void __launch_bounds__(kThreads) k_bwd_chunk(Params P) {
  extern __shared__ float smem[];
  SmemAlloc sa{smem, 0};
  Ctx cx;
  load_ctx(P, sa, cx);
  const int L = cx.L, dphi = P.dphi, dv = P.dv, n = cx.n, c = cx.c;
  float* Psi = sa.take(L * dphi);
  float* dY = sa.take(L * dv);
  float* hS = sa.take(L + 1);
  float* hZS = sa.take(L + 1);
  float* hZZ = sa.take(L + 1);
  float* eS = sa.take((L + 1) * L);
  float* eZ = sa.take((L + 1) * L);
  float* stage = sa.take(kStageFloats);
  load_rows_psi(P, cx, Psi);
  load_rows_dy(P, cx, dY);
  __syncthreads();
  adj_coefs(P, cx, 0, hS, hZS, hZZ, eS, eZ);
  __syncthreads();
  const int64_t D2 = (int64_t)dv * dphi;
  float* dst = P.adj + ((int64_t)n * P.nch + c) * 2 * D2;
  bgemm(stage, dv, dphi, [&](int nn, int m, float acc) { dst[nn * dphi + m] = acc; },
        seg(L, [&](int nn, int q) { return eS[q] * dY[q * dv + nn]; },
            [&](int q, int m) { return Psi[q * dphi + m]; }));
  bgemm(stage, dv, dphi, [&](int nn, int m, float acc) { dst[D2 + nn * dphi + m] = acc; },
        seg(L, [&](int nn, int q) { return eZ[q] * dY[q * dv + nn]; },
            [&](int q, int m) { return Psi[q * dphi + m]; }));
  if (threadIdx.x == 0) {
    float* s = P.acs + ((int64_t)n * P.nch + c) * 4;
    s[0] = hS[0]; s[1] = hZS[0]; s[2] = hZZ[0]; s[3] = 0.f;
  }
}

// ===========================================================================
// B2: reverse scan over chunks (same access scheme as F2): the adjoint
// arriving at each chunk end (in place), and the gradients of the carried
// S0 / Z0. dry = 1: segment transform from a zero adjoint.
// ===========================================================================
template <int VEC>
__global__ void __launch_bounds__(kThreads) k_bwd_scan(Params P, int dry) {
  using V = typename VecT<VEC>::T;
  extern __shared__ float4 scs[];
  const int n = blockIdx.y, nch = P.nch;
  const int64_t D2 = (int64_t)P.dv * P.dphi, DV = D2 / VEC;
  const int64_t x = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const float4* cs = stage_chunk_scalars(P.acs, n, nch, scs);
  if (dry && blockIdx.x == 0 && threadIdx.x == 0) {
    float A = 1.f, B = 0.f, Cc = 1.f;
    for (int c = nch - 1; c >= 0; --c) {
      B = cs[c].y * A + cs[c].z * B;
      A = cs[c].x * A;
      Cc = cs[c].z * Cc;
    }
    P.seg_coef[n * 3 + 0] = A; P.seg_coef[n * 3 + 1] = B; P.seg_coef[n * 3 + 2] = Cc;
  }
  if (x >= DV) return;
  V FS = vzero(V()), FZ = vzero(V());
  if (!dry) {
    float* fs = reinterpret_cast<float*>(&FS);
    float* fz = reinterpret_cast<float*>(&FZ);
    for (int v = 0; v < VEC; ++v) {
      const int64_t e = n * D2 + x * VEC + v;
      if (P.dS_end) {
        fs[v] = P.dS_end[e];
        if (P.apply_mask) {  // clamp(-100, 100) passes gradient where -100 <= S_T <= 100
          const float s = P.ST[e];
          if (!(s >= -100.f && s <= 100.f)) fs[v] = 0.f;
        }
      }
      if (P.dZ_end) fz[v] = P.dZ_end[e];
    }
  }
  V* __restrict__ st = reinterpret_cast<V*>(P.adj) + (int64_t)n * nch * 2 * DV;
  const __nv_bfloat16* sb =
      P.inc_bf16 ? reinterpret_cast<const __nv_bfloat16*>(P.adj) + (int64_t)n * nch * 2 * D2 : nullptr;
  auto ld = [&](int64_t i) { return ld_inc<V>(st, sb, i); };
  const int cl = nch - 1;
  V dS0 = ld((int64_t)cl * 2 * DV + x), dZ0 = ld((int64_t)cl * 2 * DV + DV + x);
  V dS1 = cl > 0 ? ld((int64_t)(cl - 1) * 2 * DV + x) : dS0;
  V dZ1 = cl > 0 ? ld((int64_t)(cl - 1) * 2 * DV + DV + x) : dZ0;
  for (int c = cl; c >= 0; --c) {
    V dS2 = dS1, dZ2 = dZ1;
    if (c - 2 >= 0) { dS2 = ld((int64_t)(c - 2) * 2 * DV + x); dZ2 = ld((int64_t)(c - 2) * 2 * DV + DV + x); }
    if (!dry) {
      if (P.adjb) {
        unsigned char* t = P.adjb + ((int64_t)n * nch + c) * 2 * 32768;
        st4_tile(t, x * VEC, FS);
        st4_tile(t + 32768, x * VEC, FZ);
      } else {
        st[(int64_t)c * 2 * DV + x] = FS;
        st[(int64_t)c * 2 * DV + DV + x] = FZ;
      }
    }
    const float4 k = cs[c];
    const V nFS = axpby(k.x, FS, 0.f, FS, dS0);
    FZ = axpby(k.y, FS, k.z, FZ, dZ0);
    FS = nFS;
    dS0 = dS1; dZ0 = dZ1; dS1 = dS2; dZ1 = dZ2;
  }
  const float* fs = reinterpret_cast<const float*>(&FS);
  const float* fz = reinterpret_cast<const float*>(&FZ);
  for (int v = 0; v < VEC; ++v) {
    const int64_t e = n * D2 + x * VEC + v;
    if (dry) {
      P.seg_dS[e] = fs[v];
      P.seg_dZ[e] = fz[v];
    } else {
      if (P.dS0) P.dS0[e] = fs[v];
      if (P.dZ0) P.dZ0[e] = fz[v];
    }
  }
}

// ===========================================================================
// B3: per chunk, all gradients that live in the chunk: d psi, d delta and
// d phi (through the window terms, own keys plus halo partials), the gate
// gradients d alpha / d eta / d beta, the window-gate gradients, and (chunk 0)
// the gradient of the carried omega buffer.
// ===========================================================================
__global__ void __launch_bounds__(kThreads) k_bwd_grads(Params P) {
  extern __shared__ float smem[];
  SmemAlloc sa{smem, 0};
  Ctx cx;
  load_ctx(P, sa, cx);
  const int K = cx.K, L = cx.L, dphi = P.dphi, dv = P.dv, n = cx.n, c = cx.c, e = P.e;
  const int XK = K + 2;  // columns of X: S_in, Z_in, R_0..R_{K-1}
  float* Phi = sa.take(K * dphi);
  float* Dl = sa.take(K * dv);
  float* dDl = sa.take(K * dv);
  float* Psi = sa.take(L * dphi);
  float* dY = sa.take(L * dv);
  float* A1 = sa.take(L * K);   // dy_q . delta_j
  float* A2 = sa.take(L * K);   // psi_q . phi_j
  float* X = sa.take((L + 2) * XK);
  float* cS = sa.take((L + 1) * K);
  float* cZ = sa.take((L + 1) * K);
  float* sS = sa.take(L + 1);
  float* sZ = sa.take(L + 1);
  float* zZ = sa.take(L + 1);
  float* hS = sa.take(L + 1);
  float* hZS = sa.take(L + 1);
  float* hZZ = sa.take(L + 1);
  float* eS = sa.take((L + 1) * L);
  float* eZ = sa.take((L + 1) * L);
  float* wZS = sa.take(K);
  float* wZZ = sa.take(K);
  float* wE = sa.take(K * L);
  float* dga = sa.take(3 * L);
  float* duj = sa.take(K);
  float* red = sa.take(32);
  float* stage = sa.take(kStageFloats);

  load_keys_phi(P, cx, Phi);
  load_keys_delta(P, cx, Dl);
  load_rows_psi(P, cx, Psi);
  load_rows_dy(P, cx, dY);
  for (int x = threadIdx.x; x < (L + 2) * XK; x += kThreads) X[x] = 0.f;
  for (int x = threadIdx.x; x < 3 * L; x += kThreads) dga[x] = 0.f;
  for (int x = threadIdx.x; x < K; x += kThreads) duj[x] = 0.f;
  __syncthreads();
  fwd_coefs(P, cx, cS, cZ, sS, sZ, zZ);
  adj_coefs(P, cx, 128, hS, hZS, hZZ, eS, eZ);
  __syncthreads();
  // window-summed adjoint coefficients of each key: dR_j = wZS_j F_S + wZZ_j F_Z + sum_q wE_j[q] D_q
  for (int x = threadIdx.x; x < K * L; x += kThreads) {
    const int j = x / L, q = x - j * L;
    float s = 0.f;
    for (int i = max(0, j - e + 1); i <= min(L - 1, j); ++i) s += wgt(P, cx, i, j) * eZ[(i + 1) * L + q];
    wE[x] = s;
  }
  for (int j = threadIdx.x; j < K; j += kThreads) {
    float a = 0.f, b = 0.f;
    for (int i = max(0, j - e + 1); i <= min(L - 1, j); ++i) {
      const float w = wgt(P, cx, i, j);
      a += w * hZS[i + 1];
      b += w * hZZ[i + 1];
    }
    wZS[j] = a;
    wZZ[j] = b;
  }
  bgemm(stage, L, K, [&](int q, int j, float acc) { A1[q * K + j] = acc; },
        seg(dv, [&](int q, int nn) { return dY[q * dv + nn]; }, [&](int nn, int j) { return Dl[j * dv + nn]; }));
  bgemm(stage, L, K, [&](int q, int j, float acc) { A2[q * K + j] = acc; },
        seg(dphi, [&](int q, int m) { return Psi[q * dphi + m]; },
            [&](int m, int j) { return Phi[j * dphi + m]; }));
  __syncthreads();

  const int64_t D2 = (int64_t)dv * dphi;
  const float* Sin = P.st + ((int64_t)n * P.nch + c) * 2 * D2;
  const float* Zin = Sin + D2;
  const float* FS = P.adj + ((int64_t)n * P.nch + c) * 2 * D2;
  const float* FZ = FS + D2;
  const float* bufn = buf_of(P, n, c);
  const int nb = bufn ? e - 1 : 0;

  // ---- Gram matrix X[a][f] = <adjoint basis a, forward basis f>
  for (int x = threadIdx.x; x < L * K; x += kThreads) {
    const int q = x / K, j = x - q * K;
    X[(2 + q) * XK + 2 + j] = A1[x] * A2[x];
  }
  {
    float s00 = 0.f, s01 = 0.f, s10 = 0.f, s11 = 0.f;
    for (int64_t x = threadIdx.x; x < D2; x += kThreads) {
      const float fs = FS[x], fz = FZ[x], si = Sin[x], zi = Zin[x];
      s00 += fs * si; s01 += fs * zi; s10 += fz * si; s11 += fz * zi;
    }
    s00 = block_sum(s00, red); s01 = block_sum(s01, red);
    s10 = block_sum(s10, red); s11 = block_sum(s11, red);
    if (threadIdx.x == 0) { X[0] = s00; X[1] = s01; X[XK] = s10; X[XK + 1] = s11; }
  }
  for (int jb = 0; jb < nb; ++jb) {
    const float* Bj = bufn + (int64_t)jb * D2;
    float s0 = 0.f, s1 = 0.f;
    for (int64_t x = threadIdx.x; x < D2; x += kThreads) { s0 += FS[x] * Bj[x]; s1 += FZ[x] * Bj[x]; }
    s0 = block_sum(s0, red);
    s1 = block_sum(s1, red);
    if (threadIdx.x == 0) { X[2 + jb] = s0; X[XK + 2 + jb] = s1; }
  }
  __syncthreads();
  // X[D_q][S_in], X[D_q][Z_in] = dy_q . (S_in psi_q), dy_q . (Z_in psi_q)
  bgemm(stage, L, 2 * dv,
        [&](int q, int n2, float acc) {
          const int col = n2 < dv ? 0 : 1, nn = n2 < dv ? n2 : n2 - dv;
          atomicAdd(&X[(2 + q) * XK + col], acc * dY[q * dv + nn]);
        },
        seg(dphi, [&](int q, int m) { return Psi[q * dphi + m]; },
            [&](int m, int n2) { return n2 < dv ? Sin[n2 * dphi + m] : Zin[(n2 - dv) * dphi + m]; }));
  // buffer columns: X[D_q][Buf_jb] = dy_q . (Buf_jb psi_q)
  for (int jb = 0; jb < nb; ++jb) {
    const float* Bj = bufn + (int64_t)jb * D2;
    bgemm(stage, L, dv, [&](int q, int nn, float acc) { atomicAdd(&X[(2 + q) * XK + 2 + jb], acc * dY[q * dv + nn]); },
          seg(dphi, [&](int q, int m) { return Psi[q * dphi + m]; }, [&](int m, int nn) { return Bj[nn * dphi + m]; }));
  }
  // P1 = Phi F_S^T: X[F_S][R_j] and the F_S part of d delta_j; then the same with F_Z.
  bgemm(stage, K, dv,
        [&](int j, int nn, float acc) {
          atomicAdd(&X[2 + j], acc * Dl[j * dv + nn]);
          dDl[j * dv + nn] = wZS[j] * acc;
        },
        seg(dphi, [&](int j, int m) { return Phi[j * dphi + m]; }, [&](int m, int nn) { return FS[nn * dphi + m]; }));
  bgemm(stage, K, dv,
        [&](int j, int nn, float acc) {
          atomicAdd(&X[XK + 2 + j], acc * Dl[j * dv + nn]);
          dDl[j * dv + nn] += wZZ[j] * acc;
        },
        seg(dphi, [&](int j, int m) { return Phi[j * dphi + m]; }, [&](int m, int nn) { return FZ[nn * dphi + m]; }));
  __syncthreads();

  // ---- gate gradients: d alpha_i = <Shat_i, S_{i-1}>, d eta_i = -<Shat_i, Z_i>,
  //      d beta_i = <Zhat_i, Z_{i-1}>, each a bilinear form in X.
  auto Sh = [&](int i, int a) { return a == 0 ? hS[i + 1] : (a == 1 ? 0.f : eS[(i + 1) * L + a - 2]); };
  auto Zh = [&](int i, int a) {
    return a == 0 ? hZS[i + 1] : (a == 1 ? hZZ[i + 1] : eZ[(i + 1) * L + a - 2]);
  };
  bgemm(stage, L + 2, L, [&](int a, int i, float acc) { atomicAdd(&dga[i], Sh(i, a) * acc); },
        seg(XK, [&](int a, int f) { return X[a * XK + f]; },
            [&](int f, int i) { return f == 0 ? sS[i] : (f == 1 ? sZ[i] : cS[i * K + f - 2]); }));
  bgemm(stage, L + 2, L, [&](int a, int i, float acc) { atomicAdd(&dga[L + i], -Sh(i, a) * acc); },
        seg(XK, [&](int a, int f) { return X[a * XK + f]; },
            [&](int f, int i) { return f == 0 ? 0.f : (f == 1 ? zZ[i + 1] : cZ[(i + 1) * K + f - 2]); }));
  if (P.mom)
    bgemm(stage, L + 2, L, [&](int a, int i, float acc) { atomicAdd(&dga[2 * L + i], Zh(i, a) * acc); },
          seg(XK, [&](int a, int f) { return X[a * XK + f]; },
              [&](int f, int i) { return f == 0 ? 0.f : (f == 1 ? zZ[i] : cZ[i * K + f - 2]); }));
  // window weights: dW(i, j) = <Zhat_i, R_j>
  if (P.gmode != ATLAS_GATE_NONE)
    bgemm(stage, L, K,
          [&](int i, int j, float acc) {
            const int jj = i - j + e - 1;
            if (jj < 0 || jj >= e) return;
            if (P.gmode == ATLAS_GATE_TOKEN) {
              if (cx.kp0 + j >= 0) atomicAdd(&duj[j], acc);
            } else if (P.dgate) {
              stio(P.dgate, ((int64_t)n * P.T + cx.t0 + i) * e + jj, acc, P.bf);
            }
          },
          seg(L + 2, [&](int i, int a) { return Zh(i, a); }, [&](int a, int j) { return X[a * XK + 2 + j]; }));

  // ---- d delta_j += sum_q wE_j[q] (psi_q . phi_j) dy_q
  bgemm(stage, K, dv, [&](int j, int nn, float acc) { dDl[j * dv + nn] += acc; },
        seg(L, [&](int j, int q) { return wE[j * L + q] * A2[q * K + j]; },
            [&](int q, int nn) { return dY[q * dv + nn]; }));
  // ---- d phi_j (window part) = dR_j^T delta_j
  bgemm(stage, K, dphi,
        [&](int j, int m, float acc) {
          const int p = cx.kp0 + j;
          if (p >= cx.t0) P.dphiR[((int64_t)n * P.T + p) * dphi + m] = acc;
          else if (p >= 0) P.hdp[(((int64_t)n * P.nch + c) * (e - 1) + j) * dphi + m] = acc;
        },
        seg(dv, [&](int j, int nn) { return wZS[j] * Dl[j * dv + nn]; }, [&](int nn, int m) { return FS[nn * dphi + m]; }),
        seg(dv, [&](int j, int nn) { return wZZ[j] * Dl[j * dv + nn]; }, [&](int nn, int m) { return FZ[nn * dphi + m]; }),
        seg(L, [&](int j, int q) { return wE[j * L + q] * A1[q * K + j]; }, [&](int q, int m) { return Psi[q * dphi + m]; }));
  // ---- d psi_i = S_{i-1}^T dy_i
  bgemm(stage, L, dphi,
        [&](int i, int m, float acc) { P.dpsi[((int64_t)n * P.T + cx.t0 + i) * dphi + m] = acc; },
        seg(dv, [&](int i, int nn) { return sS[i] * dY[i * dv + nn]; }, [&](int nn, int m) { return Sin[nn * dphi + m]; }),
        seg(P.mom ? dv : 0, [&](int i, int nn) { return sZ[i] * dY[i * dv + nn]; },
            [&](int nn, int m) { return Zin[nn * dphi + m]; }),
        seg(K, [&](int i, int j) { return cS[i * K + j] * A1[i * K + j]; }, [&](int j, int m) { return Phi[j * dphi + m]; }),
        seg(nb * dv,
            [&](int i, int kk) {
              const int jb = kk / dv;
              return cS[i * K + jb] * dY[i * dv + kk - jb * dv];
            },
            [&](int kk, int m) {
              const int jb = kk / dv;
              return bufn[((int64_t)jb * dv + kk - jb * dv) * dphi + m];
            }));
  // ---- gradient of the carried buffer entries (chunk 0)
  if (c == 0 && P.dbuf && e > 1) {
    float* db = P.dbuf + (int64_t)n * (e - 1) * D2;
    for (int jb = 0; jb < e - 1; ++jb)
      bgemm(stage, dv, dphi,
            [&](int nn, int m, float acc) {
              db[(int64_t)jb * D2 + nn * dphi + m] = acc + wZS[jb] * FS[nn * dphi + m] + wZZ[jb] * FZ[nn * dphi + m];
            },
            seg(L, [&](int nn, int q) { return wE[jb * L + q] * dY[q * dv + nn]; },
                [&](int q, int m) { return Psi[q * dphi + m]; }));
  }
  __syncthreads();
  // ---- write out
  for (int x = threadIdx.x; x < K * dv; x += kThreads) {
    const int j = x / dv, nn = x - j * dv, p = cx.kp0 + j;
    if (p >= cx.t0) P.ddel[((int64_t)n * P.T + p) * dv + nn] = dDl[x];
    else if (p >= 0) P.hdd[(((int64_t)n * P.nch + c) * (e - 1) + j) * dv + nn] = dDl[x];
  }
  if (P.gmode == ATLAS_GATE_TOKEN)
    for (int j = threadIdx.x; j < K; j += kThreads) {
      const int p = cx.kp0 + j;
      if (p >= cx.t0) P.du[(int64_t)n * P.T + p] = duj[j];
      else if (p >= 0) P.hdu[((int64_t)n * P.nch + c) * (e - 1) + j] = duj[j];
    }
  for (int i = threadIdx.x; i < L; i += kThreads) {
    const int64_t r = (int64_t)n * P.T + cx.t0 + i;
    if (P.ddecay) stio(P.ddecay, r, dga[i], P.bf);
    if (P.dlr) stio(P.dlr, r, dga[L + i], P.bf);
    if (P.mom && P.dbeta) stio(P.dbeta, r, dga[2 * L + i], P.bf);
  }
}

// Gradient arriving through the returned omega buffer (rnn_memory.py:684):
// dense [d_v x d_phi] per entry, back into delta, phi, u (or the old buffer).
__global__ void __launch_bounds__(kThreads) k_bwd_bufout(Params P) {
  extern __shared__ float smem[];
  const int mI = blockIdx.x, n = blockIdx.y, e = P.e, dv = P.dv, dphi = P.dphi;
  const int p = P.T - (e - 1) + mI;
  const int64_t D2 = (int64_t)dv * dphi;
  const float* G = P.dbuf_out + ((int64_t)n * (e - 1) + mI) * D2;
  if (p < 0) {
    if (P.dbuf) {
      float* db = P.dbuf + ((int64_t)n * (e - 1) + p + e - 1) * D2;
      for (int64_t x = threadIdx.x; x < D2; x += kThreads) db[x] += G[x];
    }
    return;
  }
  float* ph = smem;          // [dphi]
  float* dl = smem + dphi;   // [dv]
  float* red = dl + dv;      // [32]
  for (int m = threadIdx.x; m < dphi; m += kThreads) ph[m] = load_phi(P, n, p, m, false);
  for (int nn = threadIdx.x; nn < dv; nn += kThreads) dl[nn] = delta_at(P, (int64_t)n * P.T + p, nn);
  __syncthreads();
  const float w = P.gmode == ATLAS_GATE_TOKEN ? ldio(P.gate, (int64_t)n * P.T + p, P.bf) : 1.f;
  for (int nn = threadIdx.x; nn < dv; nn += kThreads) {
    float s = 0.f;
    for (int m = 0; m < dphi; ++m) s += G[nn * dphi + m] * ph[m];
    const int64_t o = ((int64_t)n * P.T + p) * dv + nn;
    if (P.ddb) P.ddb[o] = __float2bfloat16_rn(__bfloat162float(P.ddb[o]) + w * s);  // tensor-core hand-off
    else P.ddel[o] += w * s;
  }
  for (int m = threadIdx.x; m < dphi; m += kThreads) {
    float s = 0.f;
    for (int nn = 0; nn < dv; ++nn) s += G[nn * dphi + m] * dl[nn];
    const int64_t o = ((int64_t)n * P.T + p) * dphi + m;
    if (P.dpb) P.dpb[o] = __float2bfloat16_rn(__bfloat162float(P.dpb[o]) + w * s);
    else P.dphiR[o] += w * s;
  }
  if (P.gmode == ATLAS_GATE_TOKEN) {
    float s = 0.f;
    for (int64_t x = threadIdx.x; x < D2; x += kThreads) {
      const int nn = (int)(x / dphi), m = (int)(x - (int64_t)nn * dphi);
      s += G[x] * dl[nn] * ph[m];
    }
    s = block_sum(s, red);
    if (threadIdx.x == 0) P.du[(int64_t)n * P.T + p] += s;
  }
}

// ===========================================================================
// B4: per token tile, fold in the halo partials and finish the per-token
// gradients: dv = -d delta, d phi = d phi_window + S_ref^T d delta, and the
// feature-map chain rule for dk / dq; u gradients in TOKEN mode.
// ===========================================================================
constexpr int kFinTile = 32;
__global__ void __launch_bounds__(kThreads) k_bwd_finalize(Params P) {
  extern __shared__ float smem[];
  SmemAlloc sa{smem, 0};
  const int n = blockIdx.y, p0 = blockIdx.x * kFinTile, dv = P.dv, dphi = P.dphi, e = P.e;
  const int TT = min(kFinTile, P.T - p0);
  float* dD = sa.take(kFinTile * dv);
  float* stage = sa.take(kStageFloats);
  // halo slot of token p in the next chunk (keys of chunk c+1 start at t0(c+1)-(e-1))
  auto halo = [&](int p) -> int {
    const int c = p / P.C;
    if (c + 1 >= P.nch) return -1;
    const int hs = (c + 1) * P.C - (e - 1);
    return p >= hs ? (c + 1) * (e - 1) + (p - hs) : -1;
  };
  for (int x = threadIdx.x; x < TT * dv; x += kThreads) {
    const int tt = x / dv, nn = x - tt * dv, p = p0 + tt;
    const int64_t gi = ((int64_t)n * P.T + p) * dv + nn;
    float d = P.ddel[gi];
    const int h = e > 1 ? halo(p) : -1;
    if (h >= 0) d += P.hdd[((int64_t)n * P.nch * (e - 1) + h) * dv + nn];
    dD[x] = d;
    P.ddel[gi] = d;
    if (P.dv_) stio(P.dv_, gi, -d, P.bf);  // delta = pred - v  (rnn_memory.py:660)
  }
  if (P.gmode == ATLAS_GATE_TOKEN && P.dgate)
    for (int tt = threadIdx.x; tt < TT; tt += kThreads) {
      const int p = p0 + tt;
      float d = P.du[(int64_t)n * P.T + p];
      const int h = e > 1 ? halo(p) : -1;
      if (h >= 0) d += P.hdu[(int64_t)n * P.nch * (e - 1) + h];
      stio(P.dgate, (int64_t)n * P.T + p, d, P.bf);
    }
  if (P.fmode != ATLAS_FMAP_TENSOR && P.dq_)
    for (int x = threadIdx.x; x < TT * dphi; x += kThreads) {
      const int64_t gi = ((int64_t)n * P.T + p0) * dphi + x;
      const float qv = ldio(P.q, gi, P.bf);
      stio(P.dq_, gi, P.dpsi[gi] * fmap_elem_grad(qv, P.fmode, P.fdeg), P.bf);
    }
  __syncthreads();
  const float* Sref = P.Sref + (int64_t)n * dv * dphi;
  bgemm(stage, TT, dphi,
        [&](int tt, int m, float acc) {
          const int p = p0 + tt;
          const int64_t gi = ((int64_t)n * P.T + p) * dphi + m;
          float g = acc + P.dphiR[gi];
          const int h = e > 1 ? halo(p) : -1;
          if (h >= 0) g += P.hdp[((int64_t)n * P.nch * (e - 1) + h) * dphi + m];
          if (P.fmode == ATLAS_FMAP_TENSOR) P.dphiR[gi] = g;
          else if (P.dk_) stio(P.dk_, gi, g * fmap_elem_grad(ldio(P.k, gi, P.bf), P.fmode, P.fdeg), P.bf);
        },
        seg(dv, [&](int tt, int nn) { return dD[tt * dv + nn]; }, [&](int nn, int m) { return Sref[nn * dphi + m]; }));
}

// B5: dS_ref = sum_t d delta_t phi_t^T  (delta = S_ref phi - v, rnn_memory.py:659)
__global__ void __launch_bounds__(kThreads) k_bwd_dsref(Params P) {
  extern __shared__ float smem[];
  const int n = blockIdx.y, dv = P.dv, dphi = P.dphi;
  const int tilesN = (dphi + 63) / 64;
  const int r0 = (blockIdx.x / tilesN) * 64, c0 = (blockIdx.x % tilesN) * 64;
  const int M = min(64, dv - r0), Nn = min(64, dphi - c0);
  const float* dd = P.ddel + (int64_t)n * P.T * dv;
  bgemm(smem, M, Nn, [&](int a, int b, float acc) { P.dSref[((int64_t)n * dv + r0 + a) * dphi + c0 + b] = acc; },
        seg(P.T, [&](int a, int t) { return dd[(int64_t)t * dv + r0 + a]; },
            [&](int t, int b) { return load_phi(P, n, t, c0 + b, false); }));
}

// ===========================================================================
// Tensor feature map phi(x) = [x ; vec(x x^T)] Proj (rnn_memory.py:125-130),
// without materialising the d + d^2 wide features.
// ===========================================================================
constexpr int kFmTile = 32;
__global__ void __launch_bounds__(kThreads) k_fmap_tensor_fwd(Params P) {
  extern __shared__ float smem[];
  const int n = blockIdx.y, t0 = blockIdx.x * kFmTile, isq = blockIdx.z, dk = P.dk, dphi = P.dphi;
  const int TT = min(kFmTile, P.T - t0);
  float* xs = smem;
  float* stage = smem + ((kFmTile * dk + 3) & ~3);
  const void* src = isq ? P.q : P.k;
  for (int x = threadIdx.x; x < TT * dk; x += kThreads) xs[x] = ldio(src, ((int64_t)n * P.T + t0) * dk + x, P.bf);
  __syncthreads();
  float* dst = (isq ? P.phiq : P.phik) + ((int64_t)n * P.T + t0) * dphi;
  bgemm(stage, TT, dphi, [&](int t, int cc, float acc) { dst[(int64_t)t * dphi + cc] = acc; },
        seg(dk + dk * dk,
            [&](int t, int kk) {
              if (kk < dk) return xs[t * dk + kk];
              const int a = (kk - dk) / dk, b = (kk - dk) - a * dk;
              return xs[t * dk + a] * xs[t * dk + b];
            },
            [&](int kk, int cc) { return P.proj[(int64_t)kk * dphi + cc]; }));
}

__global__ void __launch_bounds__(kThreads) k_fmap_tensor_bwd(Params P) {
  extern __shared__ float smem[];
  const int n = blockIdx.y, t0 = blockIdx.x * kFmTile, isq = blockIdx.z, dk = P.dk, dphi = P.dphi;
  const int TT = min(kFmTile, P.T - t0);
  float* xs = smem;
  float* dx = xs + ((kFmTile * dk + 3) & ~3);
  float* gs = dx + ((kFmTile * dk + 3) & ~3);
  float* stage = gs + ((kFmTile * dphi + 3) & ~3);
  const void* src = isq ? P.q : P.k;
  const float* g = (isq ? P.dpsi : P.dphiR) + ((int64_t)n * P.T + t0) * dphi;
  for (int x = threadIdx.x; x < TT * dk; x += kThreads) {
    xs[x] = ldio(src, ((int64_t)n * P.T + t0) * dk + x, P.bf);
    dx[x] = 0.f;
  }
  for (int x = threadIdx.x; x < TT * dphi; x += kThreads) gs[x] = g[x];
  __syncthreads();
  bgemm(stage, TT, dk + dk * dk,
        [&](int t, int kk, float acc) {
          if (kk < dk) { atomicAdd(&dx[t * dk + kk], acc); return; }
          const int a = (kk - dk) / dk, b = (kk - dk) - a * dk;
          atomicAdd(&dx[t * dk + a], acc * xs[t * dk + b]);
          atomicAdd(&dx[t * dk + b], acc * xs[t * dk + a]);
        },
        seg(dphi, [&](int t, int cc) { return gs[t * dphi + cc]; },
            [&](int cc, int kk) { return P.proj[(int64_t)kk * dphi + cc]; }));
  __syncthreads();
  void* out = isq ? P.dq_ : P.dk_;
  if (out)
    for (int x = threadIdx.x; x < TT * dk; x += kThreads) stio(out, ((int64_t)n * P.T + t0) * dk + x, dx[x], P.bf);
}

}  // namespace atlas
