// Chunk scans of the tensor-core path as one resident wave.
//
// The state recurrence over chunks (S_{c+1} = a_c S_c + b_c Z_c + dS_c,
// Z_{c+1} = c_c Z_c + dZ_c; the adjoint runs the transposed recurrence from the
// last chunk down) is sequential in c and independent per state element. The
// generic scans (k_fwd_scan / k_bwd_scan) give every thread one float4 of one
// unit's state and need several waves of CTAs for N = 128 units, each wave
// running the whole chain. Here one CTA of kScanThreads runs per SM and every
// thread keeps F float4 slots of state in registers (slot s of thread t holds
// global float4 index base + s * G, G = all threads of the grid), with the
// next chunk's bf16 increments loaded while the current chunk is applied. For
// more slots than 4 per thread (128 registers) the host launches several rounds;
// the scan is bandwidth-bound, so two rounds of 4 cost what one round of 8 would.
// Slot indices are 32-bit (N * 4096 < 2^31, checked by the host).
#pragma once
#include "tc_common.cuh"

namespace atlas {
namespace tc {

constexpr int kScanThreads = 512;
constexpr int kDV4 = kD * kD / 4;  // float4 slots per 128 x 128 state (4096)

__device__ __forceinline__ float4 bf4(uint2 u) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// Forward: S, Z from S0 / Z0 through every chunk; writes the bf16 chunk-start
// tiles (P.stb), then S_T, the clamped S_end and Z_end. Same results as
// k_fwd_scan<4> with dry = 0 on the tensor-core path.
template <int F>
__global__ void __launch_bounds__(kScanThreads, 1) k_fwd_scan_tc(Params P, int round) {
  const int nch = P.nch;
  const int total = P.N * kDV4, G = gridDim.x * kScanThreads;
  const int base = round * F * G + blockIdx.x * kScanThreads + threadIdx.x;
  const __nv_bfloat16* inc = reinterpret_cast<const __nv_bfloat16*>(P.st);
  const float4* cs4 = reinterpret_cast<const float4*>(P.cs);
  auto inc_at = [&](int g, int c, int which) -> uint2 {
    const int n = g >> 12, x = g & (kDV4 - 1);
    return *reinterpret_cast<const uint2*>(inc + (((int64_t)n * nch + c) * 2 + which) * (kD * kD) + x * 4);
  };
  float4 S[F], Z[F];
  uint2 iS[F], iZ[F];
#pragma unroll
  for (int s = 0; s < F; ++s) {
    const int g = base + s * G;
    S[s] = Z[s] = make_float4(0.f, 0.f, 0.f, 0.f);
    iS[s] = iZ[s] = make_uint2(0u, 0u);
    if (g < total) {
      S[s] = reinterpret_cast<const float4*>(P.S0)[g];
      if (P.Z0) Z[s] = reinterpret_cast<const float4*>(P.Z0)[g];
      iS[s] = inc_at(g, 0, 0);
      iZ[s] = inc_at(g, 0, 1);
    }
  }
  for (int c = 0; c < nch; ++c) {
    uint2 nS[F], nZ[F];
#pragma unroll
    for (int s = 0; s < F; ++s) {
      const int g = base + s * G;
      nS[s] = iS[s];
      nZ[s] = iZ[s];
      if (g < total && c + 1 < nch) {
        nS[s] = inc_at(g, c + 1, 0);
        nZ[s] = inc_at(g, c + 1, 1);
      }
    }
#pragma unroll
    for (int s = 0; s < F; ++s) {
      const int g = base + s * G;
      if (g < total) {
        const int n = g >> 12, x = g & (kDV4 - 1);
        unsigned char* t = P.stb + ((int64_t)n * nch + c) * 2 * kTileBytes;
        st4_tile(t, x * 4, S[s]);
        st4_tile(t + kTileBytes, x * 4, Z[s]);
        const float4 k = cs4[(int64_t)n * nch + c];
        const float4 dS = bf4(iS[s]), dZ = bf4(iZ[s]);
        const float4 nS4 = axpby(k.x, S[s], k.y, Z[s], dS);
        Z[s] = axpby(k.z, Z[s], 0.f, Z[s], dZ);
        S[s] = nS4;
      }
      iS[s] = nS[s];
      iZ[s] = nZ[s];
    }
  }
#pragma unroll
  for (int s = 0; s < F; ++s) {
    const int g = base + s * G;
    if (g < total) {
      const float4 v = S[s];
      reinterpret_cast<float4*>(P.ST)[g] = v;
      reinterpret_cast<float4*>(P.S_end)[g] =  // rnn_memory.py:701
          make_float4(fminf(fmaxf(v.x, -100.f), 100.f), fminf(fmaxf(v.y, -100.f), 100.f),
                      fminf(fmaxf(v.z, -100.f), 100.f), fminf(fmaxf(v.w, -100.f), 100.f));
      if (P.Z_end) reinterpret_cast<float4*>(P.Z_end)[g] = Z[s];  // rnn_memory.py:702
    }
  }
}

// Backward: the adjoint (F_S, F_Z) from dS_end (masked where the forward clamp
// saturated) and dZ_end down through every chunk; writes the bf16 adjoint tiles
// (P.adjb) at each chunk end, then dS0 / dZ0. Same results as k_bwd_scan<4>
// with dry = 0 on the tensor-core path.
template <int F>
__global__ void __launch_bounds__(kScanThreads, 1) k_bwd_scan_tc(Params P, int round) {
  const int nch = P.nch;
  const int total = P.N * kDV4, G = gridDim.x * kScanThreads;
  const int base = round * F * G + blockIdx.x * kScanThreads + threadIdx.x;
  const __nv_bfloat16* inc = reinterpret_cast<const __nv_bfloat16*>(P.adj);
  const float4* cs4 = reinterpret_cast<const float4*>(P.acs);
  auto inc_at = [&](int g, int c, int which) -> uint2 {
    const int n = g >> 12, x = g & (kDV4 - 1);
    return *reinterpret_cast<const uint2*>(inc + (((int64_t)n * nch + c) * 2 + which) * (kD * kD) + x * 4);
  };
  float4 FS[F], FZ[F];
  uint2 iS[F], iZ[F];
#pragma unroll
  for (int s = 0; s < F; ++s) {
    const int g = base + s * G;
    FS[s] = FZ[s] = make_float4(0.f, 0.f, 0.f, 0.f);
    iS[s] = iZ[s] = make_uint2(0u, 0u);
    if (g < total) {
      if (P.dS_end) {
        float4 v = reinterpret_cast<const float4*>(P.dS_end)[g];
        if (P.apply_mask) {  // clamp(-100, 100) passes gradient where -100 <= S_T <= 100
          const float4 t = reinterpret_cast<const float4*>(P.ST)[g];
          if (!(t.x >= -100.f && t.x <= 100.f)) v.x = 0.f;
          if (!(t.y >= -100.f && t.y <= 100.f)) v.y = 0.f;
          if (!(t.z >= -100.f && t.z <= 100.f)) v.z = 0.f;
          if (!(t.w >= -100.f && t.w <= 100.f)) v.w = 0.f;
        }
        FS[s] = v;
      }
      if (P.dZ_end) FZ[s] = reinterpret_cast<const float4*>(P.dZ_end)[g];
      iS[s] = inc_at(g, nch - 1, 0);
      iZ[s] = inc_at(g, nch - 1, 1);
    }
  }
  for (int c = nch - 1; c >= 0; --c) {
    uint2 nS[F], nZ[F];
#pragma unroll
    for (int s = 0; s < F; ++s) {
      const int g = base + s * G;
      nS[s] = iS[s];
      nZ[s] = iZ[s];
      if (g < total && c >= 1) {
        nS[s] = inc_at(g, c - 1, 0);
        nZ[s] = inc_at(g, c - 1, 1);
      }
    }
#pragma unroll
    for (int s = 0; s < F; ++s) {
      const int g = base + s * G;
      if (g < total) {
        const int n = g >> 12, x = g & (kDV4 - 1);
        unsigned char* t = P.adjb + ((int64_t)n * nch + c) * 2 * kTileBytes;
        st4_tile(t, x * 4, FS[s]);
        st4_tile(t + kTileBytes, x * 4, FZ[s]);
        const float4 k = cs4[(int64_t)n * nch + c];
        const float4 dS = bf4(iS[s]), dZ = bf4(iZ[s]);
        const float4 nFS = axpby(k.x, FS[s], 0.f, FS[s], dS);
        FZ[s] = axpby(k.y, FS[s], k.z, FZ[s], dZ);
        FS[s] = nFS;
      }
      iS[s] = nS[s];
      iZ[s] = nZ[s];
    }
  }
#pragma unroll
  for (int s = 0; s < F; ++s) {
    const int g = base + s * G;
    if (g < total) {
      if (P.dS0) reinterpret_cast<float4*>(P.dS0)[g] = FS[s];
      if (P.dZ0) reinterpret_cast<float4*>(P.dZ0)[g] = FZ[s];
    }
  }
}

}  // namespace tc
}  // namespace atlas
