// Chunk scans of the tensor-core path as one resident wave.
//
// The state recurrence over chunks (S_{c+1} = a_c S_c + b_c Z_c + dS_c,
// Z_{c+1} = c_c Z_c + dZ_c; the adjoint runs the transposed recurrence from the
// last chunk down) is sequential in c and independent per state element. The
// generic scans (k_fwd_scan / k_bwd_scan) give every thread one float4 of one
// unit's state and need several waves of CTAs for N = 128 units, each wave
// running the whole chain. Here one CTA of kScanThreads runs per SM and every
// thread keeps F groups of 8 state elements (one 16-byte bf16 unit of the
// increments and of the state tiles) in registers: group s of thread t is
// global group base + s * G, G = all threads of the grid. F (1, 2 or 4) is the
// smallest that covers the units in one round; the ring of kScanSlots / F
// chunks (192 KB of shared memory either way) keeps that many chunks' increments
// in flight through cp.async, each thread reading back only its own entries, so
// a step waits for nothing but its own chunk and few units (F = 1) still keep
// enough bytes in flight per SM. For more than 4 groups per thread the host
// launches several rounds. A CTA has up to kScanThreads threads: the host sizes
// it so the groups spread over every SM. Group indices are 32-bit (N * 2048 < 2^31, checked
// by the host).
#pragma once
#include "tc_common.cuh"

namespace atlas {
namespace tc {

constexpr int kScanThreads = 512;
constexpr int kScanSlots = 12;                   // (groups per thread) x (chunks in the ring)
constexpr int kOct = kD * kD / 8;                // 8-element groups per 128 x 128 state (2048)
constexpr int kScanRingBytes = kScanSlots * 2 * kScanThreads * 16;  // 192 KB
// F groups of 8 elements per thread and round (1, 2 or 4), kScanSlots / F chunks in flight.
template <int F>
struct ScanGeom {
  static constexpr int kDepth = kScanSlots / F;
  // chunk scalars loaded this many steps before use (registers: 4 F kAhead per thread)
  static constexpr int kAhead = F == 1 ? 8 : (F == 2 ? 4 : 1);
};

__device__ __forceinline__ void unpack8(uint4 u, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  __align__(16) __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return *reinterpret_cast<uint4*>(h);
}
// Byte offset of group xo (elements 8 xo .. 8 xo + 7, one row) in a core-matrix tile.
__device__ __forceinline__ uint32_t oct_off(int xo) {
  const int r = xo >> 4, cb = xo & 15;
  return (uint32_t)(((r >> 3) * 16 + cb) * 128 + (r & 7) * 16);
}
__device__ __forceinline__ void ld8f4(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void st8f4(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void scan_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

// The two 16-byte increment units (dS, dZ) of the F groups at chunk c into ring slot d.
template <int F>
__device__ __forceinline__ void scan_issue(unsigned char* ring, const __nv_bfloat16* inc, int nch, int c, int d,
                                           int base, int G, int total) {
#pragma unroll
  for (int s = 0; s < F; ++s) {
    const int g = base + s * G;
    const int n = g >> 11, xo = g & (kOct - 1);
    const __nv_bfloat16* src = inc + (((int64_t)n * nch + c) * 2) * (kD * kD) + xo * 8;
    unsigned char* dst = ring + (((d * F + s) * 2) * kScanThreads + threadIdx.x) * 16;
    const bool ok = g < total;
    cp16(dst, ok ? static_cast<const void*>(src) : static_cast<const void*>(inc), ok);
    cp16(dst + kScanThreads * 16, ok ? static_cast<const void*>(src + kD * kD) : static_cast<const void*>(inc), ok);
  }
  scan_commit();
}
template <int PENDING>
__device__ __forceinline__ void scan_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(PENDING) : "memory");
}
template <int F>
__device__ __forceinline__ void scan_take(const unsigned char* ring, int d, int s, float (&dS)[8], float (&dZ)[8]) {
  const unsigned char* p = ring + (((d * F + s) * 2) * kScanThreads + threadIdx.x) * 16;
  unpack8(*reinterpret_cast<const uint4*>(p), dS);
  unpack8(*reinterpret_cast<const uint4*>(p + kScanThreads * 16), dZ);
}
// Forward: S, Z from S0 / Z0 through every chunk; writes the bf16 chunk-start
// tiles (P.stb), then S_T, the clamped S_end and Z_end. Same recurrence as
// k_fwd_scan<4> on the tensor-core path. dry = 1: start from zero, write no
// tiles, emit the segment transform (seg_dS, seg_dZ and the composed scalars
// seg_coef, accumulated by the thread that holds group 0 of the unit).
template <int F>
__global__ void __launch_bounds__(kScanThreads, 1) k_fwd_scan_tc(Params P, int round, int dry) {
  constexpr int kDepth = ScanGeom<F>::kDepth, kAhead = ScanGeom<F>::kAhead;
  extern __shared__ __align__(16) unsigned char ring[];
  const int nch = P.nch;
  const int total = P.N * kOct, G = gridDim.x * blockDim.x;
  const int base = round * F * G + blockIdx.x * blockDim.x + threadIdx.x;
  const __nv_bfloat16* inc = reinterpret_cast<const __nv_bfloat16*>(P.st);
  const float4* cs4 = reinterpret_cast<const float4*>(P.cs);
  for (int c = 0; c < kDepth - 1; ++c) {
    if (c < nch) scan_issue<F>(ring, inc, nch, c, c, base, G, total);
    else scan_commit();
  }
  float S[F][8], Z[F][8];
  float cA[F], cB[F], cC[F];  // composed chunk scalars (dry; used where group s is group 0 of a unit)
#pragma unroll
  for (int s = 0; s < F; ++s) {
    const int g = base + s * G;
#pragma unroll
    for (int i = 0; i < 8; ++i) S[s][i] = Z[s][i] = 0.f;
    cA[s] = 1.f; cB[s] = 0.f; cC[s] = 1.f;
    if (g < total && !dry) {
      ld8f4(P.S0 + (int64_t)g * 8, S[s]);
      if (P.Z0) ld8f4(P.Z0 + (int64_t)g * 8, Z[s]);
    }
  }
  // the scalars of chunk c sit in kq[.][c % kAhead], loaded kAhead steps earlier; the step
  // loop is unrolled by kAhead so that slot is a fixed register
  float4 kq[F][kAhead];
  auto kld = [&](int s, int c) {
    const int g = base + s * G;
    return (g < total && c < nch) ? cs4[(int64_t)(g >> 11) * nch + c] : make_float4(0.f, 0.f, 0.f, 0.f);
  };
#pragma unroll
  for (int s = 0; s < F; ++s)
#pragma unroll
    for (int j = 0; j < kAhead; ++j) kq[s][j] = kld(s, j);
  for (int c0 = 0; c0 < nch; c0 += kAhead) {
#pragma unroll
    for (int j = 0; j < kAhead; ++j) {
      const int c = c0 + j;
      if (c >= nch) break;
      const int cn = c + kDepth - 1;
      if (cn < nch) scan_issue<F>(ring, inc, nch, cn, cn % kDepth, base, G, total);
      else scan_commit();
      float4 kc[F];
#pragma unroll
      for (int s = 0; s < F; ++s) {
        kc[s] = kq[s][j];
        kq[s][j] = kld(s, c + kAhead);
      }
      scan_wait<kDepth - 1>();
      const int d = c % kDepth;
#pragma unroll
      for (int s = 0; s < F; ++s) {
        const int g = base + s * G;
        if (g < total) {
          const int n = g >> 11, xo = g & (kOct - 1);
          if (!dry) {
            unsigned char* t = P.stb + ((int64_t)n * nch + c) * 2 * kTileBytes + oct_off(xo);
            *reinterpret_cast<uint4*>(t) = pack8(S[s]);
            *reinterpret_cast<uint4*>(t + kTileBytes) = pack8(Z[s]);
          }
          const float4 k = kc[s];
          if (dry && xo == 0) {
            cB[s] = k.x * cB[s] + k.y * cC[s];
            cA[s] *= k.x;
            cC[s] *= k.z;
          }
          float dS[8], dZ[8];
          scan_take<F>(ring, d, s, dS, dZ);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float nS = k.x * S[s][i] + k.y * Z[s][i] + dS[i];
            Z[s][i] = k.z * Z[s][i] + dZ[i];
            S[s][i] = nS;
          }
        }
      }
    }
  }
#pragma unroll
  for (int s = 0; s < F; ++s) {
    const int g = base + s * G;
    if (g >= total) continue;
    if (dry) {
      st8f4(P.seg_dS + (int64_t)g * 8, S[s]);
      st8f4(P.seg_dZ + (int64_t)g * 8, Z[s]);
      if ((g & (kOct - 1)) == 0) {
        const int n = g >> 11;
        P.seg_coef[n * 3 + 0] = cA[s]; P.seg_coef[n * 3 + 1] = cB[s]; P.seg_coef[n * 3 + 2] = cC[s];
      }
    } else {
      float cl[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) cl[i] = fminf(fmaxf(S[s][i], -100.f), 100.f);  // rnn_memory.py:701
      st8f4(P.ST + (int64_t)g * 8, S[s]);
      st8f4(P.S_end + (int64_t)g * 8, cl);
      if (P.Z_end) st8f4(P.Z_end + (int64_t)g * 8, Z[s]);  // rnn_memory.py:702
    }
  }
}

// Backward: the adjoint (F_S, F_Z) from dS_end (masked where the forward clamp
// saturated) and dZ_end down through every chunk; writes the bf16 adjoint tiles
// (P.adjb) at each chunk end, then dS0 / dZ0. Same recurrence as k_bwd_scan<4>
// on the tensor-core path. dry = 1: from a zero adjoint, no tiles, segment
// transform out (as the forward).
template <int F>
__global__ void __launch_bounds__(kScanThreads, 1) k_bwd_scan_tc(Params P, int round, int dry) {
  constexpr int kDepth = ScanGeom<F>::kDepth, kAhead = ScanGeom<F>::kAhead;
  extern __shared__ __align__(16) unsigned char ring[];
  const int nch = P.nch;
  const int total = P.N * kOct, G = gridDim.x * blockDim.x;
  const int base = round * F * G + blockIdx.x * blockDim.x + threadIdx.x;
  const __nv_bfloat16* inc = reinterpret_cast<const __nv_bfloat16*>(P.adj);
  const float4* cs4 = reinterpret_cast<const float4*>(P.acs);
  for (int k = 0; k < kDepth - 1; ++k) {
    const int c = nch - 1 - k;
    if (c >= 0) scan_issue<F>(ring, inc, nch, c, k, base, G, total);
    else scan_commit();
  }
  float FS[F][8], FZ[F][8];
  float cA[F], cB[F], cC[F];
#pragma unroll
  for (int s = 0; s < F; ++s) {
    const int g = base + s * G;
#pragma unroll
    for (int i = 0; i < 8; ++i) FS[s][i] = FZ[s][i] = 0.f;
    cA[s] = 1.f; cB[s] = 0.f; cC[s] = 1.f;
    if (g < total && !dry) {
      if (P.dS_end) {
        ld8f4(P.dS_end + (int64_t)g * 8, FS[s]);
        if (P.apply_mask) {  // clamp(-100, 100) passes gradient where -100 <= S_T <= 100
          float t[8];
          ld8f4(P.ST + (int64_t)g * 8, t);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (!(t[i] >= -100.f && t[i] <= 100.f)) FS[s][i] = 0.f;
        }
      }
      if (P.dZ_end) ld8f4(P.dZ_end + (int64_t)g * 8, FZ[s]);
    }
  }
  // the scalars of step k (chunk nch - 1 - k) sit in kq[.][k % kAhead], loaded kAhead steps earlier
  float4 kq[F][kAhead];
  auto kld = [&](int s, int k) {
    const int g = base + s * G;
    return (g < total && k < nch) ? cs4[(int64_t)(g >> 11) * nch + (nch - 1 - k)] : make_float4(0.f, 0.f, 0.f, 0.f);
  };
#pragma unroll
  for (int s = 0; s < F; ++s)
#pragma unroll
    for (int j = 0; j < kAhead; ++j) kq[s][j] = kld(s, j);
  for (int k0 = 0; k0 < nch; k0 += kAhead) {
#pragma unroll
    for (int j = 0; j < kAhead; ++j) {
      const int k = k0 + j;  // step k handles chunk c = nch - 1 - k
      if (k >= nch) break;
      const int c = nch - 1 - k, kn = k + kDepth - 1, cn = nch - 1 - kn;
      if (cn >= 0) scan_issue<F>(ring, inc, nch, cn, kn % kDepth, base, G, total);
      else scan_commit();
      float4 kc[F];
#pragma unroll
      for (int s = 0; s < F; ++s) {
        kc[s] = kq[s][j];
        kq[s][j] = kld(s, k + kAhead);
      }
      scan_wait<kDepth - 1>();
      const int d = k % kDepth;
#pragma unroll
      for (int s = 0; s < F; ++s) {
        const int g = base + s * G;
        if (g < total) {
          const int n = g >> 11, xo = g & (kOct - 1);
          if (!dry) {
            unsigned char* t = P.adjb + ((int64_t)n * nch + c) * 2 * kTileBytes + oct_off(xo);
            *reinterpret_cast<uint4*>(t) = pack8(FS[s]);
            *reinterpret_cast<uint4*>(t + kTileBytes) = pack8(FZ[s]);
          }
          const float4 a = kc[s];
          if (dry && xo == 0) {
            cB[s] = a.y * cA[s] + a.z * cB[s];
            cA[s] *= a.x;
            cC[s] *= a.z;
          }
          float dS[8], dZ[8];
          scan_take<F>(ring, d, s, dS, dZ);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float nFS = a.x * FS[s][i] + dS[i];
            FZ[s][i] = a.y * FS[s][i] + a.z * FZ[s][i] + dZ[i];
            FS[s][i] = nFS;
          }
        }
      }
    }
  }
#pragma unroll
  for (int s = 0; s < F; ++s) {
    const int g = base + s * G;
    if (g >= total) continue;
    if (dry) {
      st8f4(P.seg_dS + (int64_t)g * 8, FS[s]);
      st8f4(P.seg_dZ + (int64_t)g * 8, FZ[s]);
      if ((g & (kOct - 1)) == 0) {
        const int n = g >> 11;
        P.seg_coef[n * 3 + 0] = cA[s]; P.seg_coef[n * 3 + 1] = cB[s]; P.seg_coef[n * 3 + 2] = cC[s];
      }
    } else {
      if (P.dS0) st8f4(P.dS0 + (int64_t)g * 8, FS[s]);
      if (P.dZ0) st8f4(P.dZ0 + (int64_t)g * 8, FZ[s]);
    }
  }
}

}  // namespace tc
}  // namespace atlas
