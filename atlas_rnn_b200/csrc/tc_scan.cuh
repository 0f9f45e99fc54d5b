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
// global group base + s * G, G = all threads of the grid. The increments of
// the next kScanDepth - 1 chunks are in flight in a shared-memory ring
// (cp.async, each thread reads back only its own entries), so a step waits for
// nothing but its own chunk. For more than 4 groups per thread the host
// launches several rounds. Group indices are 32-bit (N * 2048 < 2^31, checked
// by the host).
#pragma once
#include "tc_common.cuh"

namespace atlas {
namespace tc {

constexpr int kScanThreads = 512;
constexpr int kScanF = 4;                        // groups of 8 elements per thread and round
constexpr int kScanDepth = 3;                    // chunks held in the ring
constexpr int kOct = kD * kD / 8;                // 8-element groups per 128 x 128 state (2048)
constexpr int kScanRingBytes = kScanDepth * kScanF * 2 * kScanThreads * 16;  // 192 KB

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

// The two 16-byte increment units (dS, dZ) of group g at chunk c into ring slot d.
__device__ __forceinline__ void scan_issue(unsigned char* ring, const __nv_bfloat16* inc, int nch, int c, int d,
                                           int base, int G, int total) {
#pragma unroll
  for (int s = 0; s < kScanF; ++s) {
    const int g = base + s * G;
    const int n = g >> 11, xo = g & (kOct - 1);
    const __nv_bfloat16* src = inc + (((int64_t)n * nch + c) * 2) * (kD * kD) + xo * 8;
    unsigned char* dst = ring + (((d * kScanF + s) * 2) * kScanThreads + threadIdx.x) * 16;
    const bool ok = g < total;
    cp16(dst, ok ? static_cast<const void*>(src) : static_cast<const void*>(inc), ok);
    cp16(dst + kScanThreads * 16, ok ? static_cast<const void*>(src + kD * kD) : static_cast<const void*>(inc), ok);
  }
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int PENDING>
__device__ __forceinline__ void scan_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(PENDING) : "memory");
}
__device__ __forceinline__ void scan_take(const unsigned char* ring, int d, int s, float (&dS)[8], float (&dZ)[8]) {
  const unsigned char* p = ring + (((d * kScanF + s) * 2) * kScanThreads + threadIdx.x) * 16;
  unpack8(*reinterpret_cast<const uint4*>(p), dS);
  unpack8(*reinterpret_cast<const uint4*>(p + kScanThreads * 16), dZ);
}

// Forward: S, Z from S0 / Z0 through every chunk; writes the bf16 chunk-start
// tiles (P.stb), then S_T, the clamped S_end and Z_end. Same recurrence as
// k_fwd_scan<4> with dry = 0 on the tensor-core path.
__global__ void __launch_bounds__(kScanThreads, 1) k_fwd_scan_tc(Params P, int round) {
  extern __shared__ __align__(16) unsigned char ring[];
  const int nch = P.nch;
  const int total = P.N * kOct, G = gridDim.x * kScanThreads;
  const int base = round * kScanF * G + blockIdx.x * kScanThreads + threadIdx.x;
  const __nv_bfloat16* inc = reinterpret_cast<const __nv_bfloat16*>(P.st);
  const float4* cs4 = reinterpret_cast<const float4*>(P.cs);
  for (int c = 0; c < kScanDepth - 1; ++c) {
    if (c < nch) scan_issue(ring, inc, nch, c, c, base, G, total);
    else asm volatile("cp.async.commit_group;\n" ::: "memory");
  }
  float S[kScanF][8], Z[kScanF][8];
#pragma unroll
  for (int s = 0; s < kScanF; ++s) {
    const int g = base + s * G;
#pragma unroll
    for (int i = 0; i < 8; ++i) S[s][i] = Z[s][i] = 0.f;
    if (g < total) {
      ld8f4(P.S0 + (int64_t)g * 8, S[s]);
      if (P.Z0) ld8f4(P.Z0 + (int64_t)g * 8, Z[s]);
    }
  }
  for (int c = 0; c < nch; ++c) {
    const int cn = c + kScanDepth - 1;
    if (cn < nch) scan_issue(ring, inc, nch, cn, cn % kScanDepth, base, G, total);
    else asm volatile("cp.async.commit_group;\n" ::: "memory");
    scan_wait<kScanDepth - 1>();
    const int d = c % kScanDepth;
#pragma unroll
    for (int s = 0; s < kScanF; ++s) {
      const int g = base + s * G;
      if (g < total) {
        const int n = g >> 11, xo = g & (kOct - 1);
        unsigned char* t = P.stb + ((int64_t)n * nch + c) * 2 * kTileBytes + oct_off(xo);
        *reinterpret_cast<uint4*>(t) = pack8(S[s]);
        *reinterpret_cast<uint4*>(t + kTileBytes) = pack8(Z[s]);
        const float4 k = cs4[(int64_t)n * nch + c];
        float dS[8], dZ[8];
        scan_take(ring, d, s, dS, dZ);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float nS = k.x * S[s][i] + k.y * Z[s][i] + dS[i];
          Z[s][i] = k.z * Z[s][i] + dZ[i];
          S[s][i] = nS;
        }
      }
    }
  }
#pragma unroll
  for (int s = 0; s < kScanF; ++s) {
    const int g = base + s * G;
    if (g < total) {
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
// with dry = 0 on the tensor-core path.
__global__ void __launch_bounds__(kScanThreads, 1) k_bwd_scan_tc(Params P, int round) {
  extern __shared__ __align__(16) unsigned char ring[];
  const int nch = P.nch;
  const int total = P.N * kOct, G = gridDim.x * kScanThreads;
  const int base = round * kScanF * G + blockIdx.x * kScanThreads + threadIdx.x;
  const __nv_bfloat16* inc = reinterpret_cast<const __nv_bfloat16*>(P.adj);
  const float4* cs4 = reinterpret_cast<const float4*>(P.acs);
  for (int k = 0; k < kScanDepth - 1; ++k) {
    const int c = nch - 1 - k;
    if (c >= 0) scan_issue(ring, inc, nch, c, k, base, G, total);
    else asm volatile("cp.async.commit_group;\n" ::: "memory");
  }
  float FS[kScanF][8], FZ[kScanF][8];
#pragma unroll
  for (int s = 0; s < kScanF; ++s) {
    const int g = base + s * G;
#pragma unroll
    for (int i = 0; i < 8; ++i) FS[s][i] = FZ[s][i] = 0.f;
    if (g < total) {
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
  for (int k = 0; k < nch; ++k) {  // step k handles chunk c = nch - 1 - k
    const int c = nch - 1 - k, kn = k + kScanDepth - 1, cn = nch - 1 - kn;
    if (cn >= 0) scan_issue(ring, inc, nch, cn, kn % kScanDepth, base, G, total);
    else asm volatile("cp.async.commit_group;\n" ::: "memory");
    scan_wait<kScanDepth - 1>();
    const int d = k % kScanDepth;
#pragma unroll
    for (int s = 0; s < kScanF; ++s) {
      const int g = base + s * G;
      if (g < total) {
        const int n = g >> 11, xo = g & (kOct - 1);
        unsigned char* t = P.adjb + ((int64_t)n * nch + c) * 2 * kTileBytes + oct_off(xo);
        *reinterpret_cast<uint4*>(t) = pack8(FS[s]);
        *reinterpret_cast<uint4*>(t + kTileBytes) = pack8(FZ[s]);
        const float4 a = cs4[(int64_t)n * nch + c];
        float dS[8], dZ[8];
        scan_take(ring, d, s, dS, dZ);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float nFS = a.x * FS[s][i] + dS[i];
          FZ[s][i] = a.y * FS[s][i] + a.z * FZ[s][i] + dZ[i];
          FS[s][i] = nFS;
        }
      }
    }
  }
#pragma unroll
  for (int s = 0; s < kScanF; ++s) {
    const int g = base + s * G;
    if (g < total) {
      if (P.dS0) st8f4(P.dS0 + (int64_t)g * 8, FS[s]);
      if (P.dZ0) st8f4(P.dZ0 + (int64_t)g * 8, FZ[s]);
    }
  }
}

}  // namespace tc
}  // namespace atlas
