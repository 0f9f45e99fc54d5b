// One decoding step (T = 1) of the memory recurrence as a single streaming
// kernel: the per-token work of rnn_memory.py:655-730 at seq_len 1, without the
// chunk machinery (no workspaces, nothing kept for a backward).
//
//   delta = S_ref phi(k) - v                          (rnn_memory.py:659-660)
//   g_raw = delta phi(k)^T, times u with token gates  (:663-668)
//   g     = window sum over [buf_in[0..e-2], g_raw]   (:673-687; window gates weight
//           entry j back by U[j], token / no gates by 1)
//   Z_end = beta Z0 + g,  S_end = clamp(alpha S0 - eta Z_end, -100, 100)
//           (without momentum: alpha S0 - eta g)      (:697-702)
//   y     = S0 phi(q)                                 (:712-717, first token)
//   buf_out = [buf_in[1..e-2], g_raw]
//
// Grid (ceil(d_v / 8), N), 256 threads: warp w owns state row r = 8 x + w; lane l
// takes columns l, l + 32, ... (d_phi <= 256), so every access of a warp is one
// contiguous row segment. HBM-bound: per unit it reads S_ref, S0, Z0 and the
// buffer once and writes S_end, Z_end and the buffer once.
#pragma once
#include "chunk_kernels.cuh"

namespace atlas {

constexpr int kDecodeRows = kThreads / 32;  // state rows per CTA
constexpr int kDecodeCols = 8;              // columns per lane (d_phi <= 256)

__global__ void __launch_bounds__(kThreads) k_decode_step(Params P) {
  __shared__ float phk[32 * kDecodeCols], phq[32 * kDecodeCols];
  const int n = blockIdx.y, lane = threadIdx.x & 31, dphi = P.dphi, dv = P.dv, e = P.e;
  for (int m = threadIdx.x; m < dphi; m += kThreads) {
    phk[m] = load_phi(P, n, 0, m, false);
    phq[m] = load_phi(P, n, 0, m, true);
  }
  __syncthreads();
  const int r = blockIdx.x * kDecodeRows + (threadIdx.x >> 5);
  if (r >= dv) return;
  const float al = ldio(P.decay, n, P.bf), et = ldio(P.lr, n, P.bf);
  const float be = P.mom ? ldio(P.beta, n, P.bf) : 0.f;
  // weights of the new term and of buffer entry kb (kb = 0 the oldest)
  float wraw = 1.f, graw_scale = 1.f;
  if (P.gmode == ATLAS_GATE_TOKEN) graw_scale = ldio(P.gate, n, P.bf);  // stored gated
  if (P.gmode == ATLAS_GATE_WINDOW) wraw = ldio(P.gate, (int64_t)n * e, P.bf);
  auto wbuf = [&](int kb) -> float {
    return P.gmode == ATLAS_GATE_WINDOW ? ldio(P.gate, (int64_t)n * e + (e - 1 - kb), P.bf) : 1.f;
  };
  const int64_t D2 = (int64_t)dv * dphi, o = (int64_t)n * D2 + (int64_t)r * dphi;
  float s0[kDecodeCols];
  float dsum = 0.f, ysum = 0.f;
#pragma unroll
  for (int i = 0; i < kDecodeCols; ++i) {
    const int c = lane + 32 * i;
    s0[i] = 0.f;
    if (c < dphi) {
      s0[i] = P.S0[o + c];
      dsum += P.Sref[o + c] * phk[c];
      ysum += s0[i] * phq[c];
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    dsum += __shfl_xor_sync(0xffffffffu, dsum, off);
    ysum += __shfl_xor_sync(0xffffffffu, ysum, off);
  }
  const float delta = dsum - ldio(P.v, (int64_t)n * dv + r, P.bf);
  if (lane == 0) stio(P.y, (int64_t)n * dv + r, ysum, P.bf);
  const int e1 = e - 1;
#pragma unroll
  for (int i = 0; i < kDecodeCols; ++i) {
    const int c = lane + 32 * i;
    if (c >= dphi) continue;
    const float graw = delta * phk[c] * graw_scale;
    float g = wraw * graw;
    for (int kb = 0; kb < e1; ++kb) {
      const float b = P.buf ? P.buf[((int64_t)n * e1 + kb) * D2 + (int64_t)r * dphi + c] : 0.f;
      g += wbuf(kb) * b;
      if (kb >= 1) P.buf_out[((int64_t)n * e1 + kb - 1) * D2 + (int64_t)r * dphi + c] = b;
    }
    if (e1 > 0) P.buf_out[((int64_t)n * e1 + e1 - 1) * D2 + (int64_t)r * dphi + c] = graw;
    float s1;
    if (P.mom) {
      const float z1 = be * (P.Z0 ? P.Z0[o + c] : 0.f) + g;
      if (P.Z_end) P.Z_end[o + c] = z1;
      s1 = al * s0[i] - et * z1;
    } else {
      s1 = al * s0[i] - et * g;
    }
    P.S_end[o + c] = fminf(fmaxf(s1, -100.f), 100.f);  // rnn_memory.py:701
  }
}

// The same step with float4 lanes (d_phi % 4 == 0, 16-byte aligned state rows):
// lane l takes columns 4 l .. 4 l + 3 (+ 128 for d_phi > 128), and every load of a
// row segment is issued before the arithmetic that needs it.
__device__ __forceinline__ float4 f4fma(float a, float4 x, float4 y) {  // a x + y
  return make_float4(a * x.x + y.x, a * x.y + y.y, a * x.z + y.z, a * x.w + y.w);
}
__global__ void __launch_bounds__(kThreads) k_decode_step4(Params P) {
  __shared__ __align__(16) float phk[256], phq[256];
  const int n = blockIdx.y, lane = threadIdx.x & 31, dphi = P.dphi, dv = P.dv, e = P.e, e1 = e - 1;
  for (int m = threadIdx.x; m < dphi; m += kThreads) {
    phk[m] = load_phi(P, n, 0, m, false);
    phq[m] = load_phi(P, n, 0, m, true);
  }
  __syncthreads();
  const int r = blockIdx.x * kDecodeRows + (threadIdx.x >> 5);
  if (r >= dv) return;
  const float al = ldio(P.decay, n, P.bf), et = ldio(P.lr, n, P.bf);
  const float be = P.mom ? ldio(P.beta, n, P.bf) : 0.f;
  float wraw = 1.f, graw_scale = 1.f;
  if (P.gmode == ATLAS_GATE_TOKEN) graw_scale = ldio(P.gate, n, P.bf);
  if (P.gmode == ATLAS_GATE_WINDOW) wraw = ldio(P.gate, (int64_t)n * e, P.bf);
  const int64_t D2 = (int64_t)dv * dphi, o = (int64_t)n * D2 + (int64_t)r * dphi;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 s0[2], sr[2], z0[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int c = 4 * lane + 128 * t;
    const bool ok = c < dphi;
    s0[t] = ok ? *reinterpret_cast<const float4*>(P.S0 + o + c) : zero;
    sr[t] = ok ? *reinterpret_cast<const float4*>(P.Sref + o + c) : zero;
    z0[t] = ok && P.mom && P.Z0 ? *reinterpret_cast<const float4*>(P.Z0 + o + c) : zero;
  }
  float dsum = 0.f, ysum = 0.f;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int c = 4 * lane + 128 * t;
    if (c < dphi) {
      const float4 pk = *reinterpret_cast<const float4*>(phk + c), pq = *reinterpret_cast<const float4*>(phq + c);
      dsum += sr[t].x * pk.x + sr[t].y * pk.y + sr[t].z * pk.z + sr[t].w * pk.w;
      ysum += s0[t].x * pq.x + s0[t].y * pq.y + s0[t].z * pq.z + s0[t].w * pq.w;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    dsum += __shfl_xor_sync(0xffffffffu, dsum, off);
    ysum += __shfl_xor_sync(0xffffffffu, ysum, off);
  }
  const float delta = dsum - ldio(P.v, (int64_t)n * dv + r, P.bf);
  if (lane == 0) stio(P.y, (int64_t)n * dv + r, ysum, P.bf);
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int c = 4 * lane + 128 * t;
    if (c >= dphi) continue;
    const float4 pk = *reinterpret_cast<const float4*>(phk + c);
    const float gs = delta * graw_scale;
    const float4 graw = make_float4(gs * pk.x, gs * pk.y, gs * pk.z, gs * pk.w);
    float4 g = make_float4(wraw * graw.x, wraw * graw.y, wraw * graw.z, wraw * graw.w);
    const float* bin = P.buf ? P.buf + (int64_t)n * e1 * D2 + (int64_t)r * dphi + c : nullptr;
    float* bout = e1 > 0 ? P.buf_out + (int64_t)n * e1 * D2 + (int64_t)r * dphi + c : nullptr;
    int kb = 0;
    for (; kb + 4 <= e1; kb += 4) {  // four buffer entries in flight at a time
      float4 b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) b[u] = bin ? *reinterpret_cast<const float4*>(bin + (kb + u) * D2) : zero;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float w = P.gmode == ATLAS_GATE_WINDOW ? ldio(P.gate, (int64_t)n * e + (e - 1 - (kb + u)), P.bf) : 1.f;
        g = f4fma(w, b[u], g);
        if (kb + u >= 1) *reinterpret_cast<float4*>(bout + (kb + u - 1) * D2) = b[u];
      }
    }
    for (; kb < e1; ++kb) {
      const float4 b = bin ? *reinterpret_cast<const float4*>(bin + kb * D2) : zero;
      const float w = P.gmode == ATLAS_GATE_WINDOW ? ldio(P.gate, (int64_t)n * e + (e - 1 - kb), P.bf) : 1.f;
      g = f4fma(w, b, g);
      if (kb >= 1) *reinterpret_cast<float4*>(bout + (kb - 1) * D2) = b;
    }
    if (e1 > 0) *reinterpret_cast<float4*>(bout + (e1 - 1) * D2) = graw;
    float4 s1;
    if (P.mom) {
      const float4 z1 = f4fma(be, z0[t], g);
      if (P.Z_end) *reinterpret_cast<float4*>(P.Z_end + o + c) = z1;
      s1 = make_float4(al * s0[t].x - et * z1.x, al * s0[t].y - et * z1.y, al * s0[t].z - et * z1.z,
                       al * s0[t].w - et * z1.w);
    } else {
      s1 = make_float4(al * s0[t].x - et * g.x, al * s0[t].y - et * g.y, al * s0[t].z - et * g.z,
                       al * s0[t].w - et * g.w);
    }
    *reinterpret_cast<float4*>(P.S_end + o + c) =  // rnn_memory.py:701
        make_float4(fminf(fmaxf(s1.x, -100.f), 100.f), fminf(fmaxf(s1.y, -100.f), 100.f),
                    fminf(fmaxf(s1.z, -100.f), 100.f), fminf(fmaxf(s1.w, -100.f), 100.f));
  }
}

}  // namespace atlas
