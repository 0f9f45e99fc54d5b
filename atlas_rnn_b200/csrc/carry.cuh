// Carry composition of the sequence-parallel split (the split-scan identity of
// tests/test_titans.py:680-707): every rank holds the segment transforms of all
// ranks, gathered into one buffer [P][len] where a rank's record is
//   coef [N][3] (padded to a multiple of 4 floats) | dS [N][D2] | dZ [N][D2].
// Forward:  (S, Z)   -> (a S + b Z + dS, c Z + dZ), ranks 0 .. P-1 in order;
//           out: the incoming (S, Z) of `rank`, S_T (unclamped), clamp(S_T) and Z_T.
// Backward: (FS, FZ) -> (a FS + dFS, b FS + c FZ + dFZ), ranks P-1 .. 0;
//           FS enters masked where the forward clamp saturated (rnn_memory.py:701);
//           out: the adjoint arriving at the end of `rank`'s segment and the
//           adjoint at the sequence start (dS0, dZ0).
// One thread per state element, reading each rank's record once: HBM-bound,
// 2 P D2 N floats in.
#pragma once
#include "common.cuh"

namespace atlas {

struct CarryArgs {
  const float* seg;  // [P][len]
  int64_t len, coef_len, ND2;
  int P, rank, N, backward;
  int64_t D2;
  const float* S0;   // forward: S0 / Z0; backward: FS_end / FZ_end (nullable = 0)
  const float* Z0;
  const float* ST;   // backward: unclamped S_T for the clamp mask (nullable = no mask)
  float *in_S, *in_Z, *out_S, *out_Sc, *out_Z;
};

__global__ void __launch_bounds__(kThreads) k_compose_carries(CarryArgs A) {
  for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < A.ND2; e += (int64_t)gridDim.x * kThreads) {
    const int n = (int)(e / A.D2);
    float S = A.S0 ? A.S0[e] : 0.f, Z = A.Z0 ? A.Z0[e] : 0.f;
    if (!A.backward) {
      for (int p = 0; p < A.P; ++p) {
        const float* r = A.seg + (int64_t)p * A.len;
        if (p == A.rank) {
          if (A.in_S) A.in_S[e] = S;
          if (A.in_Z) A.in_Z[e] = Z;
        }
        const float a = r[n * 3], b = r[n * 3 + 1], c = r[n * 3 + 2];
        const float dS = r[A.coef_len + e], dZ = r[A.coef_len + A.ND2 + e];
        const float nS = a * S + b * Z + dS;
        Z = c * Z + dZ;
        S = nS;
      }
      if (A.out_S) A.out_S[e] = S;
      if (A.out_Sc) A.out_Sc[e] = fminf(fmaxf(S, -100.f), 100.f);  // rnn_memory.py:701
      if (A.out_Z) A.out_Z[e] = Z;
    } else {
      if (A.ST && !(A.ST[e] >= -100.f && A.ST[e] <= 100.f)) S = 0.f;  // clamp gradient
      for (int p = A.P - 1; p >= 0; --p) {
        const float* r = A.seg + (int64_t)p * A.len;
        if (p == A.rank) {
          if (A.in_S) A.in_S[e] = S;
          if (A.in_Z) A.in_Z[e] = Z;
        }
        const float a = r[n * 3], b = r[n * 3 + 1], c = r[n * 3 + 2];
        const float dS = r[A.coef_len + e], dZ = r[A.coef_len + A.ND2 + e];
        const float nS = a * S + dS;
        Z = b * S + c * Z + dZ;
        S = nS;
      }
      if (A.out_S) A.out_S[e] = S;
      if (A.out_Z) A.out_Z[e] = Z;
    }
  }
}

}  // namespace atlas
