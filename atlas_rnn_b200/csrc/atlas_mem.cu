// C ABI of libatlas_mem.so: argument checks, workspace layout and the launch
// sequences of the forward and backward passes. Declarations and the reference
// interfaces they replace are in include/atlas_mem.h.
#include <cudaTypedefs.h>
#include <mutex>

#include <algorithm>
#include <cstdlib>

#include "chunk_kernels.cuh"
#include "tc_bwd.cuh"
#include "tc_scan.cuh"
#include "tc_fmap.cuh"
#include "decode.cuh"
#include "scan_op.cuh"
#include "omega_store.cuh"
#include "affine_scan.cuh"
#include "carry.cuh"
#include "dwconv.cuh"
#include "headprep.cuh"
#include "umma_selftest.cuh"

using namespace atlas;

namespace {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }
inline int r4(int n) { return (n + 3) & ~3; }

// The chunk kernels have tensor-core versions (1 forward chunk increments,
// 2 forward outputs, 4 backward chunk increments, 8 backward gradients); a
// shape runs either all of them or none, since they share bf16 workspaces.
constexpr int kTcAll = 15;

// Tensor cores for bf16 io with d_phi = d_v = 128 and window <= 16;
// ATLAS_MEM_TC=0 selects the CUDA-core kernels instead.
int tc_groups(const AtlasMemShape* s) {
  if (s->dtype_io != ATLAS_BF16 || s->d_phi != tc::kD || s->d_v != tc::kD || s->window > 16) return 0;
  if (const char* env = std::getenv("ATLAS_MEM_TC"))
    if (std::atoi(env) == 0) return 0;
  return kTcAll;
}

// The tensor feature map runs on tensor cores (tc_fmap.cuh) for bf16 io and
// the head sizes it handles; otherwise on CUDA cores (k_fmap_tensor_*).
bool fmap_tc(const AtlasMemShape* s) {
  return s->fmap_mode == ATLAS_FMAP_TENSOR && tc::fmap_tc_ok(s->d_k, s->d_phi, s->dtype_io == ATLAS_BF16);
}

// Tokens per chunk: the caller's choice, else 128 - e when every chunk kernel
// runs on tensor cores (keys = chunk + e - 1 fill a 128-row tile), else the
// CUDA-core kernels' 32.
int chunk_of(const AtlasMemShape* s) {
  if (s->chunk > 0) return s->chunk;
  if (tc_groups(s) == kTcAll) return 128 - s->window;
  return s->window - 1 > 32 ? s->window - 1 : 32;
}

struct Layout {
  int C, nch;
  size_t saved, fwd, bwd;
  size_t st, delta, ST, cs, phik, phiq, dlb, stb, srb, projb;  // in saved
  size_t adj, acs, dpsi, ddel, dphiR, hdd, hdp, du, hdu;       // in bwd scratch
  size_t xq, xf, xs, gt, adjb, ddb, dpb, dpsib;                 // in bwd scratch (tensor-core path)
};

Layout make_layout(const AtlasMemShape* s) {
  Layout L{};
  L.C = chunk_of(s);
  L.nch = (int)((s->T + L.C - 1) / L.C);
  const size_t N = (size_t)s->N, T = (size_t)s->T, nch = (size_t)L.nch;
  const size_t D2 = (size_t)s->d_v * s->d_phi, e1 = (size_t)(s->window - 1);
  const bool tens = s->fmap_mode == ATLAS_FMAP_TENSOR;
  size_t o = 0;
  auto put = [&](size_t bytes) { const size_t at = o; o = align_up(o + bytes); return at; };
  const bool tcm = tc_groups(s) == kTcAll;
  L.st = put(N * nch * 2 * D2 * 4);
  L.delta = tcm ? 0 : put(N * T * s->d_v * 4);
  L.dlb = tcm ? put(N * T * s->d_v * 2) : 0;
  L.stb = tcm ? put(N * nch * 2 * (size_t)tc::kTileBytes) : 0;
  L.srb = tcm ? put(N * (size_t)tc::kTileBytes) : 0;
  L.ST = put(N * D2 * 4);
  L.cs = put(N * nch * 4 * 4);
  L.phik = tens ? put(N * T * s->d_phi * 4) : 0;
  L.phiq = tens ? put(N * T * s->d_phi * 4) : 0;
  L.projb = fmap_tc(s) ? put((size_t)(s->d_k + 1) * tc::fm_chunk_bytes(s->d_k, s->d_phi)) : 0;
  L.saved = o;
  L.fwd = 0;
  o = 0;
  L.adj = put(N * nch * 2 * D2 * 4);
  L.acs = put(N * nch * 4 * 4);
  L.dpsi = put(N * T * s->d_phi * 4);
  L.ddel = put(N * T * s->d_v * 4);
  L.dphiR = put(N * T * s->d_phi * 4);
  L.hdd = put(N * nch * (e1 ? e1 : 1) * s->d_v * 4);
  L.hdp = put(N * nch * (e1 ? e1 : 1) * s->d_phi * 4);
  L.du = put(N * T * 4);
  L.hdu = put(N * nch * (e1 ? e1 : 1) * 4);
  if (tc_groups(s) & 8) {
    L.xq = put(N * nch * 128 * 2 * 4);
    L.xf = put(N * nch * 128 * 2 * 4);
    L.xs = put(N * nch * 4 * 4);
    L.gt = put(N * nch * (size_t)tc::kTileBytes);
    L.adjb = put(N * nch * 2 * (size_t)tc::kTileBytes);
    L.ddb = put(N * T * s->d_v * 2);
    L.dpb = put(N * T * s->d_phi * 2);
    L.dpsib = put(N * T * s->d_phi * 2);
  }
  L.bwd = o;
  return L;
}

// Dynamic shared memory of each kernel; mirrors the SmemAlloc::take sequences.
struct Smem {
  size_t f1, f3, b1, b3, fin, dsref, bufout, fmf, fmb, tc_f1, tc_f3, buf_y, tc_b1, tc_b4, tc_b6, buf_b;
};
Smem smem_sizes(const AtlasMemShape* s, int C) {
  const int e = s->window, L = C, K = C + e - 1, dphi = s->d_phi, dv = s->d_v, dk = s->d_k;
  const int ctx = r4(C) * 3 + r4(C + e) + r4(C * e);
  const int coefF = 2 * r4((L + 1) * K) + 3 * r4(L + 1);
  const int coefA = 3 * r4(L + 1) + 2 * r4((L + 1) * L);
  Smem m{};
  m.f1 = 4 * (size_t)(ctx + r4(K * dphi) + r4(K * dv) + coefF + kStageFloats);
  m.f3 = 4 * (size_t)(ctx + r4(K * dphi) + r4(K * dv) + r4(L * dphi) + r4(L * K) + coefF + kStageFloats);
  m.b1 = 4 * (size_t)(ctx + r4(L * dphi) + r4(L * dv) + coefA + kStageFloats);
  m.b3 = 4 * (size_t)(ctx + r4(K * dphi) + 2 * r4(K * dv) + r4(L * dphi) + r4(L * dv) + 2 * r4(L * K) +
                      r4((L + 2) * (K + 2)) + coefF + coefA + 2 * r4(K) + r4(K * L) + r4(3 * L) + r4(K) + 32 +
                      kStageFloats);
  m.fin = 4 * (size_t)(r4(kFinTile * dv) + kStageFloats);
  m.dsref = 4 * (size_t)kStageFloats;
  m.bufout = 4 * (size_t)(dphi + dv + 32);
  m.fmf = 4 * (size_t)(r4(kFmTile * dk) + kStageFloats);
  m.fmb = 4 * (size_t)(2 * r4(kFmTile * dk) + r4(kFmTile * dphi) + kStageFloats);
  const int tctx = tc::ctx_floats(C, e);
  m.tc_f1 = 3 * (size_t)tc::kTileBytes + 4 * (size_t)(tctx + 5 * tc::kR);
  m.tc_f3 = 6 * (size_t)tc::kTileBytes + 4 * (size_t)(tctx + 3 * 132);
  m.buf_y = 4 * (size_t)(ctx + r4(C * (e > 1 ? e - 1 : 1)) + r4(C * dphi) + kStageFloats);
  m.tc_b1 = 3 * (size_t)tc::kTileBytes + 4 * (size_t)(tctx + 6 * 132);
  m.tc_b4 = 6 * (size_t)tc::kTileBytes +
            4 * (size_t)(tctx + 6 * 132 + 2 * 2 * tc::kR + 4 + tc::kR + 4 * (tc::kT / 32) +
                         tc::kGateParts * (tc::kWG - 1) * tc::kR + 2 * tc::kR);
  m.tc_b6 = 6 * (size_t)tc::kTileBytes +
            4 * (size_t)(tctx + 6 * 132 + 4 * tc::kR + 4 + tc::kR + tc::kGateParts * (tc::kWG - 1) * tc::kR);
  m.buf_b = 4 * (size_t)(ctx + r4(C * dphi) + r4(C * dv) + 3 * r4(C * (e > 1 ? e - 1 : 1)) + 3 * r4(C + 1) + 32 +
                         kStageFloats);
  return m;
}

int max_smem_optin() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return 0;
  return v;
}

// Raise the dynamic shared-memory cap of every kernel once per device.
std::mutex g_attr_mu;
bool g_attr_done[64];
int ensure_attrs() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ATLAS_ERR_LAUNCH;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (dev < 64 && g_attr_done[dev]) return ATLAS_OK;
  const int mx = max_smem_optin();
  const void* ks[] = {(const void*)k_fwd_chunk,   (const void*)k_fwd_out,      (const void*)k_bwd_chunk,
                      (const void*)k_bwd_grads,   (const void*)k_bwd_finalize, (const void*)k_bwd_dsref,
                      (const void*)k_bwd_bufout,  (const void*)k_fmap_tensor_fwd, (const void*)k_fmap_tensor_bwd,
                      (const void*)k_fwd_scan<1>, (const void*)k_fwd_scan<4>, (const void*)k_bwd_scan<1>,
                      (const void*)k_bwd_scan<4>, (const void*)tc::k_fwd_chunk_tc, (const void*)tc::k_fwd_out_tc,
                      (const void*)tc::k_fwd_buf_y, (const void*)tc::k_bwd_chunk_tc, (const void*)tc::k_bwd_state_gates_tc,
                      (const void*)tc::k_bwd_buf_tc,
                      (const void*)tc::k_bwd_finalize_tc, (const void*)tc::k_bwd_dsref_tc, (const void*)tc::k_bwd_keys_tc,
                      (const void*)tc::k_fwd_scan_tc<1>, (const void*)tc::k_fwd_scan_tc<2>,
                      (const void*)tc::k_fwd_scan_tc<4>, (const void*)tc::k_bwd_scan_tc<1>,
                      (const void*)tc::k_bwd_scan_tc<2>, (const void*)tc::k_bwd_scan_tc<4>,
                      (const void*)tc::k_fmap_fwd_tc, (const void*)tc::k_fmap_bwd_tc,
                      (const void*)k_affine_scan_fwd, (const void*)k_affine_scan_bwd};
  for (const void* k : ks) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, k) != cudaSuccess) return ATLAS_ERR_LAUNCH;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, mx - (int)fa.sharedSizeBytes) !=
        cudaSuccess)
      return ATLAS_ERR_LAUNCH;
  }
  if (dev < 64) g_attr_done[dev] = true;
  return ATLAS_OK;
}

int validate_shape(const AtlasMemShape* s) {
  if (!s) return ATLAS_ERR_INVALID_ARG;
  if (s->N < 1 || s->T < 1 || s->d_k < 1 || s->d_phi < 1 || s->d_v < 1 || s->window < 1)
    return ATLAS_ERR_INVALID_ARG;
  if (s->fmap_mode < 0 || s->fmap_mode > 2 || s->gate_mode < 0 || s->gate_mode > 2) return ATLAS_ERR_INVALID_ARG;
  if (s->dtype_io != ATLAS_F32 && s->dtype_io != ATLAS_BF16) return ATLAS_ERR_INVALID_ARG;
  if (s->momentum != 0 && s->momentum != 1) return ATLAS_ERR_INVALID_ARG;
  if (s->fmap_mode != ATLAS_FMAP_TENSOR && s->d_phi != s->d_k) return ATLAS_ERR_INVALID_ARG;
  if (s->fmap_mode == ATLAS_FMAP_TENSOR && s->fmap_degree <= 1) return ATLAS_ERR_INVALID_ARG;
  if (s->d_phi > 256 || s->d_v > 256 || s->d_k > 256) return ATLAS_ERR_UNSUPPORTED;
  if (s->N > 65535 || s->T > (int64_t)1 << 30) return ATLAS_ERR_UNSUPPORTED;
  const int C = chunk_of(s);
  const int tcg = tc_groups(s);
  if (C < 1 || C < s->window - 1) return ATLAS_ERR_UNSUPPORTED;
  if (tcg != kTcAll && (C > 64 || C + s->window > 127)) return ATLAS_ERR_UNSUPPORTED;
  if (tcg && C + s->window > 128) return ATLAS_ERR_UNSUPPORTED;
  if ((int64_t)s->N * s->T * (s->d_v > s->d_phi ? s->d_v : s->d_phi) > ((int64_t)1 << 40)) return ATLAS_ERR_UNSUPPORTED;
  const Smem m = smem_sizes(s, C);
  const size_t mx = (size_t)max_smem_optin() - 1024;  // static shared memory of the tensor-core kernels
  if (mx + 1024 == 0) return ATLAS_ERR_LAUNCH;
  const size_t scan_smem = (size_t)((s->T + C - 1) / C) * 16;
  const size_t big[] = {(tcg & 1) ? 0 : m.f1, (tcg & 2) ? 0 : m.f3, (tcg & 4) ? 0 : m.b1, (tcg & 8) ? 0 : m.b3,
                        m.fin, m.fmf, m.fmb, scan_smem, tcg ? m.tc_f1 : 0, tcg ? m.tc_f3 : 0, tcg ? m.buf_y : 0,
                        tcg ? m.tc_b6 : 0, tcg ? m.buf_b : 0};
  for (size_t b : big)
    if (b > mx) return ATLAS_ERR_UNSUPPORTED;
  return ATLAS_OK;
}

int validate_fwd(const AtlasMemShape* s, const AtlasMemFwd* f, bool need_outputs) {
  if (!f) return ATLAS_ERR_INVALID_ARG;
  if (!f->k || !f->q || !f->v || !f->lr || !f->decay || !f->S_ref || !f->S0) return ATLAS_ERR_INVALID_ARG;
  if (s->momentum && !f->beta) return ATLAS_ERR_INVALID_ARG;
  if (s->gate_mode != ATLAS_GATE_NONE && !f->gate) return ATLAS_ERR_INVALID_ARG;
  if (s->fmap_mode == ATLAS_FMAP_TENSOR && !f->proj) return ATLAS_ERR_INVALID_ARG;
  if (need_outputs && (!f->y || !f->S_end)) return ATLAS_ERR_INVALID_ARG;
  return ATLAS_OK;
}

Params make_params(const AtlasMemShape* s, const Layout& L, const AtlasMemFwd* f, const AtlasMemBwd* b,
                   const void* saved, void* scratch) {
  Params P{};
  P.N = (int)s->N; P.T = (int)s->T; P.dk = s->d_k; P.dphi = s->d_phi; P.dv = s->d_v; P.e = s->window;
  P.fmode = s->fmap_mode; P.fdeg = s->fmap_degree; P.gmode = s->gate_mode; P.mom = s->momentum;
  P.bf = s->dtype_io == ATLAS_BF16; P.C = L.C; P.nch = L.nch;
  if (f) {
    P.k = f->k; P.q = f->q; P.v = f->v; P.lr = f->lr; P.decay = f->decay; P.beta = s->momentum ? f->beta : nullptr;
    P.gate = f->gate; P.Sref = f->S_ref; P.S0 = f->S0; P.Z0 = s->momentum ? f->Z0 : nullptr;
    P.buf = s->window > 1 ? f->buf_in : nullptr; P.proj = f->proj;
    P.y = f->y; P.S_end = f->S_end; P.Z_end = s->momentum ? f->Z_end : nullptr; P.buf_out = f->buf_out;
    P.status = f->status;
  }
  if (b) {
    P.dy = b->dy; P.dS_end = b->dS_end; P.dZ_end = s->momentum ? b->dZ_end : nullptr;
    P.dbuf_out = s->window > 1 ? b->dbuf_out : nullptr;
    P.dk_ = b->dk; P.dq_ = b->dq; P.dv_ = b->dv; P.dlr = b->dlr; P.ddecay = b->ddecay;
    P.dbeta = s->momentum ? b->dbeta : nullptr; P.dgate = s->gate_mode != ATLAS_GATE_NONE ? b->dgate : nullptr;
    P.dSref = b->dS_ref; P.dS0 = b->dS0; P.dZ0 = s->momentum ? b->dZ0 : nullptr;
    P.dbuf = s->window > 1 ? b->dbuf_in : nullptr;
    P.status = b->status;
  }
  char* sv = (char*)const_cast<void*>(saved);
  if (sv) {
    const bool tcm = tc_groups(s) == kTcAll;
    P.st = (float*)(sv + L.st); P.ST = (float*)(sv + L.ST);
    P.delta = tcm ? nullptr : (float*)(sv + L.delta);
    P.dlb = tcm ? (__nv_bfloat16*)(sv + L.dlb) : nullptr;
    P.stb = tcm ? (unsigned char*)(sv + L.stb) : nullptr;
    P.srb = tcm ? (unsigned char*)(sv + L.srb) : nullptr;
    P.inc_bf16 = tcm ? 1 : 0;
    P.cs = (float*)(sv + L.cs);
    P.phik = s->fmap_mode == ATLAS_FMAP_TENSOR ? (float*)(sv + L.phik) : nullptr;
    P.phiq = s->fmap_mode == ATLAS_FMAP_TENSOR ? (float*)(sv + L.phiq) : nullptr;
    P.projb = fmap_tc(s) ? (unsigned char*)(sv + L.projb) : nullptr;
  }
  if (scratch) {
    char* sc = (char*)scratch;
    P.adj = (float*)(sc + L.adj); P.acs = (float*)(sc + L.acs); P.dpsi = (float*)(sc + L.dpsi);
    P.ddel = (float*)(sc + L.ddel); P.dphiR = (float*)(sc + L.dphiR); P.hdd = (float*)(sc + L.hdd);
    P.hdp = (float*)(sc + L.hdp); P.du = (float*)(sc + L.du); P.hdu = (float*)(sc + L.hdu);
    if (tc_groups(s) & 8) {
      P.xq = (float*)(sc + L.xq); P.xf = (float*)(sc + L.xf); P.xs = (float*)(sc + L.xs); P.gt = sc + L.gt;
      P.adjb = (unsigned char*)(sc + L.adjb);
      P.ddb = (__nv_bfloat16*)(sc + L.ddb);
      P.dpb = (__nv_bfloat16*)(sc + L.dpb);
      P.dpsib = (__nv_bfloat16*)(sc + L.dpsib);
    }
  }
  P.apply_mask = 1;
  return P;
}

// ---- launch accounting and optional per-kernel CUDA-event timing ----------
enum KernelId {
  KID_FMAP_FWD, KID_FWD_CHUNK, KID_FWD_SCAN, KID_FWD_OUT, KID_BUF_OUT, KID_BWD_CHUNK, KID_BWD_SCAN,
  KID_BWD_GRADS, KID_BWD_BUFOUT, KID_BWD_FINAL, KID_BWD_DSREF, KID_FMAP_BWD, KID_FWD_CHUNK_TC, KID_FWD_OUT_TC, KID_FWD_BUF_Y,
  KID_BWD_CHUNK_TC, KID_BWD_STATE_GATES_TC, KID_BWD_BUF_TC, KID_BWD_FINAL_TC, KID_BWD_DSREF_TC, KID_BWD_KEYS_TC, KID_SREF_TILE, KID_DECODE, KID_SCAN_OP_FWD, KID_SCAN_OP_BWD, KID_CARRY, KID_DWCONV_FWD, KID_DWCONV_BWD, KID_HEADPREP_FWD, KID_HEADPREP_BWD, KID_PROJ_TILES, KID_FMAP_FWD_TC, KID_FMAP_BWD_TC, KID_OMEGA_STORE_FWD, KID_OMEGA_STORE_BWD, KID_AFFINE_FWD, KID_AFFINE_BWD, KID_COUNT
};
const char* const kKernelNames[KID_COUNT] = {
  "k_fmap_tensor_fwd", "k_fwd_chunk", "k_fwd_scan", "k_fwd_out", "k_buf_out", "k_bwd_chunk", "k_bwd_scan",
  "k_bwd_grads", "k_bwd_bufout", "k_bwd_finalize", "k_bwd_dsref", "k_fmap_tensor_bwd", "k_fwd_chunk_tc", "k_fwd_out_tc", "k_fwd_buf_y",
  "k_bwd_chunk_tc", "k_bwd_state_gates_tc", "k_bwd_buf_tc", "k_bwd_finalize_tc", "k_bwd_dsref_tc", "k_bwd_keys_tc", "k_sref_tile", "k_decode_step", "k_scan_op_fwd", "k_scan_op_bwd", "k_compose_carries", "k_dwconv3_fwd", "k_dwconv3_bwd", "k_head_prep_fwd", "k_head_prep_bwd", "k_proj_tiles", "k_fmap_fwd_tc", "k_fmap_bwd_tc", "k_omega_store_fwd", "k_omega_store_bwd", "k_affine_scan_fwd", "k_affine_scan_bwd"};

constexpr int kMaxTimed = 8192;
struct Prof {
  std::mutex mu;
  bool timing = false;
  long long launches = 0;
  int pending = 0;
  cudaEvent_t ev[2 * kMaxTimed];
  bool ev_ready = false;
  int kid[kMaxTimed];
  double ms[KID_COUNT] = {};
  long long cnt[KID_COUNT] = {};
};
Prof g_prof;

void prof_collect_locked() {
  for (int i = 0; i < g_prof.pending; ++i) {
    float ms = 0.f;
    cudaEventSynchronize(g_prof.ev[2 * i + 1]);
    cudaEventElapsedTime(&ms, g_prof.ev[2 * i], g_prof.ev[2 * i + 1]);
    g_prof.ms[g_prof.kid[i]] += ms;
    g_prof.cnt[g_prof.kid[i]] += 1;
  }
  g_prof.pending = 0;
}

int prof_begin(int kid, cudaStream_t st) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  g_prof.launches++;
  if (!g_prof.timing) return -1;
  if (g_prof.pending == kMaxTimed) prof_collect_locked();
  const int i = g_prof.pending++;
  g_prof.kid[i] = kid;
  cudaEventRecord(g_prof.ev[2 * i], st);
  return i;
}
void prof_end(int slot, cudaStream_t st) {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lk(g_prof.mu);
  cudaEventRecord(g_prof.ev[2 * slot + 1], st);
}

#define LAUNCH_CHECK()                                              \
  do {                                                              \
    if (cudaGetLastError() != cudaSuccess) return ATLAS_ERR_LAUNCH; \
  } while (0)

// Launch with an explicit thread count: LAUNCH_T(id, kernel, grid, threads, smem, stream, args...)
#define LAUNCH_T(KID, KERNEL, GRID, THREADS, SMEM, STREAM, ...)   \
  do {                                                            \
    const int slot_ = prof_begin(KID, STREAM);                    \
    KERNEL<<<GRID, THREADS, SMEM, STREAM>>>(__VA_ARGS__);         \
    LAUNCH_CHECK();                                               \
    prof_end(slot_, STREAM);                                      \
  } while (0)

// Launch `kernel` with accounting: LAUNCH(id, kernel, grid, smem, stream, args...)
#define LAUNCH(KID, KERNEL, GRID, SMEM, STREAM, ...)              \
  do {                                                            \
    const int slot_ = prof_begin(KID, STREAM);                    \
    KERNEL<<<GRID, kThreads, SMEM, STREAM>>>(__VA_ARGS__);        \
    LAUNCH_CHECK();                                               \
    prof_end(slot_, STREAM);                                      \
  } while (0)

// Sequential chunk scans: float4 per thread when the state size allows it.
int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cached[dev] = v;
  }
  return cached[dev];
}

// One resident wave of tc::k_{fwd,bwd}_scan_tc: F groups of 8 elements per thread, F the smallest of
// 1, 2, 4 that covers the units (rounds of F = 4 beyond that).
template <int F>
int launch_scan_tc_f(bool fwd, const Params& P, int dry, int rounds, int threads, cudaStream_t st) {
  const int grid = sm_count();
  for (int r = 0; r < rounds; ++r) {
    if (fwd)
      LAUNCH_T(KID_FWD_SCAN, tc::k_fwd_scan_tc<F>, dim3(grid), threads, tc::kScanRingBytes, st, P, r, dry);
    else
      LAUNCH_T(KID_BWD_SCAN, tc::k_bwd_scan_tc<F>, dim3(grid), threads, tc::kScanRingBytes, st, P, r, dry);
  }
  return ATLAS_OK;
}
int launch_scan_tc(bool fwd, const Params& P, int dry, cudaStream_t st) {
  const int64_t sms = sm_count(), G = sms * tc::kScanThreads, total = (int64_t)P.N * tc::kOct;
  const int64_t per = (total + G - 1) / G;  // groups per thread at full CTAs
  const int F = per <= 1 ? 1 : (per <= 2 ? 2 : 4);
  // threads per CTA: the fewest warps that still cover one round of F groups per thread on every SM
  const int64_t need = (total + F * sms - 1) / (F * sms);
  const int threads = per > 4 ? tc::kScanThreads : (int)std::min<int64_t>(tc::kScanThreads, (need + 31) / 32 * 32);
  if (F == 1) return launch_scan_tc_f<1>(fwd, P, dry, 1, threads, st);
  if (F == 2) return launch_scan_tc_f<2>(fwd, P, dry, 1, threads, st);
  return launch_scan_tc_f<4>(fwd, P, dry, (int)((per + 3) / 4), threads, st);
}

int launch_scan(bool fwd, const Params& P, int dry, cudaStream_t st) {
  const int64_t D2 = (int64_t)P.dv * P.dphi;
  if (P.inc_bf16 && (dry || (fwd ? P.stb != nullptr : P.adjb != nullptr)) && P.dv == tc::kD &&
      P.dphi == tc::kD && (int64_t)P.N * tc::kOct < ((int64_t)1 << 31) &&
      std::getenv("ATLAS_MEM_SCAN_GENERIC") == nullptr)
    return launch_scan_tc(fwd, P, dry, st);
  const size_t smem = (size_t)P.nch * sizeof(float4);
  const bool v4 = (D2 % 4) == 0;
  const int64_t units = v4 ? D2 / 4 : D2;
  const dim3 grid((unsigned)((units + kThreads - 1) / kThreads), P.N);
  if (fwd) {
    if (v4) LAUNCH(KID_FWD_SCAN, k_fwd_scan<4>, grid, smem, st, P, dry);
    else LAUNCH(KID_FWD_SCAN, k_fwd_scan<1>, grid, smem, st, P, dry);
  } else {
    if (v4) LAUNCH(KID_BWD_SCAN, k_bwd_scan<4>, grid, smem, st, P, dry);
    else LAUNCH(KID_BWD_SCAN, k_bwd_scan<1>, grid, smem, st, P, dry);
  }
  return ATLAS_OK;
}

int run_fwd_local(const AtlasMemShape* s, const Params& P, cudaStream_t st) {
  const Smem m = smem_sizes(s, P.C);
  const dim3 gch(P.nch, P.N);
  if (P.fmode == ATLAS_FMAP_TENSOR) {
    if (fmap_tc(s)) {
      LAUNCH(KID_PROJ_TILES, tc::k_proj_tiles, dim3(P.dk + 1), 0, st, P);
      LAUNCH_T(KID_FMAP_FWD_TC, tc::k_fmap_fwd_tc, dim3((P.T + tc::kFmRows - 1) / tc::kFmRows, P.N, 2), tc::kFmT,
               tc::fm_fwd_smem(P.dk, P.dphi), st, P);
    } else {
      LAUNCH(KID_FMAP_FWD, k_fmap_tensor_fwd, dim3((P.T + kFmTile - 1) / kFmTile, P.N, 2), m.fmf, st, P);
    }
  }
  if (tc_groups(s) & 1) {
    LAUNCH(KID_SREF_TILE, tc::k_sref_tile, dim3(P.N), 0, st, P);
    LAUNCH_T(KID_FWD_CHUNK_TC, tc::k_fwd_chunk_tc, gch, tc::kT, m.tc_f1, st, P);
  }
  else LAUNCH(KID_FWD_CHUNK, k_fwd_chunk, gch, m.f1, st, P);
  return ATLAS_OK;
}

int run_fwd_finish(const AtlasMemShape* s, const Params& P, cudaStream_t st) {
  const Smem m = smem_sizes(s, P.C);
  if (int v = launch_scan(true, P, 0, st)) return v;
  if (tc_groups(s) & 2) {
    LAUNCH_T(KID_FWD_OUT_TC, tc::k_fwd_out_tc, dim3((unsigned)std::min(P.nch * P.N, sm_count())), tc::kT, m.tc_f3,
             st, P);
    if (P.buf && P.e > 1)
      LAUNCH(KID_FWD_BUF_Y, tc::k_fwd_buf_y, dim3((P.dv + 63) / 64, P.N), m.buf_y, st, P);
  } else {
    LAUNCH(KID_FWD_OUT, k_fwd_out, dim3(P.nch, P.N), m.f3, st, P);
  }
  if (P.e > 1 && P.buf_out) {
    LAUNCH(KID_BUF_OUT, k_buf_out, dim3(P.e - 1, P.N), 0, st, P);
  }
  return ATLAS_OK;
}

int run_bwd_local(const AtlasMemShape* s, const Params& P, cudaStream_t st) {
  const Smem m = smem_sizes(s, P.C);
  if (tc_groups(s) & 4) LAUNCH_T(KID_BWD_CHUNK_TC, tc::k_bwd_chunk_tc, dim3(P.nch, P.N), tc::kT, m.tc_b1, st, P);
  else LAUNCH(KID_BWD_CHUNK, k_bwd_chunk, dim3(P.nch, P.N), m.b1, st, P);
  return ATLAS_OK;
}

int run_bwd_finish(const AtlasMemShape* s, const Params& P, cudaStream_t st) {
  const Smem m = smem_sizes(s, P.C);
  if (int v = launch_scan(false, P, 0, st)) return v;
  if (tc_groups(s) & 8) {
    const dim3 g(P.nch, P.N);
    // keys (d psi part I5, G, xf), the carried-buffer terms of chunk 0 (G columns, xf, d psi),
    // then the state side and the gate gradients (d psi completed)
    LAUNCH_T(KID_BWD_KEYS_TC, tc::k_bwd_keys_tc, dim3((unsigned)std::min(P.nch * P.N, sm_count())), tc::kT,
             m.tc_b6, st, P);  // persistent
    if (P.e > 1 && (P.buf || P.dbuf)) LAUNCH(KID_BWD_BUF_TC, tc::k_bwd_buf_tc, dim3(1, P.N), m.buf_b, st, P);
    LAUNCH_T(KID_BWD_STATE_GATES_TC, tc::k_bwd_state_gates_tc, g, tc::kT, m.tc_b4, st, P);
  } else {
    LAUNCH(KID_BWD_GRADS, k_bwd_grads, dim3(P.nch, P.N), m.b3, st, P);
  }
  if (P.e > 1 && P.dbuf_out) {
    LAUNCH(KID_BWD_BUFOUT, k_bwd_bufout, dim3(P.e - 1, P.N), m.bufout, st, P);
  }
  if (tc_groups(s) & 8)
    LAUNCH_T(KID_BWD_FINAL_TC, tc::k_bwd_finalize_tc, dim3((P.T + tc::kR - 1) / tc::kR, P.N), tc::kT,
             2 * (size_t)tc::kTileBytes, st, P);
  else
  LAUNCH(KID_BWD_FINAL, k_bwd_finalize, dim3((P.T + kFinTile - 1) / kFinTile, P.N), m.fin, st, P);
  if (P.dSref) {
    if (tc_groups(s) & 8) {
      // about two CTAs per SM over (token segment, unit)
      const int ntiles = (P.T + tc::kR - 1) / tc::kR;
      const int segs = std::max(1, std::min(ntiles, (2 * 148 + P.N - 1) / P.N));
      const int per = (ntiles + segs - 1) / segs;
      if (cudaMemsetAsync(P.dSref, 0, (size_t)P.N * P.dv * P.dphi * sizeof(float), st) != cudaSuccess)
        return ATLAS_ERR_LAUNCH;
      LAUNCH_T(KID_BWD_DSREF_TC, tc::k_bwd_dsref_tc, dim3((ntiles + per - 1) / per, P.N), tc::kT,
               2 * (size_t)tc::kTileBytes, st, P, per);
    } else {
      const int tiles = ((P.dv + 63) / 64) * ((P.dphi + 63) / 64);
      LAUNCH(KID_BWD_DSREF, k_bwd_dsref, dim3(tiles, P.N), m.dsref, st, P);
    }
  }
  if (P.fmode == ATLAS_FMAP_TENSOR && (P.dk_ || P.dq_)) {
    if (fmap_tc(s))
      LAUNCH_T(KID_FMAP_BWD_TC, tc::k_fmap_bwd_tc, dim3((P.T + tc::kR - 1) / tc::kR, P.N, 2), tc::kFmT,
               tc::fm_bwd_smem(P.dk, P.dphi), st, P);
    else
      LAUNCH(KID_FMAP_BWD, k_fmap_tensor_bwd, dim3((P.T + kFmTile - 1) / kFmTile, P.N, 2), m.fmb, st, P);
  }
  return ATLAS_OK;
}

// ---- fixed device scratch for atlas_mem_forward_noalloc ---------------------
// Forward workspace for callers that cannot allocate. It is a file-scope
// device array, so every GPU that loads this library holds it until exit.
constexpr size_t kNoAllocScratchBytes = (size_t)32 << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the array on the current device. Host code cannot use the
// symbol itself (it names a host-side stand-in), so the address is looked up
// with that device current. It is looked up on every call rather than cached:
// after a context reset the module is loaded again and the array can move.
// The first lookup on a device loads the module there, which is not allowed
// while a stream is being captured; that case gets its own error code.
int noalloc_scratch(cudaStream_t st, void** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
    (void)cudaGetLastError();
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
      return ATLAS_ERR_NOALLOC_CAPTURE;
    return ATLAS_ERR_LAUNCH;
  }
  *out = p;
  return ATLAS_OK;
}

// ---- TMA descriptors of the bf16 row operands (tensor-core kernels) ----------
PFN_cuTensorMapEncodeTiled_v12000 tma_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// A bf16 [N, T, 128] row-major array as the 4-D view (8 elements, T rows, 16
// column blocks, N units): a box {8, 8, 16, 1} is one 8-row group of a tile in
// the core-matrix layout, and rows outside [0, T) of a unit read as zeros.
int encode_rows(CUtensorMap* m, const void* base, int64_t N, int64_t T) {
  if (!base) return ATLAS_OK;
  if (reinterpret_cast<uintptr_t>(base) % 16) return ATLAS_ERR_INVALID_ARG;
  PFN_cuTensorMapEncodeTiled_v12000 enc = tma_encoder();
  if (!enc) return ATLAS_ERR_LAUNCH;
  const cuuint64_t dims[4] = {8, (cuuint64_t)T, (cuuint64_t)(tc::kD / 8), (cuuint64_t)N};
  const cuuint64_t strides[3] = {(cuuint64_t)tc::kD * 2, 16, (cuuint64_t)T * tc::kD * 2};
  const cuuint32_t box[4] = {8, 8, (cuuint32_t)(tc::kD / 8), 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ATLAS_OK : ATLAS_ERR_LAUNCH;
}

// Descriptors for the operands the tensor-core kernels load by TMA.
int encode_tma(Params& P, const AtlasMemShape* s) {
  if (!tc_groups(s)) return ATLAS_OK;
  int v;
  if (P.fmode != ATLAS_FMAP_TENSOR) {
    if ((v = encode_rows(&P.tm_q, P.q, P.N, P.T))) return v;
    if ((v = encode_rows(&P.tm_k, P.k, P.N, P.T))) return v;
  }
  if ((v = encode_rows(&P.tm_dy, P.dy, P.N, P.T))) return v;
  if ((v = encode_rows(&P.tm_dl, P.dlb, P.N, P.T))) return v;
  return ATLAS_OK;
}

int check_ws(const Layout& L, const void* saved, size_t saved_bytes, const void* scratch, size_t scratch_bytes,
             bool need_scratch) {
  if (!saved || saved_bytes < L.saved) return ATLAS_ERR_WORKSPACE;
  if (need_scratch && (!scratch || scratch_bytes < L.bwd)) return ATLAS_ERR_WORKSPACE;
  return ATLAS_OK;
}

}  // namespace

// ---- q/k/v depthwise convolutions (dwconv.cuh) ----
template <int K, class X, class Y>
int dwconv_fwd_t(const void* x, const float* wq, const float* wk, const float* wv, void* yq, void* yk, void* yv,
                 int64_t B, int64_t T, int64_t C, cudaStream_t st) {
  const dim3 grid((unsigned)((C + kConvThreads - 1) / kConvThreads), (unsigned)((T + kConvRun - 1) / kConvRun),
                  (unsigned)B);
  LAUNCH_T(KID_DWCONV_FWD, (k_dwconv3_fwd<K, X, Y>), grid, kConvThreads, 0, st, (const X*)x, wq, wk, wv, (Y*)yq,
           (Y*)yk, (Y*)yv, T, C);
  return ATLAS_OK;
}
template <int K, class X, class Y>
int dwconv_bwd_t(const void* x, const float* wq, const float* wk, const float* wv, const void* dq, const void* dk,
                 const void* dv, void* dx, float* dw, int64_t B, int64_t T, int64_t C, cudaStream_t st) {
  const dim3 grid((unsigned)((C + kConvThreads - 1) / kConvThreads), (unsigned)((T + kConvRun - 1) / kConvRun),
                  (unsigned)B);
  LAUNCH_T(KID_DWCONV_BWD, (k_dwconv3_bwd<K, X, Y>), grid, kConvThreads, 0, st, (const X*)x, wq, wk, wv,
           (const Y*)dq, (const Y*)dk, (const Y*)dv, (X*)dx, dw, T, C);
  return ATLAS_OK;
}
template <class X, class Y>
int dwconv_dispatch(bool fwd, int K, const void* x, const float* wq, const float* wk, const float* wv, void* a,
                    void* b, void* c, const void* dq, const void* dk, const void* dv, float* dw, int64_t B,
                    int64_t T, int64_t C, cudaStream_t st) {
#define ATLAS_DWCONV_CASE(KK)                                                                   \
  case KK:                                                                                      \
    return fwd ? dwconv_fwd_t<KK, X, Y>(x, wq, wk, wv, a, b, c, B, T, C, st)                    \
               : dwconv_bwd_t<KK, X, Y>(x, wq, wk, wv, dq, dk, dv, a, dw, B, T, C, st);
  switch (K) {
    ATLAS_DWCONV_CASE(2)
    ATLAS_DWCONV_CASE(3)
    ATLAS_DWCONV_CASE(4)
    ATLAS_DWCONV_CASE(5)
    ATLAS_DWCONV_CASE(6)
    ATLAS_DWCONV_CASE(7)
    ATLAS_DWCONV_CASE(8)
    default:
      return ATLAS_ERR_INVALID_ARG;
  }
#undef ATLAS_DWCONV_CASE
}
int dwconv_types(bool fwd, int K, int dtype_x, int dtype_y, const void* x, const float* wq, const float* wk,
                 const float* wv, void* a, void* b, void* c, const void* dq, const void* dk, const void* dv,
                 float* dw, int64_t B, int64_t T, int64_t C, cudaStream_t st) {
  const bool xb = dtype_x == ATLAS_BF16, yb = dtype_y == ATLAS_BF16;
  if (xb && yb) return dwconv_dispatch<__nv_bfloat16, __nv_bfloat16>(fwd, K, x, wq, wk, wv, a, b, c, dq, dk, dv, dw, B, T, C, st);
  if (xb) return dwconv_dispatch<__nv_bfloat16, float>(fwd, K, x, wq, wk, wv, a, b, c, dq, dk, dv, dw, B, T, C, st);
  if (yb) return dwconv_dispatch<float, __nv_bfloat16>(fwd, K, x, wq, wk, wv, a, b, c, dq, dk, dv, dw, B, T, C, st);
  return dwconv_dispatch<float, float>(fwd, K, x, wq, wk, wv, a, b, c, dq, dk, dv, dw, B, T, C, st);
}
bool dtype_ok(int d) { return d == ATLAS_F32 || d == ATLAS_BF16; }

// ---- head preparation (headprep.cuh) ----
template <int PER, class I, class O>
int head_prep_t(bool fwd, const void* t, const float* gamma, void* o, const void* g, void* dt, float* dgamma,
                int64_t B, int64_t T, int H, int Dp, cudaStream_t st) {
  const int64_t BT = B * T;
  const dim3 grid((unsigned)H, (unsigned)((BT + kHpRows - 1) / kHpRows));
  if (fwd)
    LAUNCH_T(KID_HEADPREP_FWD, (k_head_prep_fwd<PER, I, O>), grid, kHpWarps * 32, 0, st, (const I*)t, gamma, (O*)o,
             BT, T, H, Dp);
  else
    LAUNCH_T(KID_HEADPREP_BWD, (k_head_prep_bwd<PER, I, O>), grid, kHpWarps * 32, 0, st, (const I*)t, gamma,
             (const O*)g, (I*)dt, dgamma, BT, T, H, Dp);
  return ATLAS_OK;
}
template <class I, class O>
int head_prep_d(bool fwd, int d, const void* t, const float* gamma, void* o, const void* g, void* dt, float* dgamma,
                int64_t B, int64_t T, int H, int Dp, cudaStream_t st) {
  switch (d) {
    case 32: return head_prep_t<1, I, O>(fwd, t, gamma, o, g, dt, dgamma, B, T, H, Dp, st);
    case 64: return head_prep_t<2, I, O>(fwd, t, gamma, o, g, dt, dgamma, B, T, H, Dp, st);
    case 96: return head_prep_t<3, I, O>(fwd, t, gamma, o, g, dt, dgamma, B, T, H, Dp, st);
    case 128: return head_prep_t<4, I, O>(fwd, t, gamma, o, g, dt, dgamma, B, T, H, Dp, st);
    default: return ATLAS_ERR_INVALID_ARG;
  }
}
int head_prep(bool fwd, int dtype_in, int dtype_out, int d, const void* t, const float* gamma, void* o,
              const void* g, void* dt, float* dgamma, int64_t B, int64_t T, int H, int Dp, cudaStream_t st) {
  const bool ib = dtype_in == ATLAS_BF16, ob = dtype_out == ATLAS_BF16;
  if (ib && ob) return head_prep_d<__nv_bfloat16, __nv_bfloat16>(fwd, d, t, gamma, o, g, dt, dgamma, B, T, H, Dp, st);
  if (ib) return head_prep_d<__nv_bfloat16, float>(fwd, d, t, gamma, o, g, dt, dgamma, B, T, H, Dp, st);
  if (ob) return head_prep_d<float, __nv_bfloat16>(fwd, d, t, gamma, o, g, dt, dgamma, B, T, H, Dp, st);
  return head_prep_d<float, float>(fwd, d, t, gamma, o, g, dt, dgamma, B, T, H, Dp, st);
}

// A barrier nothing arrives on, waited on through the tensor-core kernels'
// bounded wait-and-report path (atlas_mem_selftest_wait_timeout).
__global__ void __launch_bounds__(tc::kT) k_wait_timeout_selftest(int* status, int polls) {
  __shared__ uint64_t mbar;
  if (threadIdx.x == 0) umma::mbar_init(&mbar, 1);
  umma::fence_before();
  __syncthreads();
  tc::Sync sy{&mbar, nullptr, 0, status};
  (void)tc::sync_wait(sy, polls);
}

extern "C" {

int atlas_mem_abi_version(void) { return ATLAS_MEM_ABI_VERSION; }

const char* atlas_mem_error_string(int code) {
  switch (code) {
    case ATLAS_OK: return "ok";
    case ATLAS_ERR_INVALID_ARG: return "invalid argument (null pointer, bad enum or inconsistent sizes)";
    case ATLAS_ERR_UNSUPPORTED: return "unsupported shape (head size > 256, window too large, or shared memory)";
    case ATLAS_ERR_WORKSPACE: return "workspace missing or smaller than atlas_mem_workspace_size()";
    case ATLAS_ERR_LAUNCH: return "CUDA kernel launch failed";
    case ATLAS_ERR_DEVICE: return "device-side status reported a fault";
    case ATLAS_ERR_NOALLOC_TOO_LARGE:
      return "shape needs more scratch than the fixed no-alloc array holds (see atlas_mem_noalloc_scratch_bytes)";
    case ATLAS_ERR_NOALLOC_CAPTURE:
      return "no-alloc scratch lookup failed during stream capture: make the first no-alloc call on this "
             "device before capturing";
    default: return "unknown error";
  }
}

int atlas_mem_workspace_size(const AtlasMemShape* shape, size_t* saved, size_t* fwd_scratch, size_t* bwd_scratch) {
  const int v = validate_shape(shape);
  if (v) return v;
  const Layout L = make_layout(shape);
  if (saved) *saved = L.saved;
  if (fwd_scratch) *fwd_scratch = L.fwd;
  if (bwd_scratch) *bwd_scratch = L.bwd;
  return ATLAS_OK;
}

int atlas_mem_forward(const AtlasMemShape* shape, const AtlasMemFwd* fwd, void* saved, size_t saved_bytes,
                      void* scratch, size_t scratch_bytes, void* stream) {
  (void)scratch; (void)scratch_bytes;
  int v = validate_shape(shape);
  if (!v) v = validate_fwd(shape, fwd, true);
  if (v) return v;
  const Layout L = make_layout(shape);
  if ((v = check_ws(L, saved, saved_bytes, nullptr, 0, false))) return v;
  if ((v = ensure_attrs())) return v;
  Params P = make_params(shape, L, fwd, nullptr, saved, nullptr);
  if (int te = encode_tma(P, shape)) return te;
  cudaStream_t st = (cudaStream_t)stream;
  if ((v = run_fwd_local(shape, P, st))) return v;
  return run_fwd_finish(shape, P, st);
}

int atlas_mem_forward_noalloc(const AtlasMemShape* shape, const AtlasMemFwd* fwd, void* stream) {
  int v = validate_shape(shape);
  if (!v) v = validate_fwd(shape, fwd, true);
  if (v) return v;
  const Layout L = make_layout(shape);
  if (L.saved > kNoAllocScratchBytes) return ATLAS_ERR_NOALLOC_TOO_LARGE;
  void* scratch = nullptr;
  if ((v = noalloc_scratch((cudaStream_t)stream, &scratch))) return v;
  if ((v = ensure_attrs())) return v;
  // Every scratch word the forward reads is written earlier in the same call,
  // so nothing has to be cleared between calls.
  Params P = make_params(shape, L, fwd, nullptr, scratch, nullptr);
  if (int te = encode_tma(P, shape)) return te;
  cudaStream_t st = (cudaStream_t)stream;
  if ((v = run_fwd_local(shape, P, st))) return v;
  return run_fwd_finish(shape, P, st);
}

int atlas_mem_final_state_raw(const AtlasMemShape* shape, const void* saved, size_t saved_bytes, float* out,
                              void* stream) {
  int v = validate_shape(shape);
  if (v) return v;
  if (!out) return ATLAS_ERR_INVALID_ARG;
  const Layout L = make_layout(shape);
  if ((v = check_ws(L, saved, saved_bytes, nullptr, 0, false))) return v;
  const size_t bytes = (size_t)shape->N * shape->d_v * shape->d_phi * sizeof(float);
  if (cudaMemcpyAsync(out, (const char*)saved + L.ST, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream) !=
      cudaSuccess)
    return ATLAS_ERR_LAUNCH;
  return ATLAS_OK;
}

size_t atlas_mem_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int atlas_mem_backward(const AtlasMemShape* shape, const AtlasMemFwd* fwd, const AtlasMemBwd* bwd,
                       const void* saved, size_t saved_bytes, void* scratch, size_t scratch_bytes, void* stream) {
  int v = validate_shape(shape);
  if (!v) v = validate_fwd(shape, fwd, false);
  if (v) return v;
  if (!bwd || !bwd->dy) return ATLAS_ERR_INVALID_ARG;
  const Layout L = make_layout(shape);
  if ((v = check_ws(L, saved, saved_bytes, scratch, scratch_bytes, true))) return v;
  if ((v = ensure_attrs())) return v;
  Params P = make_params(shape, L, fwd, bwd, saved, scratch);
  if (int te = encode_tma(P, shape)) return te;
  cudaStream_t st = (cudaStream_t)stream;
  if ((v = run_bwd_local(shape, P, st))) return v;
  return run_bwd_finish(shape, P, st);
}

int atlas_mem_decode_step(const AtlasMemShape* shape, const AtlasMemFwd* fwd, void* stream) {
  int v;
  if ((v = validate_shape(shape))) return v;
  if (shape->T != 1 || shape->fmap_mode == ATLAS_FMAP_TENSOR || shape->d_phi > 256 || shape->d_v > 256)
    return ATLAS_ERR_UNSUPPORTED;
  if ((v = validate_fwd(shape, fwd, true))) return v;
  if (shape->window > 1 && (!fwd->buf_out || fwd->buf_out == fwd->buf_in)) return ATLAS_ERR_INVALID_ARG;
  const Layout L = make_layout(shape);
  Params P = make_params(shape, L, fwd, nullptr, nullptr, nullptr);
  if (int te = encode_tma(P, shape)) return te;
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((unsigned)((shape->d_v + kDecodeRows - 1) / kDecodeRows), (unsigned)shape->N);
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = shape->d_phi % 4 == 0 && al16(fwd->S_ref) && al16(fwd->S0) && al16(fwd->S_end) &&
                   (!fwd->Z0 || al16(fwd->Z0)) && (!fwd->Z_end || al16(fwd->Z_end)) &&
                   (!fwd->buf_in || al16(fwd->buf_in)) && (!fwd->buf_out || al16(fwd->buf_out));
  if (vec) LAUNCH(KID_DECODE, k_decode_step4, grid, 0, st, P);
  else LAUNCH(KID_DECODE, k_decode_step, grid, 0, st, P);
  return ATLAS_OK;
}

int atlas_scan_forward(const float* gates, const void* inputs, const float* prev, void* out, int64_t B, int64_t T,
                       int64_t D, int dtype_io, int remove_prev, void* stream) {
  if (!gates || !inputs || !out || B < 1 || T < 1 || D < 1) return ATLAS_ERR_INVALID_ARG;
  if (dtype_io != ATLAS_F32 && dtype_io != ATLAS_BF16) return ATLAS_ERR_INVALID_ARG;
  const int off = (prev && !remove_prev) ? 1 : 0;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned gx = (unsigned)((D + kScanOpThreads - 1) / kScanOpThreads);
  for (int64_t b0 = 0; b0 < B; b0 += 65535) {
    const dim3 grid(gx, (unsigned)std::min<int64_t>(65535, B - b0));
    if (dtype_io == ATLAS_F32)
      LAUNCH_T(KID_SCAN_OP_FWD, k_scan_op_fwd<float>, grid, kScanOpThreads, 0, st, gates, (const float*)inputs, prev,
               (float*)out, T, D, off, b0);
    else
      LAUNCH_T(KID_SCAN_OP_FWD, k_scan_op_fwd<__nv_bfloat16>, grid, kScanOpThreads, 0, st, gates,
               (const __nv_bfloat16*)inputs, prev, (__nv_bfloat16*)out, T, D, off, b0);
  }
  return ATLAS_OK;
}

int atlas_omega_store_forward(const float* beta, const void* surprise, const float* last_momentum, const float* gate,
                              const float* buf_in, const float* keep, const float* last_update, void* out,
                              float* momentum_all, float* momentum_last, float* buf_out, int64_t B, int64_t T,
                              int64_t D, int window, int dtype_io, void* stream) {
  if (!surprise || !keep || !out || B < 1 || T < 1 || D < 1 || window < 1) return ATLAS_ERR_INVALID_ARG;
  if (dtype_io != ATLAS_F32 && dtype_io != ATLAS_BF16) return ATLAS_ERR_INVALID_ARG;
  if (window > kOmegaMaxWindow || B > 65535) return ATLAS_ERR_UNSUPPORTED;
  if (window > 1 && !buf_out) return ATLAS_ERR_INVALID_ARG;
  OmegaStoreArgs A{};
  A.beta = beta; A.u = gate; A.a = keep; A.s = surprise; A.m0 = last_momentum; A.buf = window > 1 ? buf_in : nullptr;
  A.h0 = last_update; A.out = out; A.m_all = beta ? momentum_all : nullptr; A.m_last = momentum_last;
  A.buf_out = window > 1 ? buf_out : nullptr; A.B = B; A.T = T; A.D = D; A.e = window; A.off = last_update ? 1 : 0;
  const dim3 grid((unsigned)((D + kScanOpThreads - 1) / kScanOpThreads), (unsigned)B);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype_io == ATLAS_F32) LAUNCH_T(KID_OMEGA_STORE_FWD, k_omega_store_fwd<float>, grid, kScanOpThreads, 0, st, A);
  else LAUNCH_T(KID_OMEGA_STORE_FWD, k_omega_store_fwd<__nv_bfloat16>, grid, kScanOpThreads, 0, st, A);
  return ATLAS_OK;
}

int atlas_omega_store_backward(const float* beta, const void* surprise, const float* last_momentum, const float* gate,
                               const float* keep, const float* last_update, const void* out,
                               const float* momentum_all, const void* d_out, const float* d_momentum_last,
                               const float* d_buf_out, void* d_surprise, float* d_beta, float* d_gate, float* d_keep,
                               float* d_last_momentum, float* d_last_update, float* d_buf_in, int64_t B, int64_t T,
                               int64_t D, int window, int dtype_io, void* stream) {
  if (!surprise || !keep || !out || !d_out || !d_surprise || !d_keep || B < 1 || T < 1 || D < 1 || window < 1)
    return ATLAS_ERR_INVALID_ARG;
  if (dtype_io != ATLAS_F32 && dtype_io != ATLAS_BF16) return ATLAS_ERR_INVALID_ARG;
  if (window > kOmegaMaxWindow || B > 65535) return ATLAS_ERR_UNSUPPORTED;
  if ((beta && (!momentum_all || !d_beta)) || (gate && !d_gate)) return ATLAS_ERR_INVALID_ARG;
  OmegaStoreArgs A{};
  A.beta = beta; A.u = gate; A.a = keep; A.s = surprise; A.m0 = last_momentum; A.h0 = last_update; A.out = (void*)out;
  A.m_all = (float*)momentum_all; A.dout = d_out; A.dm_last = d_momentum_last;
  A.dbuf_out = window > 1 ? d_buf_out : nullptr; A.ds = d_surprise; A.dbeta = d_beta; A.du = d_gate; A.da = d_keep;
  A.dm0 = d_last_momentum; A.dh0 = d_last_update; A.dbuf = window > 1 ? d_buf_in : nullptr;
  A.B = B; A.T = T; A.D = D; A.e = window; A.off = last_update ? 1 : 0;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t bt = (size_t)B * T * sizeof(float);
  if (cudaMemsetAsync(d_keep, 0, bt, st) != cudaSuccess) return ATLAS_ERR_LAUNCH;
  if (beta && cudaMemsetAsync(d_beta, 0, bt, st) != cudaSuccess) return ATLAS_ERR_LAUNCH;
  if (gate && cudaMemsetAsync(d_gate, 0, bt, st) != cudaSuccess) return ATLAS_ERR_LAUNCH;
  const dim3 grid((unsigned)((D + kScanOpThreads - 1) / kScanOpThreads), (unsigned)B);
  if (dtype_io == ATLAS_F32) LAUNCH_T(KID_OMEGA_STORE_BWD, k_omega_store_bwd<float>, grid, kScanOpThreads, 0, st, A);
  else LAUNCH_T(KID_OMEGA_STORE_BWD, k_omega_store_bwd<__nv_bfloat16>, grid, kScanOpThreads, 0, st, A);
  return ATLAS_OK;
}

namespace {
int affine_check(const void* a, const void* b, int64_t N, int64_t T, int R, int D) {
  if (!a || !b || N < 1 || T < 1 || R < 1 || D < 1) return ATLAS_ERR_INVALID_ARG;
  if (R % 8 || D % 8 || R > kAffMaxD || D > kAffMaxD || N > 2147483647 || T > 2147483647)
    return ATLAS_ERR_UNSUPPORTED;
  return ATLAS_OK;
}
}  // namespace

int atlas_affine_scan_forward(const float* A, const float* B, const float* prev, float* out, int64_t N, int64_t T,
                              int R, int D, int remove_prev, void* stream) {
  int v = affine_check(A, B, N, T, R, D);
  if (v) return v;
  if (!out) return ATLAS_ERR_INVALID_ARG;
  if ((v = ensure_attrs())) return v;
  const int off = (prev && !remove_prev) ? 1 : 0;
  const size_t smem = (size_t)(D + R) * (D + 4) * sizeof(float);
  LAUNCH_T(KID_AFFINE_FWD, k_affine_scan_fwd, dim3((unsigned)N), kAffThreads, smem, (cudaStream_t)stream, A, B,
           prev, out, (int)T, R, D, off);
  return ATLAS_OK;
}

int atlas_affine_scan_backward(const float* A, const float* prev, const float* out, const float* d_out, float* d_A,
                               float* d_B, float* d_prev, int64_t N, int64_t T, int R, int D, int remove_prev,
                               void* stream) {
  int v = affine_check(A, out, N, T, R, D);
  if (v) return v;
  if (!d_out || !d_A || !d_B) return ATLAS_ERR_INVALID_ARG;
  if ((v = ensure_attrs())) return v;
  const int off = (prev && !remove_prev) ? 1 : 0;
  const size_t smem = (size_t)(D + 2 * R) * (D + 4) * sizeof(float);
  LAUNCH_T(KID_AFFINE_BWD, k_affine_scan_bwd, dim3((unsigned)N), kAffThreads, smem, (cudaStream_t)stream, A, prev,
           out, d_out, d_A, d_B, prev ? d_prev : nullptr, (int)T, R, D, off);
  return ATLAS_OK;
}

int atlas_scan_backward(const float* gates, const void* out, const float* prev, const void* dout, float* d_gates,
                        void* d_inputs, float* d_prev, int64_t B, int64_t T, int64_t D, int dtype_io,
                        int remove_prev, void* stream) {
  if (!gates || !out || !dout || !d_gates || !d_inputs || B < 1 || T < 1 || D < 1) return ATLAS_ERR_INVALID_ARG;
  if (dtype_io != ATLAS_F32 && dtype_io != ATLAS_BF16) return ATLAS_ERR_INVALID_ARG;
  const int off = (prev && !remove_prev) ? 1 : 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(d_gates, 0, (size_t)B * T * sizeof(float), st) != cudaSuccess) return ATLAS_ERR_LAUNCH;
  const unsigned gx = (unsigned)((D + kScanOpThreads - 1) / kScanOpThreads);
  for (int64_t b0 = 0; b0 < B; b0 += 65535) {
    const dim3 grid(gx, (unsigned)std::min<int64_t>(65535, B - b0));
    if (dtype_io == ATLAS_F32)
      LAUNCH_T(KID_SCAN_OP_BWD, k_scan_op_bwd<float>, grid, kScanOpThreads, 0, st, gates, (const float*)out, prev,
               (const float*)dout, d_gates, (float*)d_inputs, d_prev, T, D, off, b0);
    else
      LAUNCH_T(KID_SCAN_OP_BWD, k_scan_op_bwd<__nv_bfloat16>, grid, kScanOpThreads, 0, st, gates,
               (const __nv_bfloat16*)out, prev, (const __nv_bfloat16*)dout, d_gates, (__nv_bfloat16*)d_inputs,
               d_prev, T, D, off, b0);
  }
  return ATLAS_OK;
}

int atlas_mem_compose_carries(const float* seg, int64_t record_len, int world, int rank, int64_t N, int64_t d2,
                              int backward, const float* S0, const float* Z0, const float* S_T, float* in_S,
                              float* in_Z, float* out_S, float* out_S_clamped, float* out_Z, void* stream) {
  const int64_t coef_len = (N * 3 + 3) / 4 * 4;
  if (!seg || world < 1 || rank < 0 || rank >= world || N < 1 || d2 < 1 || record_len < coef_len + 2 * N * d2)
    return ATLAS_ERR_INVALID_ARG;
  CarryArgs A{seg, record_len, coef_len, N * d2, world, rank, (int)N, backward ? 1 : 0, d2,
              S0, Z0, backward ? S_T : nullptr, in_S, in_Z, out_S, backward ? nullptr : out_S_clamped, out_Z};
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t blocks = std::min<int64_t>((A.ND2 + kThreads - 1) / kThreads, (int64_t)sm_count() * 8);
  LAUNCH(KID_CARRY, k_compose_carries, dim3((unsigned)blocks), 0, st, A);
  return ATLAS_OK;
}

int atlas_dwconv3_forward(const void* x, int dtype_x, const float* w_q, const float* w_k, const float* w_v, int K,
                          void* y_q, void* y_k, void* y_v, int dtype_y, int64_t B, int64_t T, int64_t C,
                          void* stream) {
  if (!x || !w_q || !w_k || !w_v || !y_q || !y_k || !y_v || B < 1 || T < 1 || C < 1 || B > 65535 ||
      !dtype_ok(dtype_x) || !dtype_ok(dtype_y) || K < 2 || K > kConvMaxK || (T + kConvRun - 1) / kConvRun > 65535)
    return ATLAS_ERR_INVALID_ARG;
  return dwconv_types(true, K, dtype_x, dtype_y, x, w_q, w_k, w_v, y_q, y_k, y_v, nullptr, nullptr, nullptr,
                      nullptr, B, T, C, (cudaStream_t)stream);
}

int atlas_dwconv3_backward(const void* x, int dtype_x, const float* w_q, const float* w_k, const float* w_v, int K,
                           const void* dy_q, const void* dy_k, const void* dy_v, int dtype_y, void* dx,
                           float* dw, int64_t B, int64_t T, int64_t C, void* stream) {
  if (!x || !w_q || !w_k || !w_v || !dy_q || !dy_k || !dy_v || !dx || !dw || B < 1 || T < 1 || C < 1 ||
      B > 65535 || !dtype_ok(dtype_x) || !dtype_ok(dtype_y) || K < 2 || K > kConvMaxK ||
      (T + kConvRun - 1) / kConvRun > 65535)
    return ATLAS_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(dw, 0, (size_t)3 * C * K * sizeof(float), st) != cudaSuccess) return ATLAS_ERR_LAUNCH;
  return dwconv_types(false, K, dtype_x, dtype_y, x, w_q, w_k, w_v, dx, nullptr, nullptr, dy_q, dy_k, dy_v, dw,
                      B, T, C, st);
}

int atlas_head_prep_forward(const void* t, int dtype_in, const float* gamma, void* out, int dtype_out, int64_t B,
                            int64_t T, int H, int d, int d_out, void* stream) {
  if (!t || !out || B < 1 || T < 1 || H < 1 || H > 65535 || d_out < d || !dtype_ok(dtype_in) ||
      !dtype_ok(dtype_out) || (B * T + kHpRows - 1) / kHpRows > 65535)
    return ATLAS_ERR_INVALID_ARG;
  return head_prep(true, dtype_in, dtype_out, d, t, gamma, out, nullptr, nullptr, nullptr, B, T, H, d_out,
                   (cudaStream_t)stream);
}

int atlas_head_prep_backward(const void* t, int dtype_in, const float* gamma, const void* grad_out, int dtype_out,
                             void* grad_t, float* grad_gamma, int64_t B, int64_t T, int H, int d, int d_out,
                             void* stream) {
  if (!t || !grad_out || !grad_t || B < 1 || T < 1 || H < 1 || H > 65535 || d_out < d || !dtype_ok(dtype_in) ||
      !dtype_ok(dtype_out) || (B * T + kHpRows - 1) / kHpRows > 65535 || (grad_gamma && !gamma))
    return ATLAS_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (grad_gamma && cudaMemsetAsync(grad_gamma, 0, (size_t)H * d * sizeof(float), st) != cudaSuccess)
    return ATLAS_ERR_LAUNCH;
  return head_prep(false, dtype_in, dtype_out, d, t, gamma, nullptr, grad_out, grad_t, grad_gamma, B, T, H, d_out,
                   st);
}

int atlas_mem_forward_local(const AtlasMemShape* shape, const AtlasMemFwd* fwd, void* saved, size_t saved_bytes,
                            void* scratch, size_t scratch_bytes, float* seg_coef, float* seg_dS, float* seg_dZ,
                            void* stream) {
  (void)scratch; (void)scratch_bytes;
  int v = validate_shape(shape);
  if (!v) v = validate_fwd(shape, fwd, false);
  if (v) return v;
  if (shape->window != 1 || !seg_coef || !seg_dS || !seg_dZ) return ATLAS_ERR_INVALID_ARG;
  const Layout L = make_layout(shape);
  if ((v = check_ws(L, saved, saved_bytes, nullptr, 0, false))) return v;
  if ((v = ensure_attrs())) return v;
  Params P = make_params(shape, L, fwd, nullptr, saved, nullptr);
  if (int te = encode_tma(P, shape)) return te;
  P.seg_coef = seg_coef; P.seg_dS = seg_dS; P.seg_dZ = seg_dZ;
  cudaStream_t st = (cudaStream_t)stream;
  if ((v = run_fwd_local(shape, P, st))) return v;
  return launch_scan(true, P, 1, st);
}

int atlas_mem_forward_finish(const AtlasMemShape* shape, const AtlasMemFwd* fwd, void* saved, size_t saved_bytes,
                             void* scratch, size_t scratch_bytes, void* stream) {
  (void)scratch; (void)scratch_bytes;
  int v = validate_shape(shape);
  if (!v) v = validate_fwd(shape, fwd, true);
  if (v) return v;
  if (shape->window != 1) return ATLAS_ERR_INVALID_ARG;
  const Layout L = make_layout(shape);
  if ((v = check_ws(L, saved, saved_bytes, nullptr, 0, false))) return v;
  if ((v = ensure_attrs())) return v;
  Params P = make_params(shape, L, fwd, nullptr, saved, nullptr);
  if (int te = encode_tma(P, shape)) return te;
  return run_fwd_finish(shape, P, (cudaStream_t)stream);
}

int atlas_mem_backward_local(const AtlasMemShape* shape, const AtlasMemFwd* fwd, const AtlasMemBwd* bwd,
                             const void* saved, size_t saved_bytes, void* scratch, size_t scratch_bytes,
                             float* seg_coef, float* seg_dS, float* seg_dZ, void* stream) {
  int v = validate_shape(shape);
  if (!v) v = validate_fwd(shape, fwd, false);
  if (v) return v;
  if (!bwd || !bwd->dy || shape->window != 1 || !seg_coef || !seg_dS || !seg_dZ) return ATLAS_ERR_INVALID_ARG;
  const Layout L = make_layout(shape);
  if ((v = check_ws(L, saved, saved_bytes, scratch, scratch_bytes, true))) return v;
  if ((v = ensure_attrs())) return v;
  Params P = make_params(shape, L, fwd, bwd, saved, scratch);
  if (int te = encode_tma(P, shape)) return te;
  P.seg_coef = seg_coef; P.seg_dS = seg_dS; P.seg_dZ = seg_dZ;
  cudaStream_t st = (cudaStream_t)stream;
  if ((v = run_bwd_local(shape, P, st))) return v;
  return launch_scan(false, P, 1, st);
}

int atlas_mem_backward_finish(const AtlasMemShape* shape, const AtlasMemFwd* fwd, const AtlasMemBwd* bwd,
                              const void* saved, size_t saved_bytes, void* scratch, size_t scratch_bytes,
                              int apply_clamp_mask, void* stream) {
  int v = validate_shape(shape);
  if (!v) v = validate_fwd(shape, fwd, false);
  if (v) return v;
  if (!bwd || !bwd->dy || shape->window != 1) return ATLAS_ERR_INVALID_ARG;
  const Layout L = make_layout(shape);
  if ((v = check_ws(L, saved, saved_bytes, scratch, scratch_bytes, true))) return v;
  if ((v = ensure_attrs())) return v;
  Params P = make_params(shape, L, fwd, bwd, saved, scratch);
  if (int te = encode_tma(P, shape)) return te;
  P.apply_mask = apply_clamp_mask ? 1 : 0;
  return run_bwd_finish(shape, P, (cudaStream_t)stream);
}

int atlas_mem_selftest_umma(const void* A, const void* B, float* D, int N, int K, int a_mn_major,
                            int b_mn_major, int* status, void* stream) {
  if (!A || !B || !D || !status) return ATLAS_ERR_INVALID_ARG;
  if (N < 16 || N > 256 || N % 16 || K < 16 || K > 128 || K % 16) return ATLAS_ERR_UNSUPPORTED;
  // operand tiles plus slack, so every descriptor read stays inside the allocation
  const size_t smem = (size_t)(128 * K + N * K) * 2 + 65536;
  if (cudaFuncSetAttribute((const void*)k_umma_selftest, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return ATLAS_ERR_LAUNCH;
  k_umma_selftest<<<1, 128, smem, (cudaStream_t)stream>>>((const __nv_bfloat16*)A, (const __nv_bfloat16*)B, D, N, K,
                                                          a_mn_major, b_mn_major, status);
  LAUNCH_CHECK();
  return ATLAS_OK;
}

size_t atlas_fmap_tensor_workspace(int d_k, int d_phi) {
  if (!tc::fmap_tc_ok(d_k, d_phi, 1)) return 0;
  return (size_t)(d_k + 1) * tc::fm_chunk_bytes(d_k, d_phi);
}

namespace {
Params fmap_params(int64_t rows, int d_k, int d_phi, const void* x, const float* proj, void* proj_tiles) {
  Params P{};
  P.N = 1; P.T = (int)rows; P.dk = d_k; P.dphi = d_phi; P.bf = 1; P.fmode = ATLAS_FMAP_TENSOR; P.fdeg = 2;
  P.k = x; P.proj = proj; P.projb = (unsigned char*)proj_tiles; P.fm_bf16 = 1;
  return P;
}
}  // namespace

int atlas_fmap_tensor_forward(int64_t rows, int d_k, int d_phi, const void* x, const float* proj, void* proj_tiles,
                              void* phi, int* status, void* stream) {
  if (!x || !proj || !proj_tiles || !phi || rows < 1) return ATLAS_ERR_INVALID_ARG;
  if (!tc::fmap_tc_ok(d_k, d_phi, 1) || rows > ((int64_t)1 << 30)) return ATLAS_ERR_UNSUPPORTED;
  int v;
  if ((v = ensure_attrs())) return v;
  Params P = fmap_params(rows, d_k, d_phi, x, proj, proj_tiles);
  P.phik = (float*)phi;
  P.status = status;
  cudaStream_t st = (cudaStream_t)stream;
  LAUNCH(KID_PROJ_TILES, tc::k_proj_tiles, dim3(d_k + 1), 0, st, P);
  LAUNCH_T(KID_FMAP_FWD_TC, tc::k_fmap_fwd_tc, dim3((unsigned)((rows + tc::kFmRows - 1) / tc::kFmRows), 1, 1), tc::kFmT,
           tc::fm_fwd_smem(d_k, d_phi), st, P);
  return ATLAS_OK;
}

int atlas_fmap_tensor_backward(int64_t rows, int d_k, int d_phi, const void* x, const void* proj_tiles,
                               const void* dphi, void* dx, int* status, void* stream) {
  if (!x || !proj_tiles || !dphi || !dx || rows < 1) return ATLAS_ERR_INVALID_ARG;
  if (!tc::fmap_tc_ok(d_k, d_phi, 1) || rows > ((int64_t)1 << 30)) return ATLAS_ERR_UNSUPPORTED;
  int v;
  if ((v = ensure_attrs())) return v;
  Params P = fmap_params(rows, d_k, d_phi, x, nullptr, const_cast<void*>(proj_tiles));
  P.dphiR = (float*)const_cast<void*>(dphi);
  P.dk_ = dx;
  P.status = status;
  LAUNCH_T(KID_FMAP_BWD_TC, tc::k_fmap_bwd_tc, dim3((unsigned)((rows + tc::kR - 1) / tc::kR), 1, 1), tc::kFmT,
           tc::fm_bwd_smem(d_k, d_phi), (cudaStream_t)stream, P);
  return ATLAS_OK;
}

int atlas_mem_read_status(const int* status, void* stream) {
  if (!status) return ATLAS_ERR_INVALID_ARG;
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return ATLAS_ERR_LAUNCH;
  int h = 0;
  if (cudaMemcpy(&h, status, sizeof(int), cudaMemcpyDefault) != cudaSuccess) return ATLAS_ERR_LAUNCH;
  return h ? ATLAS_ERR_DEVICE : ATLAS_OK;
}

int atlas_mem_selftest_wait_timeout(int* status, int polls, void* stream) {
  if (!status || polls < 1 || polls > (1 << 20)) return ATLAS_ERR_INVALID_ARG;
  k_wait_timeout_selftest<<<1, tc::kT, 0, (cudaStream_t)stream>>>(status, polls);
  LAUNCH_CHECK();
  return ATLAS_OK;
}

int atlas_mem_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  if (on && !g_prof.ev_ready) {
    for (int i = 0; i < 2 * kMaxTimed; ++i)
      if (cudaEventCreate(&g_prof.ev[i]) != cudaSuccess) return ATLAS_ERR_LAUNCH;
    g_prof.ev_ready = true;
  }
  if (g_prof.pending) prof_collect_locked();
  g_prof.timing = on != 0;
  g_prof.launches = 0;
  for (int k = 0; k < KID_COUNT; ++k) { g_prof.ms[k] = 0.0; g_prof.cnt[k] = 0; }
  return ATLAS_OK;
}

int atlas_mem_profile_read(int kernel_id, double* total_ms, long long* launches) {
  if (kernel_id < 0 || kernel_id >= KID_COUNT) return ATLAS_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lk(g_prof.mu);
  if (g_prof.pending) prof_collect_locked();
  if (total_ms) *total_ms = g_prof.ms[kernel_id];
  if (launches) *launches = g_prof.cnt[kernel_id];
  return ATLAS_OK;
}

#ifdef ATLAS_PHASE_PROF
// Latency-study build only (not part of the ABI header): copy out, and optionally
// clear, the 64 phase counters of atlas::PhaseClock.
int atlas_mem_phase_read(unsigned long long* out, int reset) {
  cudaDeviceSynchronize();
  if (cudaMemcpyFromSymbol(out, atlas::g_phase, sizeof(unsigned long long) * 64) != cudaSuccess) return ATLAS_ERR_LAUNCH;
  if (reset) {
    static const unsigned long long zero[64] = {};
    if (cudaMemcpyToSymbol(atlas::g_phase, zero, sizeof(zero)) != cudaSuccess) return ATLAS_ERR_LAUNCH;
  }
  return ATLAS_OK;
}
#endif

long long atlas_mem_launch_count(void) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  return g_prof.launches;
}

int atlas_mem_kernel_count(void) { return KID_COUNT; }

const char* atlas_mem_kernel_name(int kernel_id) {
  return (kernel_id >= 0 && kernel_id < KID_COUNT) ? kKernelNames[kernel_id] : "";
}

}  // extern "C"
