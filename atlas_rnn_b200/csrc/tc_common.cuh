// Shared pieces of the tensor-core (tcgen05) chunk kernels.
//
// Every tensor-core chunk kernel runs kWG warpgroups of 128 threads. Warp w
// reaches TMEM lanes [32 (w % 4), 32 (w % 4) + 32), so thread t owns row
// t % 128 of every 128-row accumulator, and the warpgroups split its columns
// (warpgroup g takes the 16-column groups [g kCPW, (g + 1) kCPW)).
// Operand tiles are 128 rows x D columns of bf16 in the core-matrix layout of
// umma.cuh (rows past the valid range are zero). d_phi = d_v = D = 128.
#pragma once
#include <cuda_bf16.h>

#include "chunk_kernels.cuh"
#include "umma.cuh"

namespace atlas {
namespace tc {

constexpr int kWG = 4;         // warpgroups per CTA
constexpr int kT = 128 * kWG;  // threads per CTA
constexpr int kR = 128;        // rows of a tile / TMEM lanes
constexpr int kCPW = 8 / kWG;  // 16-column groups of a 128-column accumulator per warpgroup
constexpr int kD = 128;        // head size handled by the tensor-core path
constexpr int kTileBytes = kR * kD * 2;

__device__ __forceinline__ int row_of() { return threadIdx.x & (kR - 1); }  // accumulator row of this thread
__device__ __forceinline__ int wg_of() { return threadIdx.x >> 7; }          // warpgroup: column half

struct Op {
  uint32_t saddr;  // shared address of the tile
  int C;           // contiguous extent of the tile (columns)
  int mn;          // 0: K-major use (K = columns), 1: MN-major use (K = rows)
};
__device__ __forceinline__ Op op(const void* tile, int C, int mn) { return Op{umma::smem_u32(tile), C, mn}; }

// D[tmem] (+)= A * B over `ksteps` K-steps of 16; issued by the calling thread.
__device__ __forceinline__ void mma_chain(uint32_t d_tmem, Op A, Op B, int ksteps, int N, bool acc_first) {
  const uint32_t idesc = umma::make_idesc(128, N, A.mn, B.mn);
  for (int s = 0; s < ksteps; ++s) {
    const uint64_t ad = A.mn ? umma::desc_mnmajor(A.saddr, A.C, s) : umma::desc_kmajor(A.saddr, A.C, s);
    const uint64_t bd = B.mn ? umma::desc_mnmajor(B.saddr, B.C, s) : umma::desc_kmajor(B.saddr, B.C, s);
    umma::mma(d_tmem, ad, bd, idesc, (s > 0 || acc_first) ? 1 : 0);
  }
}

// Per-CTA tensor-core state: TMEM base, one mbarrier and its phase, a status word.
// Code a kernel writes to the caller's status word when a bounded wait ran out.
constexpr int kDevStatMmaTimeout = 1;

struct Sync {
  uint64_t* mbar;
  uint32_t* tbase;
  uint32_t phase;
  int* status;
};

// Allocate `ncols` TMEM columns (kernels using at most 256 can run two CTAs
// per SM) and init the barrier (all threads call).
__device__ __forceinline__ uint32_t tc_setup(Sync& s, uint32_t ncols = 512) {
  if (threadIdx.x < 32) {
    umma::tmem_alloc(s.tbase, ncols);
    umma::tmem_relinquish();
  }
  if (threadIdx.x == 0) umma::mbar_init(s.mbar, 1);
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  s.phase = 0;
  return *s.tbase;
}

// Make this thread's generic smem writes visible to the tensor core and sync.
__device__ __forceinline__ void smem_to_tc() {
  umma::fence_async_smem();
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
}

// Bounded wait of every thread of the CTA on the barrier's current phase.
// Returns true (the same value in every thread) when the phase completed.
// When any thread's wait ran out, thread 0 records kDevStatMmaTimeout in the
// status word (if one was given), the threads that gave up wait once more,
// again bounded, so that tensor-core work still in flight can drain, and every
// thread gets false: the caller must skip its TMEM reads, release TMEM and
// return. All threads of the CTA must call it at the same point.
__device__ __forceinline__ bool sync_wait(Sync& s, long long polls = (1ll << 22)) {
  const bool ok = umma::mbar_wait(s.mbar, s.phase, polls);
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0 && s.status) atomicExch(s.status, kDevStatMmaTimeout);
    if (!ok) umma::mbar_wait(s.mbar, s.phase, polls);
    return false;
  }
  s.phase ^= 1u;
  umma::fence_after();
  return true;
}

// Thread 0 commits the MMAs issued so far; everybody waits for them (bounded,
// reported as in sync_wait).
__device__ __forceinline__ bool mma_wait(Sync& s) {
  if (threadIdx.x == 0) umma::commit(s.mbar);
  return sync_wait(s);
}

// Release TMEM (all threads call; after the last TMEM access).
__device__ __forceinline__ void tc_teardown(uint32_t tm, uint32_t ncols = 512) {
  umma::fence_before();
  __syncthreads();
  if (threadIdx.x < 32) umma::tmem_dealloc(tm, ncols);
}

// In a tensor-core kernel: wait for the MMAs issued so far; if the bounded
// wait ran out (reported in the status word), let this thread's cp.async
// copies land, release the CTA's `ncols` TMEM columns and leave the kernel.
#define ATLAS_MMA_WAIT_OR_LEAVE(sy, tm, ncols)             \
  do {                                                      \
    if (!mma_wait(sy)) {                                    \
      asm volatile("cp.async.wait_all;\n" ::: "memory");   \
      tc_teardown(tm, ncols);                               \
      return;                                               \
    }                                                       \
  } while (0)

// TMEM address of row (this thread's lane) and column `col`.
__device__ __forceinline__ uint32_t lane_addr(uint32_t tm, int col) {
  return tm + ((uint32_t)(((threadIdx.x >> 5) & 3) * 32) << 16) + (uint32_t)col;
}

// Pack 8 floats to bf16 and store one 16-byte unit of a tile.
__device__ __forceinline__ uint4 pack_unit(const float (&v)[8]) {
  __align__(16) __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return *reinterpret_cast<uint4*>(h);
}
__device__ __forceinline__ void unpack_unit(uint4 u, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store_unit(unsigned char* tile, int r, int cb, int C, const float (&v)[8]) {
  __align__(16) __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(tile + umma::unit_off(r, cb, C)) = *reinterpret_cast<uint4*>(h);
}
__device__ __forceinline__ void load_unit(const unsigned char* tile, int r, int cb, int C, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(tile + umma::unit_off(r, cb, C));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Affine recurrence over the L <= 128 tokens of a chunk on one warp (all 32
// lanes call it): x = x0 before the first step, then x <- a(i) x + b(i) for
// i = 0 .. L-1 (FWD) or i = L-1 .. 0 (!FWD); out(i, x) receives x after step i.
// Each lane composes 4 consecutive steps into one affine map; the lane maps
// are combined by 5 shuffle rounds (prefix of maps), so the chain costs
// O(log) instead of L dependent steps.
template <bool FWD, class FA, class FB, class FO>
__device__ __forceinline__ void warp_affine_scan(int L, float x0, FA fa, FB fb, FO out) {
  const int lane = threadIdx.x & 31;
  float ak[4], bk[4], A = 1.f, B = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int st = 4 * lane + k, i = FWD ? st : L - 1 - st;
    ak[k] = 1.f;
    bk[k] = 0.f;
    if (st < L) {
      ak[k] = fa(i);
      bk[k] = fb(i);
    }
    B = ak[k] * B + bk[k];
    A = ak[k] * A;
  }
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {  // inclusive prefix of the lane maps
    const float Ap = __shfl_up_sync(0xffffffffu, A, off), Bp = __shfl_up_sync(0xffffffffu, B, off);
    if (lane >= off) {
      B = A * Bp + B;
      A = A * Ap;
    }
  }
  float Ae = __shfl_up_sync(0xffffffffu, A, 1), Be = __shfl_up_sync(0xffffffffu, B, 1);
  if (lane == 0) { Ae = 1.f; Be = 0.f; }
  float x = Ae * x0 + Be;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int st = 4 * lane + k, i = FWD ? st : L - 1 - st;
    if (st < L) {
      x = ak[k] * x + bk[k];
      out(i, x);
    }
  }
}

// State-path scalars of the chunk after i tokens (i = 0..L), one warp:
// sS[i] = prod alpha, zZ[i] = prod beta, sZ[i+1] = alpha_i sZ[i] - eta_i zZ[i+1].
__device__ __forceinline__ void fwd_scalars_warp(const Ctx& cx, float* sS, float* sZ, float* zZ) {
  const int L = cx.L;
  if ((threadIdx.x & 31) == 0) { sS[0] = 1.f; sZ[0] = 0.f; zZ[0] = 1.f; }
  warp_affine_scan<true>(L, 1.f, [&](int i) { return cx.al[i]; }, [](int) { return 0.f; },
                         [&](int i, float x) { sS[i + 1] = x; });
  warp_affine_scan<true>(L, 1.f, [&](int i) { return cx.be[i]; }, [](int) { return 0.f; },
                         [&](int i, float x) { zZ[i + 1] = x; });
  __syncwarp();
  warp_affine_scan<true>(L, 0.f, [&](int i) { return cx.al[i]; }, [&](int i) { return -cx.et[i] * zZ[i + 1]; },
                         [&](int i, float x) { sZ[i + 1] = x; });
  __syncwarp();
}
// Adjoint-transform scalars of the chunk from its end down to row r (r = 0..L),
// one warp: hS[r] = alpha_r hS[r+1], hZZ[r] = beta_r hZZ[r+1],
// hZS[r] = beta_r hZS[r+1] - eta_{r-1} hS[r]; hS[L] = hZZ[L] = 1, hZS[L] = -eta_{L-1}.
__device__ __forceinline__ void adj_scalars_warp(const Ctx& cx, float* hS, float* hZS, float* hZZ) {
  const int L = cx.L;
  if ((threadIdx.x & 31) == 0) { hS[L] = 1.f; hZZ[L] = 1.f; hZS[L] = -cx.et[L - 1]; }
  warp_affine_scan<false>(L, 1.f, [&](int r) { return cx.al[r]; }, [](int) { return 0.f; },
                          [&](int r, float x) { hS[r] = x; });
  warp_affine_scan<false>(L, 1.f, [&](int r) { return cx.be[r]; }, [](int) { return 0.f; },
                          [&](int r, float x) { hZZ[r] = x; });
  __syncwarp();
  warp_affine_scan<false>(L, -cx.et[L - 1], [&](int r) { return cx.be[r]; },
                          [&](int r) { return -(r >= 1 ? cx.et[r - 1] : 0.f) * hS[r]; },
                          [&](int r, float x) { hZS[r] = x; });
  __syncwarp();
}

// Zero a tile with the 128 threads of the calling warpgroup.
__device__ __forceinline__ void zero_tile_wg(unsigned char* tile) {
  for (int u = threadIdx.x & 127; u < kTileBytes / 16; u += 128)
    reinterpret_cast<uint4*>(tile)[u] = make_uint4(0u, 0u, 0u, 0u);
}

// Unit u of a 128 x C tile (cpr = C / 8 units per row) in shared-memory address
// order: unit_off(r, cb, C) == 16 u, so consecutive threads touch consecutive
// 16-byte units (no bank conflicts), and a warp covers 8 rows x 4 column blocks
// (64 contiguous bytes of each source row).
__device__ __forceinline__ void unit_rc(int u, int cpr, int& r, int& cb) {
  r = ((u >> 3) / cpr) * 8 + (u & 7);
  cb = (u >> 3) % cpr;
}

// Fill a 128 x C tile; src(r, c0, v) fills v[0..7] for columns c0..c0+7 of row r.
// Units go in shared-memory order (unit_rc) unless rowmajor, which walks the
// source rows in order (for sources that also write global rows back).
// Threads [first, first + count) take part (the others return at once); each
// gathers 8 units before storing any, so 8 loads are in flight per thread.
template <class F>
__device__ __forceinline__ void fill_tile(unsigned char* tile, int C, F src, int first = 0, int count = kT,
                                          bool rowmajor = false) {
  constexpr int kBatch = 8;
  const int me = (int)threadIdx.x - first;
  if (me < 0 || me >= count) return;
  const int cpr = C / 8, units = 128 * cpr;
  for (int base = me; base < units; base += count * kBatch) {
    float v[kBatch][8];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int u = base + k * count;
      int r, cb;
      if (rowmajor) { r = u / cpr; cb = u % cpr; } else { unit_rc(u, cpr, r, cb); }
      if (u < units) src(r, cb * 8, v[k]);
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int u = base + k * count;
      if (u >= units) continue;
      if (rowmajor) store_unit(tile, u / cpr, u % cpr, C, v[k]);
      else *reinterpret_cast<uint4*>(tile + 16 * u) = pack_unit(v[k]);
    }
  }
}
// ---------------------------------------------------------------------------
// Asynchronous tile loads (cp.async, 16 bytes, L2 only). Every thread issues
// its copies without waiting, so a whole tile set is in flight at once; a zero
// unit is a copy of 0 source bytes (the destination is zero-filled). The
// caller ends the set with async_wait() (own copies) and a block barrier, and
// may then rewrite units in place (feature map, row scaling) before the MMA.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp16(void* dst_smem, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(umma::smem_u32(dst_smem)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void async_wait() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  asm volatile("cp.async.wait_all;\n" ::: "memory");
}
// A 32 KB tile already in the core-matrix layout.
__device__ __forceinline__ void async_copy_tile(unsigned char* tile, const unsigned char* src, int first = 0,
                                                int count = kT) {
  const int me = (int)threadIdx.x - first;
  if (me < 0 || me >= count) return;
  for (int u = me; u < kTileBytes / 16; u += count) cp16(tile + 16 * u, src + 16 * u, true);
}
// Rows of a bf16 row-major [*, 128] matrix: rowp(r) is row r or nullptr (zero row).
// `base` is any valid global address (the source operand of a zero-filled copy).
template <class F>
__device__ __forceinline__ void async_rows(unsigned char* tile, F rowp, const void* base, int first = 0,
                                           int count = kT) {
  constexpr int kCpr = kD / 8;
  const int me = (int)threadIdx.x - first;
  if (me < 0 || me >= count) return;
  for (int u = me; u < kTileBytes / 16; u += count) {
    int r, cb;
    unit_rc(u, kCpr, r, cb);
    const __nv_bfloat16* row = rowp(r);
    cp16(tile + 16 * u, row ? static_cast<const void*>(row + cb * 8) : base, row != nullptr);
  }
}
// Rewrite every unit of rows [0, rows) in place: f(r, v[8]) (after the barrier
// that follows async_wait()).
template <class F>
__device__ __forceinline__ void xform_rows(unsigned char* tile, int rows, F f, int first = 0, int count = kT) {
  constexpr int kCpr = kD / 8;
  const int me = (int)threadIdx.x - first;
  if (me < 0 || me >= count) return;
  for (int u = me; u < kR * kCpr; u += count) {
    int r, cb;
    unit_rc(u, kCpr, r, cb);
    if (r >= rows) continue;
    float v[8];
    unpack_unit(*reinterpret_cast<const uint4*>(tile + 16 * u), v);
    f(r, v);
    *reinterpret_cast<uint4*>(tile + 16 * u) = pack_unit(v);
  }
}

// ---------------------------------------------------------------------------
// TMA tile loads. One thread issues them; they complete on a CTA mbarrier with
// a transaction count (expect_tx per tile, one arrive per batch), and every
// thread that reads the tiles waits on the barrier's phase.
//  * rows of a bf16 [N, T, 128] operand: 16 cp.async.bulk.tensor loads of one
//    8-row group each through the 4-D descriptor in Params (rows outside
//    [0, T) of the unit arrive as zeros);
//  * a 32 KB tile already in the core-matrix layout: one cp.async.bulk copy.
// No multicast: every load reads this GPU's memory into this CTA only.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;\n" ::"r"(umma::smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(umma::smem_u32(bar)) : "memory");
}
// 128 rows [row0, row0 + 128) of unit n into `tile` (issuing thread only).
__device__ __forceinline__ void tma_rows(const CUtensorMap* map, unsigned char* tile, int n, int row0,
                                         uint64_t* bar) {
  mbar_expect_tx(bar, kTileBytes);
#pragma unroll 1
  for (int g = 0; g < kR / 8; ++g) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];\n" ::"r"(umma::smem_u32(tile + g * (kTileBytes / 16))),
        "l"(map), "r"(0), "r"(row0 + 8 * g), "r"(0), "r"(n), "r"(umma::smem_u32(bar))
        : "memory");
  }
}
// A 32 KB core-matrix tile from global memory (16-byte aligned) into `tile` (issuing thread only).
__device__ __forceinline__ void tma_tile(unsigned char* tile, const void* src, uint64_t* bar) {
  mbar_expect_tx(bar, kTileBytes);
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          umma::smem_u32(tile)),
      "l"(src), "r"(kTileBytes), "r"(umma::smem_u32(bar))
      : "memory");
}
// Loads in flight on one barrier.
struct TmaBatch {
  uint64_t* bar;
  uint32_t phase;
};
__device__ __forceinline__ void tma_init(TmaBatch& b) {  // one thread, before the CTA barrier of tc_setup
  umma::mbar_init(b.bar, 1);
  b.phase = 0;
}
// The issuing thread closes the batch after its loads.
__device__ __forceinline__ void tma_commit(TmaBatch& b) { mbar_arrive(b.bar); }
// Bounded wait of the calling thread for the batch (every reader calls it). A
// wait that runs out is recorded in the status word and waited once more, so
// that no copy is left in flight into shared memory the CTA gives up.
__device__ __forceinline__ void tma_wait(TmaBatch& b, int* status) {
  if (!umma::mbar_wait(b.bar, b.phase)) {
    if (status) atomicExch(status, kDevStatMmaTimeout);
    umma::mbar_wait(b.bar, b.phase);
  }
  b.phase ^= 1u;
}
// Zero rows [from, 128) of a tile (the rows a 128-row TMA box brings in past the
// chunk's last token); threads [first, first + count).
__device__ __forceinline__ void zero_rows_from(unsigned char* tile, int from, int first = 0, int count = kT) {
  const int me = (int)threadIdx.x - first;
  if (me < 0 || me >= count || from >= kR) return;
  const int units = (kR - from) * (kD / 8);
  for (int x = me; x < units; x += count) {
    const int r = from + x / (kD / 8), cb = x % (kD / 8);
    *reinterpret_cast<uint4*>(tile + umma::unit_off(r, cb, kD)) = make_uint4(0u, 0u, 0u, 0u);
  }
}

// Rows of a 128 x 128 bf16 tile (core-matrix layout) out to global memory:
// dst(r) is the global row of tile row r, or nullptr to skip it. Units go in
// shared-memory order (unit_rc), so the reads are conflict-free and a warp
// writes 8 rows x 64 contiguous bytes -- whole 32-byte sectors, where a
// thread-per-row epilogue writes 16 bytes of 32 different rows per store.
template <class F>
__device__ __forceinline__ void store_rows_from_tile(const unsigned char* tile, F dst) {
  for (int u = threadIdx.x; u < kTileBytes / 16; u += kT) {
    int r, cb;
    unit_rc(u, kD / 8, r, cb);
    __nv_bfloat16* row = dst(r);
    if (row) *reinterpret_cast<uint4*>(row + cb * 8) = reinterpret_cast<const uint4*>(tile)[u];
  }
}
// 16 accumulator values of row r, columns [16 c16, 16 c16 + 16), into a bf16 tile.
__device__ __forceinline__ void stage16(unsigned char* tile, int r, int c16, float (&v)[16]) {
  store_unit(tile, r, 2 * c16, kD, *reinterpret_cast<float(*)[8]>(v));
  store_unit(tile, r, 2 * c16 + 1, kD, *reinterpret_cast<float(*)[8]>(v + 8));
}

__device__ __forceinline__ float bf_at(const unsigned char* tile, int r, int c) {
  return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(tile + umma::elem_off(r, c, kD)));
}

// Warpgroups 2.. load tiles while warpgroups 0 and 1 run coefficient recurrences.
constexpr int kFillFirst = 256, kFillCount = kT - 256;

__device__ __forceinline__ void zero8(float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = 0.f;
}

// 8 io values starting at element `off` (bf16 as one 16-byte load when aligned).
__device__ __forceinline__ void ld8io(const void* p, int64_t off, int bf, float (&v)[8]) {
  if (bf) {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p) + off);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + off);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + off + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}
__device__ __forceinline__ void ld8f(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// phi (keys, !isq) or psi (isq) of token t, columns c0..c0+7.
__device__ __forceinline__ void phi8(const Params& P, int n, int t, int c0, bool isq, float (&v)[8]) {
  const int64_t row = (int64_t)n * P.T + t;
  if (P.fmode == ATLAS_FMAP_TENSOR) {
    ld8f((isq ? P.phiq : P.phik) + row * P.dphi + c0, v);
    return;
  }
  ld8io(isq ? P.q : P.k, row * P.dk + c0, P.bf, v);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = fmap_elem(v[i], P.fmode, P.fdeg);
}

// 16 floats as bf16 to global, 32 bytes.
__device__ __forceinline__ void st16bf(void* dst, const float (&v)[16]) {
  __align__(16) __nv_bfloat162 h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = reinterpret_cast<uint4*>(h)[0];
  d[1] = reinterpret_cast<uint4*>(h)[1];
}

// 16 floats to global (fp32), 64 bytes.
__device__ __forceinline__ void st16f(float* dst, const float (&v)[16]) {
  float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

}  // namespace tc
}  // namespace atlas
