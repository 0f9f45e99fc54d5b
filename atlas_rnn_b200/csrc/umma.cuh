// Thin wrappers over the sm_100a tensor-core instructions (tcgen05.* / mbarrier)
// used by the fused kernels, written as inline PTX.
//
// Shared-memory operand layout ("core-matrix tiled"): a tile of R rows by C
// columns of bf16 (C the contiguous dimension, a multiple of 8) is stored as
// 16-byte units of 8 consecutive columns; unit (r, cb) lives at byte
//     ((r / 8) * (C / 8) + cb) * 128 + (r % 8) * 16.
// With no swizzle this one layout is the canonical UMMA layout for both
//  * a K-major operand (rows = M or N, columns = K): LBO = 128, SBO = C*16,
//    K-step s (16 columns) starts 256*s bytes in;
//  * an MN-major operand (rows = K, columns = M or N): LBO = C*16, SBO = 128,
//    K-step s (16 rows) starts 2*C*16*s bytes in.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace atlas {
namespace umma {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// byte offset of the 16-byte unit (r, cb) in a tile with C columns
__device__ __forceinline__ uint32_t unit_off(int r, int cb, int C) {
  return (uint32_t)(((r >> 3) * (C >> 3) + cb) * 128 + (r & 7) * 16);
}
// byte offset of element (r, c) in the same tile (bf16)
__device__ __forceinline__ uint32_t elem_off(int r, int c, int C) { return unit_off(r, c >> 3, C) + (c & 7) * 2; }

// 64-bit shared-memory matrix descriptor, no swizzle, version 1 (sm_100).
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // version
  // base offset 0, lbo mode 0, layout type 0 (SWIZZLE_NONE)
  return d;
}
// Descriptor of K-step s of a K-major operand stored in a tile with C (= K extent) columns.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile_saddr, int C, int s) {
  return make_desc(tile_saddr + 256u * s, 128u, (uint32_t)C * 16u);
}
// Descriptor of K-step s of an MN-major operand stored in a tile with C (= M/N extent) columns.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile_saddr, int C, int s) {
  return make_desc(tile_saddr + 2u * (uint32_t)C * 16u * s, (uint32_t)C * 16u, 128u);
}

// Instruction descriptor, kind::f16: D f32, A/B bf16, A/B major (0 K, 1 MN), M x N.
__device__ __forceinline__ uint32_t make_idesc(int M, int N, int a_mn, int b_mn) {
  uint32_t d = 0;
  d |= 1u << 4;                 // D format f32
  d |= 1u << 7;                 // A format bf16
  d |= 1u << 10;                // B format bf16
  d |= (uint32_t)(a_mn & 1) << 15;
  d |= (uint32_t)(b_mn & 1) << 16;
  d |= (uint32_t)((N >> 3) & 0x3F) << 17;
  d |= (uint32_t)((M >> 4) & 0x1F) << 24;
  return d;
}

// D[tmem] (+)= A * B, issued by one thread.
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
      :
      : "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued MMAs of this thread complete.
__device__ __forceinline__ void commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n"
               :
               : "r"(smem_u32(mbar))
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" : : "r"(smem_u32(mbar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;\n" : : : "memory");
}

// Bounded wait for the phase with the given parity; returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, long long max_iters = (1ll << 22)) {
  const uint32_t a = smem_u32(mbar);
  for (long long i = 0; i < max_iters; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
// Make generic-proxy shared-memory writes visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// TMEM allocation (one full warp executes these).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n"
               :
               : "r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" : : "r"(taddr), "r"(ncols) : "memory");
}

// Load 16 consecutive fp32 columns of this thread's TMEM lane (32x32b shape):
// warp w of a warpgroup reads lanes [32w, 32w+32); taddr carries lane base in bits 16+.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n"
      :
      : "r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
// One 32-bit column per lane.
__device__ __forceinline__ void tmem_st1(uint32_t taddr, float v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};\n" ::"r"(taddr), "r"(__float_as_uint(v)) : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

}  // namespace umma
}  // namespace atlas
