// sm_100a tensor-core and TMA helpers: tcgen05 (TMEM alloc, MMA, commit, ld)
// and 2-D tensor-map bulk loads into this CTA only.  Descriptor bit layouts follow
// the PTX ISA for tcgen05 shared-memory matrix descriptors and the kind::f16
// instruction descriptor.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace kiv {
namespace tc {

// ---------------------------------------------------------------- TMEM
// Allocate `ncols` TMEM columns (power of two >= 32); the base address is
// written to *dst (shared memory).  Called by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy writes to shared memory -> visible to the async proxy (MMA operands)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------- descriptors
// Shared-memory matrix descriptor, K-major operand stored in the 128-byte
// swizzled layout that a SWIZZLE_128B TMA box of 64 16-bit elements writes:
// rows 128 B apart, 8-row groups 1024 B apart (SBO), 16-byte chunks XOR-ed
// with the row index within the group.  Base must be 1024-byte aligned;
// advancing K by 16 elements inside the 128-byte row adds 32 bytes.
__device__ __forceinline__ uint64_t sdesc_k128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);        // start address, bits [0,14)
  d |= (uint64_t)1 << 16;                              // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                    // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                              // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                              // layout: SWIZZLE_128B
  return d;
}

// The same for the 64-byte swizzled layout a SWIZZLE_64B TMA box of 32
// 16-bit elements writes: rows 64 B apart, 8-row groups 512 B apart (SBO),
// 16-byte chunks XOR-ed with (row / 2) % 4.  Base 512-byte aligned; advancing
// K by 16 elements inside the 64-byte row adds 32 bytes.
__device__ __forceinline__ uint64_t sdesc_k64(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);        // start address, bits [0,14)
  d |= (uint64_t)1 << 16;                              // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(512 >> 4) << 32;                     // stride byte offset: 8 rows x 64 B
  d |= (uint64_t)1 << 46;                              // descriptor version (sm_100)
  d |= (uint64_t)4 << 61;                              // layout: SWIZZLE_64B
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulate, A and B of the same
// 16-bit type (bf16 when `bf16`, else fp16), both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N) {
  return (1u << 4)                                    // D format: f32
         | ((bf16 ? 1u : 0u) << 7)                     // A format
         | ((bf16 ? 1u : 0u) << 10)                    // B format
         | ((uint32_t)(N >> 3) << 17)                  // N / 8
         | ((uint32_t)(M >> 4) << 24);                 // M / 16
}

// D[tmem] (+)= A[smem desc] x B[smem desc]^T, issued by one thread
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// mbarrier arrives once all tcgen05 operations issued so far by this thread complete
__device__ __forceinline__ void commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 columns of 32-bit from TMEM (lane base = 32 * (warp % 4))
__device__ __forceinline__ void ld_32x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ TMA
// 2-D tiled bulk load into this CTA: box at element coordinates (x, y);
// x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t x, int32_t y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// 4-D tiled bulk load into this CTA (x innermost, same alignment rule)
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int32_t x, int32_t y, int32_t z,
                                            int32_t w, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace tc

// host: encode a tiled tensor map (rank 2-5) of a 16-bit store dtype; strides
// in bytes for dimensions 1..rank-1; no interleave, zero fill out of bounds
kiv_status encode_tiled(CUtensorMap *map, int dtype, int rank, const void *base, const uint64_t *dims,
                        const uint64_t *strides, const uint32_t *box, CUtensorMapSwizzle swizzle);

}  // namespace kiv
