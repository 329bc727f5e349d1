// tcgen05 (5th-generation tensor core) primitives for sm_100a, as inline PTX:
// tensor-memory allocation, shared-memory matrix descriptors, the block-scaled
// NVFP4 MMA (kind::mxf4nvf4, e4m3 scales per 16 elements), scale-factor copies
// into tensor memory, commits to mbarriers, and tensor-memory loads.
//
// Descriptor formats follow the PTX ISA (tcgen05 "shared memory descriptor"
// and "instruction descriptor" tables).
#pragma once
#include <cstdint>

namespace nvfp4 {
namespace tc {

// ---- tensor memory allocation (one full warp executes these) -----------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(dst_smem), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols));
}

// Pair (cta_group::2) forms: one warp in EACH CTA of the pair executes the
// allocation calls.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(dst_smem), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols));
}

// Pair MMA (issued by the leader CTA only): M = 256 split 128/128 over the
// pair's tensor memories, A and B read from both CTAs' shared memory at the
// same offsets, scales from both CTAs' tensor memory at the same columns.
__device__ __forceinline__ void mma_mxf4nvf4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                  uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n}\n"
      :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem));
}

// Arrive once on the mbarrier at the same shared-memory offset in every CTA of
// `cta_mask` when the pair's prior tcgen05 async ops of this thread finish (a
// commit, not a load: no data moves).
__device__ __forceinline__ void commit_pair_both(uint32_t bar, uint16_t cta_mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               :: "r"(bar), "h"(cta_mask) : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- shared-memory matrix descriptor ------------------------------------
// bits 0-13 start>>4, 16-29 leading byte offset>>4, 32-45 stride byte
// offset>>4, 46-47 version (1 on sm_100), 49-51 base offset, 61-63 layout
// (0 none, 2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}

// K-major operand tile written by TMA with 128-byte swizzle: rows of 128
// bytes, 8-row atoms of 1024 bytes.  The tile base must be 1024-aligned;
// the k-th 64-element (32-byte) slice of a row starts 32*k bytes further.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) { return smem_desc(addr, 16, 1024, 2); }

// One 128x4 block of e4m3 scales (512 bytes = 32 rows of 16 bytes, 8-row
// groups 128 bytes apart, no swizzle) as the source of a 32x128b copy.
__device__ __forceinline__ uint64_t desc_sf_block(uint32_t addr) { return smem_desc(addr, 16, 128, 0); }

// ---- instruction descriptor: kind::mxf4nvf4, e2m1 x e2m1, ue4m3 scales ----
// bits 4-5 B scale id, 7-9 A format (e2m1 = 1), 10-12 B format, 15/16 A/B
// major (0 = K), 17-22 N>>3, 23 scale format (0 = ue4m3), 24-28 M>>4,
// 29-30 A scale id, 31 K size (0 = K64).
__host__ __device__ constexpr uint32_t idesc_mxf4nvf4(int M, int N) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D(tmem) (+)= A(smem) . B(smem)^T with per-16 e4m3 scales from tmem.
__device__ __forceinline__ void mma_mxf4nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n}\n"
      :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem));
}

// Copies a 32-row x 16-byte shared-memory block to tensor memory lanes 0-31
// and replicates it to lanes 32-63, 64-95 and 96-127 (4 columns).
__device__ __forceinline__ void cp_sf_32x128b_x4(uint32_t tmem, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" :: "r"(tmem), "l"(sdesc));
}

// Arrive once on an mbarrier when all prior tcgen05 async ops of this thread finish.
__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane
// (32 * (warp % 4) + i) of tensor memory, columns col..col+31.
__device__ __forceinline__ void ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Each thread writes 4 consecutive 32-bit columns of its own lane
// (lane 32 * (warp % 4) + thread).
__device__ __forceinline__ void st_32x32b_x4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};"
               :: "r"(taddr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ void st_32x32b_x2(uint32_t taddr, uint32_t a, uint32_t b) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" :: "r"(taddr), "r"(a), "r"(b) : "memory");
}

__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace tc
}  // namespace nvfp4
