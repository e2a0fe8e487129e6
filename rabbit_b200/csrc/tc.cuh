// tc.cuh -- sm_100a tensor-core primitives: TMEM allocation, tcgen05 block-scaled MMA
// (kind::mxf4, E2M1 x E2M1 with E8M0 scales per 32 elements), TMEM loads/stores, and 2-D TMA
// tensor loads into 128-byte-swizzled shared memory. Inline PTX only; no cluster multicast.
//
// Layouts used by every kernel here (from the tcgen05 descriptor formats):
//  * Operand tiles in shared memory are K-major with the 128-byte swizzle: row r of a tile sits at
//    byte 128 * r (groups of 8 rows = 1024 B, the tile base 1024-aligned) and its 16-byte chunk c
//    at chunk position c ^ (r & 7). One row holds 128 bytes = 256 E2M1 values of K. A 2-D TMA
//    load with CU_TENSOR_MAP_SWIZZLE_128B and a 128-byte inner box writes exactly this.
//  * Scale factors live in TMEM. For an operand with rows m (M rows of A, or N rows of B), the
//    four E8M0 bytes of k-blocks 4g..4g+3 of row m are one 32-bit word at TMEM lane (m % 32) +
//    32 q for every sub-partition q (replicated), column base + 4 g + m / 32 (rows < 128). An
//    MMA consuming k-blocks 2s, 2s+1 of that group is given column base + 4 g and byte 2 (s % 2)
//    in address bits 31:30.
#pragma once

#include <stdint.h>

#include "pipe.cuh"

namespace rmoe {

// ---- TMEM allocation (one full warp) ----
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrives (once) on `bar` when every tcgen05 operation issued so far by this thread completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Completion of every tcgen05 operation this thread issued (MMAs, scale-factor copies) before
// the CTA frees its TMEM: on a run that stopped early (a bounded wait ran out) no consumer waited
// for the last ones. `bar` is a one-use mbarrier (count 1); the wait is bounded too.
__device__ __forceinline__ void tc_drain(uint64_t* bar, unsigned* err) {
  tc_commit(bar);
  mbar_wait_bounded(bar, 0, err, 0x400000u);
}

// ---- shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart ----
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;        // start address
  d |= 1ull << 16;                     // leading byte offset (unused for swizzled K-major)
  d |= (1024ull >> 4) << 32;           // stride byte offset: next group of 8 rows
  d |= 1ull << 46;                     // descriptor version (sm_100)
  d |= 2ull << 61;                     // SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::mxf4 (E2M1 x E2M1, E8M0 scales, f32 accumulate), M = 128,
// K-major A and B; the scale-factor byte ids are filled per MMA.
__host__ __device__ constexpr uint32_t mxf4_idesc(int n) {
  return (1u << 7)                          // A format E2M1
         | (1u << 10)                       // B format E2M1
         | (static_cast<uint32_t>(n >> 3) << 17)  // N / 8
         | (1u << 23)                       // scale format UE8M0
         | (static_cast<uint32_t>(128 >> 4) << 24);  // M / 16
}

// Same, with the instruction descriptor already carrying the scale-factor byte ids and no
// compiler memory barrier, so a run of MMAs issues back to back (the issuing thread's own
// instruction latency, not the tensor core, otherwise bounds the issue rate). Ordering with
// later memory operations comes from the tcgen05.commit that follows the run.
__device__ __forceinline__ void mma_mxf4_run(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t id,
                                             uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(id), "r"(accumulate), "r"(tsfa), "r"(tsfb));
}

// D[tmem_d] (+)= A[desc_a] . B[desc_b]^T with per-32 scales from TMEM (block32 = 2 scales per
// row per K = 64 step).
__device__ __forceinline__ void mma_mxf4(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                         uint32_t idesc, uint32_t tsfa, uint32_t tsfb,
                                         uint32_t accumulate) {
  const uint32_t id = idesc | (((tsfa >> 30) & 3u) << 29) | (((tsfb >> 30) & 3u) << 4);
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(id), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// ---- shared memory -> TMEM copies (asynchronous, in issue order with this thread's MMAs) ----
// Source: 32 rows x 16 bytes, rows contiguous (8-row core matrices 128 B apart, no swizzle).
__device__ __forceinline__ uint64_t rows16_desc(const void* src) {
  const uint64_t addr = smem_u32(src);
  return ((addr >> 4) & 0x3FFFull) | ((128ull >> 4) << 32) | (1ull << 46);
}
// Row r of the source lands in TMEM lane r of every sub-partition (r, r + 32, r + 64, r + 96),
// its four 32-bit words in columns taddr .. taddr + 3.
__device__ __forceinline__ void tmem_cp_rows16_x4(uint32_t taddr, uint64_t desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc) : "memory");
}

// ---- TMEM <-> registers (a warp accesses the 32 lanes of its sub-partition) ----
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(a), "r"(b),
               "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive columns of this warp's 32 lanes (one wait for all of them).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// ---- 2-D TMA tile load (no multicast) completing transaction bytes on `bar` ----
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

}  // namespace rmoe
