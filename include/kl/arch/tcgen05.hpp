#pragma once

// Tensor-memory (TMEM) allocation, tcgen05.mma issue/commit and TMEM -> register loads.
// No counterpart in the reference: kernel_lib/include/kl/config.hpp:8 anticipates these
// instructions but ships none.
//
// CtaGroup = 1: one CTA owns the MMA. CtaGroup = 2: a CTA pair (cluster ranks 2i, 2i+1) computes a
// 256-row tile, each CTA holding 128 rows of A, half of B and 128 TMEM lanes of the accumulator;
// the even CTA issues the MMA.

#include <cstdint>

#include <kl/config.hpp>

namespace kl {

#if defined(__CUDACC__)

// Whole warp; writes the TMEM base address to shared memory at `slot`. ncols: power of 2 in [32, 512].
template <int CtaGroup>
KL_DEVICE void tmem_alloc(uint32_t slot, uint32_t ncols) {
  static_assert(CtaGroup == 1 || CtaGroup == 2);
  if constexpr (CtaGroup == 1)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols)
                 : "memory");
}

template <int CtaGroup>
KL_DEVICE void tmem_relinquish() {
  if constexpr (CtaGroup == 1)
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  else
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int CtaGroup>
KL_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  if constexpr (CtaGroup == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
  else
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

KL_DEVICE void tcgen05_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KL_DEVICE void tcgen05_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, 16-bit inputs (kind::f16: f16 or bf16, fp32 or f16 accumulate).
template <int CtaGroup>
KL_DEVICE void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  if constexpr (CtaGroup == 1)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Same for 8-bit float inputs (kind::f8f6f4; e4m3 / e5m2, fp32 accumulate).
template <int CtaGroup>
KL_DEVICE void umma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  if constexpr (CtaGroup == 1)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Block-scaled 8-bit float inputs (kind::mxf8f6f4.block_scale, one UE8M0 scale per 32 K-elements
// of each row of A and B): D (+)= sum_k (A[m,k] * 2^(sfa[m, k/32] - 127)) * (B[n,k] * 2^(sfb[n,
// k/32] - 127)). sfa_tmem / sfb_tmem are the TMEM columns holding the scales (layout written by
// tmem_cp_32x128b_warpx4); which byte of each 32-bit scale word this MMA uses is the idesc's
// a_sf_id / b_sf_id. With CtaGroup 2 each CTA of the pair holds the scales of its own 128 rows of
// A and of all N rows of B, at the same TMEM columns.
template <int CtaGroup>
KL_DEVICE void umma_mxf8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t sfa_tmem,
                            uint32_t sfb_tmem, uint32_t accumulate) {
  if constexpr (CtaGroup == 1)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// Block-scaled packed fp4 inputs (kind::mxf4.block_scale.block32: e2m1 A and B, two per byte, one
// UE8M0 scale per 32 K-elements, K = 64 per MMA): each MMA reads two consecutive scale bytes of
// every row, the idesc's scale-factor ids (0 or 2) naming the first.
template <int CtaGroup>
KL_DEVICE void umma_mxf4_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t sfa_tmem,
                            uint32_t sfb_tmem, uint32_t accumulate) {
  if constexpr (CtaGroup == 1)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// NVFP4: packed e2m1 with one UE4M3 scale per 16 K-elements (kind::mxf4nvf4.block_scale.block16);
// each MMA (64 elements) reads a whole 32-bit scale word of every row (scale-factor id 0).
template <int CtaGroup>
KL_DEVICE void umma_nvf4_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t sfa_tmem,
                            uint32_t sfb_tmem, uint32_t accumulate) {
  if constexpr (CtaGroup == 1)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
            d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
            d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// Shared memory -> TMEM copy of 32 rows x 128 bits, replicated into all four 32-lane quarters
// (lane q*32 + i, columns [col, col + 4) receive row i). `src_desc` is a no-swizzle K-major
// matrix descriptor of the 32 rows (16 bytes each, 8-row groups 128 bytes apart). Ordered with the
// tcgen05.mma issued after it by the same thread. With CtaGroup 2 the even CTA issues it and each
// CTA of the pair copies from its own shared memory into its own TMEM.
template <int CtaGroup>
KL_DEVICE void tmem_cp_32x128b_warpx4(uint32_t taddr, uint64_t src_desc) {
  if constexpr (CtaGroup == 1)
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc) : "memory");
  else
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc) : "memory");
}

// Arrive once on `bar` (a shared::cluster address) when every tcgen05 operation this thread issued
// so far has completed. With CtaGroup 2 the barrier may be in either CTA of the pair.
template <int CtaGroup>
KL_DEVICE void umma_commit(uint32_t bar) {
  if constexpr (CtaGroup == 1)
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 TMEM lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane (taddr.lane + t),
// columns [taddr.col, taddr.col + 32). The warp may only touch its own 32-lane quarter
// (warp_id % 4). Results are valid after tmem_wait_ld().
KL_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 columns.
KL_DEVICE void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

KL_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

#endif  // __CUDACC__

}  // namespace kl
