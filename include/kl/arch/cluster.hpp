#pragma once

// Thread-block-cluster helpers: CTA rank, the hardware cluster barrier, and mapping a shared
// address to the same offset in another CTA of the cluster.
// No counterpart in the reference: kernel_lib ships descriptor encoders only.

#include <cstdint>

#include <kl/config.hpp>

namespace kl {

#if defined(__CUDACC__)

KL_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

KL_DEVICE uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// All threads of every CTA in the cluster must take part (the .aligned forms need whole warps).
KL_DEVICE void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
KL_DEVICE void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
KL_DEVICE void cluster_sync() {
  cluster_arrive();
  cluster_wait();
}

// The shared::cluster address of `smem_addr` (a shared::cta address) in CTA `cta_rank`.
KL_DEVICE uint32_t mapa_shared(uint32_t smem_addr, uint32_t cta_rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(cta_rank));
  return r;
}

// One lane of the (fully active) warp gets true.
KL_DEVICE bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

#endif  // __CUDACC__

}  // namespace kl
