#pragma once

// mbarrier wrappers (shared-memory transaction barriers) with bounded waits.
// No counterpart in the reference: kernel_lib ships descriptor encoders only.
//
// Every wait in kl is bounded: mbarrier_wait() gives up after `timeout_ns` of %globaltimer and
// returns false, so a kernel whose producer died reports an error instead of hanging the GPU.

#include <cstdint>

#include <kl/config.hpp>

namespace kl {

#if defined(__CUDACC__)

KL_DEVICE uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

KL_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

KL_DEVICE void mbarrier_init(uint32_t bar, uint32_t arrivals) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(arrivals) : "memory");
}

// Make barrier initialisation visible to the async proxy (TMA, tcgen05) and to the cluster.
KL_DEVICE void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

KL_DEVICE void mbarrier_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive and add `tx_bytes` to the transaction count the current phase waits for.
KL_DEVICE void mbarrier_arrive_expect_tx(uint32_t bar, uint32_t tx_bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(tx_bytes)
               : "memory");
}

// Arrive on a barrier of another CTA in the cluster (`cluster_bar` comes from mapa_shared).
KL_DEVICE void mbarrier_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// One probe: true once the phase with parity `parity` has completed.
KL_DEVICE bool mbarrier_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase with parity `parity`. Returns false after `timeout_ns`.
KL_DEVICE bool mbarrier_wait(uint32_t bar, uint32_t parity, uint64_t timeout_ns) {
  if (mbarrier_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (mbarrier_try_wait(bar, parity)) return true;
    if ((n & 15u) == 0 && globaltimer_ns() - t0 > timeout_ns) return false;
  }
}

#endif  // __CUDACC__

}  // namespace kl
