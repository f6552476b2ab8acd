#pragma once

// Stores through an NVLink multicast address (multimem.st): one store instruction writes the same
// 16 bytes into every GPU's memory bound to the multicast object, the NVSwitch doing the fan-out.
// No counterpart in the reference (kernel_lib has no multi-GPU code).
//
// Only stores are issued here: nothing in this library reads through a multicast address, and no
// TMA copy is given one.

#include <cstdint>

#include <kl/config.hpp>

namespace kl {

#if defined(__CUDACC__)

// 16 bytes (four 32-bit words, stored bit for bit) to a 16-byte-aligned multicast address. Relaxed,
// system scope: a consumer on another GPU sees them after a system-scope fence on this side
// (multimem_fence) and a synchronisation that orders its reads after it.
KL_DEVICE void multimem_st_v4(void* mc_addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Orders this thread's earlier multicast stores before anything it does afterwards, for observers
// on every GPU.
KL_DEVICE void multimem_fence() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

#endif  // __CUDACC__

}  // namespace kl
