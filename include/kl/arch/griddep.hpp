#pragma once

// Programmatic dependent launch (PTX griddepcontrol): a kernel launched with the
// programmatic-stream-serialization attribute may start while the kernel before it on the stream
// is still running, as soon as every CTA of that kernel has signalled `griddep_launch_dependents`
// (or exited) and an SM has room. It runs its prologue (barrier init, TMEM allocation, tensor-map
// prefetch) in the other kernel's shadow and must call `griddep_wait` before it touches global
// memory: that returns once the kernels it depends on have completed and their writes are visible.
// Without the attribute (or with no kernel before it) both are no-ops.
// No counterpart in the reference: kernel_lib launches nothing.

#include <kl/config.hpp>

namespace kl {

#if defined(__CUDACC__)

KL_DEVICE void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

KL_DEVICE void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

#endif  // __CUDACC__

}  // namespace kl
