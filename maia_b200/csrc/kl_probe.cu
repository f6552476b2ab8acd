// The failure path of kl's bounded waits, run on purpose: a single thread waits on an mbarrier
// that no one arrives on. The wait gives up after `timeout_ns`, records a status bit and the
// kernel returns normally, leaving the context usable.

#include <cuda_runtime.h>

#include <kl/arch/mbarrier.hpp>
#include <kl/gemm/gemm_kernel.cuh>

#include "kl_internal.cuh"

namespace {

constexpr int kStatusProbeTimeout = 16;

__global__ void wait_probe_kernel(int* status, unsigned long long timeout_ns) {
  __shared__ alignas(8) unsigned long long bar;
  const uint32_t b = kl::smem_addr(&bar);
  kl::mbarrier_init(b, 1);
  kl::fence_barrier_init();
  // Phase 0 never completes: nothing arrives.
  if (!kl::mbarrier_wait(b, 0, timeout_ns)) atomicOr(status, kStatusProbeTimeout);
}

}  // namespace

namespace kl::capi {

kl_status launch_wait_probe(int* status, unsigned long long timeout_ns, cudaStream_t stream) {
  wait_probe_kernel<<<1, 1, 0, stream>>>(status, timeout_ns);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KL_OK : cuda_fail(e, "wait probe launch");
}

}  // namespace kl::capi
