#pragma once

// Launch helper and variant dispatchers of the tile kernels (gemm_tn_kernel), shared by the
// translation units that instantiate them. Internal to libkl_b200.so.

#include <cuda_runtime.h>

#include <kl/gemm/gemm.hpp>
#include <kl_gemm.h>

#include "kl_internal.cuh"

namespace kl::capi {

// Queue the tile kernel `Cfg` for `pr`, reporting into the device status word.
template <class Cfg>
kl_status run_cfg(kl::gemm::Problem const& pr, cudaStream_t stream, kl::gemm::LaunchInfo* info) {
  int* status = nullptr;
  kl_status s = device_status_ptr(&status);
  if (s != KL_OK) return s;
  cudaError_t e = kl::gemm::launch_tn<Cfg>(pr, status, wait_timeout_ns(), stream, info);
  if (e != cudaSuccess) return cuda_fail(e, "kl_gemm launch");
  return KL_OK;
}

// Each returns KL_ERR_NOT_SUPPORTED, without touching the last-error message, when it has no
// kernel for the request; *handled says whether it had one.
// kl_tile_types.cu: (f16, f16), (f16, f32), (e4m3, f32), (e5m2, bf16), (e5m2, f32).
kl_status run_tile_types(int32_t ab_type, int32_t c_type, kl::gemm::Problem const& pr, bool pair, cudaStream_t stream,
                         kl::gemm::LaunchInfo* info, bool* handled);
// kl_tile_swizzle.cu: 64- and 32-byte operand swizzle, bf16 inputs, bf16 or f32 C.
kl_status run_tile_swizzle(int32_t swizzle, int32_t ab_type, int32_t c_type, kl::gemm::Problem const& pr, bool pair,
                           cudaStream_t stream, kl::gemm::LaunchInfo* info, bool* handled);

// kl_tile_mx.cu: block-scaled GEMMs (MXFP8, MXFP4, NVFP4), bf16 or f32 C. `pair`: 256 x 256 tiles on a
// CTA pair; one CTA: variant 0/1 = 128 x 256 tiles with one accumulator, 2 = 128 x 128 with two.
// mode: 1 = MX (UE8M0 scales per 32 elements), 2 = NVFP4 (UE4M3 per 16, e2m1 only).
kl_status run_tile_mx(int32_t mode, int32_t ab_type, int32_t c_type, int32_t variant, bool pair,
                      kl::gemm::Problem const& pr, cudaStream_t stream, kl::gemm::LaunchInfo* info, bool* handled);

}  // namespace kl::capi
