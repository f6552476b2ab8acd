#pragma once

// Launch helper and variant dispatchers of the tile kernels (gemm_tn_kernel), shared by the
// translation units that instantiate them. Internal to libkl_b200.so.

#include <cuda_runtime.h>

#include <kl/gemm/gemm.hpp>
#include <kl_gemm.h>

#include "kl_internal.cuh"

namespace kl::capi {

// Queue the tile kernel `Cfg` for `pr`, reporting into the device status word.
// A launch whose schedule splits its tail gets the stream's workspace (unless the caller
// brought one); without it the launch deals whole tiles.
template <class Cfg>
kl_status run_cfg(kl::gemm::Problem const& pr0, cudaStream_t stream, kl::gemm::LaunchInfo* info) {
  int* status = nullptr;
  kl_status s = device_status_ptr(&status);
  if (s != KL_OK) return s;
  kl::gemm::Problem pr = pr0;
  if (pr.stream_k >= 0 && pr.sk_workspace == nullptr) {
    int dev = 0, max_workers = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = kl::gemm::detail::prepare_kernel<Cfg>(dev, &max_workers);
    if (e != cudaSuccess) return cuda_fail(e, "kl_gemm setup");
    if (kl::gemm::tn_schedule<Cfg>(pr, max_workers).sk_tiles > 0) {
      void* ws = nullptr;
      s = tile_stream_k_workspace(stream, &ws);
      if (s != KL_OK) return s;
      pr.sk_workspace = ws;
      pr.sk_workspace_bytes = ws != nullptr ? kl::gemm::kTnStreamKWorkspaceBytes : 0;
    }
  }
  cudaError_t e = kl::gemm::launch_tn<Cfg>(pr, status, wait_timeout_ns(), stream, info);
  if (e != cudaSuccess) return cuda_fail(e, "kl_gemm launch");
  return KL_OK;
}

// The block-scaled tile configurations (stage counts for 8-bit-per-element shared-memory tiles:
// fp8, and fp6 which TMA unpacks to one element per byte; packed fp4 tiles hold twice the K).
namespace mx {

using kl::gemm::TnConfig;

// One CTA, 128 x 256 tiles: one TMEM accumulator (the scales take the rest), 3 stages of 49.5 KB.
template <typename InT, typename OutT, int V>
using Mx256 = TnConfig<InT, OutT, 1, 256, 3, false, false, false, kl::Swizzle128B, V>;
// One CTA, 128 x 128 tiles: two accumulators (epilogue overlapped), 5 stages of 33 KB.
template <typename InT, typename OutT, int V>
using Mx128 = TnConfig<InT, OutT, 1, 128, 5, false, false, false, kl::Swizzle128B, V>;
// CTA pair, 256 x 256 tiles: one accumulator per CTA, 5 stages of 33.5 KB per CTA (fp8).
template <typename InT, typename OutT, int V>
using MxPair = TnConfig<InT, OutT, 2, 256, 5, false, false, false, kl::Swizzle128B, V>;
// CTA pair, 256 x 192 tiles: two accumulators (2 x 192 columns leave room for the scales), 6 stages
// of 29.5 KB per CTA (fp8; 5 for NVFP4's larger scale tiles). B's 192-row tiles start 0 or 64 rows
// into a 128-row scale block.
template <typename InT, typename OutT, int V>
using MxPair192 = TnConfig<InT, OutT, 2, 192, V == 16 ? 5 : 6, false, false, false, kl::Swizzle128B, V>;
// CTA pair, 256 x 128 tiles: two accumulators, 7 stages of 25 KB per CTA (fp8).
template <typename InT, typename OutT, int V>
using MxPair128 = TnConfig<InT, OutT, 2, 128, V == 16 ? 6 : 7, false, false, false, kl::Swizzle128B, V>;

template <typename InT, typename OutT, int V = 32>
kl_status run_mx(int32_t variant, bool pair, kl::gemm::Problem const& pr, cudaStream_t stream,
                 kl::gemm::LaunchInfo* info) {
  if (pair)
    return variant == 2   ? run_cfg<MxPair128<InT, OutT, V>>(pr, stream, info)
           : variant == 3 ? run_cfg<MxPair192<InT, OutT, V>>(pr, stream, info)
                          : run_cfg<MxPair<InT, OutT, V>>(pr, stream, info);
  return variant == 2 ? run_cfg<Mx128<InT, OutT, V>>(pr, stream, info) : run_cfg<Mx256<InT, OutT, V>>(pr, stream, info);
}

}  // namespace mx

// Each returns KL_ERR_NOT_SUPPORTED, without touching the last-error message, when it has no
// kernel for the request; *handled says whether it had one.
// kl_tile_types.cu: (f16, f16), (f16, f32), (e4m3, f32), (e5m2, bf16), (e5m2, f32).
kl_status run_tile_types(int32_t ab_type, int32_t c_type, kl::gemm::Problem const& pr, bool pair, cudaStream_t stream,
                         kl::gemm::LaunchInfo* info, bool* handled);
// kl_tile_swizzle.cu: 64- and 32-byte operand swizzle, bf16 inputs, bf16 or f32 C.
kl_status run_tile_swizzle(int32_t swizzle, int32_t ab_type, int32_t c_type, kl::gemm::Problem const& pr, bool pair,
                           cudaStream_t stream, kl::gemm::LaunchInfo* info, bool* handled);

// kl_tile_wide.cu: 256 x 512 CTA-pair tiles (two MMAs of N = 256 per stage of A), (bf16, bf16) and
// (e4m3, bf16), K-major, 128-byte swizzle.
kl_status run_tile_wide(int32_t ab_type, int32_t c_type, kl::gemm::Problem const& pr, cudaStream_t stream,
                        kl::gemm::LaunchInfo* info, bool* handled);
// Whether the pair's default (variant 0) takes the wide tiles for this problem: bf16 in and out,
// one problem, no split tail on the 256 x 256 tiles and at least their share of busy worker-waves.
bool wide_tiles_pay(int32_t ab_type, int32_t c_type, kl::gemm::Problem const& pr);

// kl_tile_mx.cu: block-scaled GEMMs (MXFP8, MXFP4, NVFP4), bf16 or f32 C. `pair`: 256 x 256 tiles on a
// CTA pair; one CTA: variant 0/1 = 128 x 256 tiles with one accumulator, 2 = 128 x 128 with two.
// mode: 1 = MX (UE8M0 scales per 32 elements), 2 = NVFP4 (UE4M3 per 16, e2m1 only).
kl_status run_tile_mx(int32_t mode, int32_t ab_type, int32_t c_type, int32_t variant, bool pair,
                      kl::gemm::Problem const& pr, cudaStream_t stream, kl::gemm::LaunchInfo* info, bool* handled);
// kl_tile_fp6.cu: MX block-scaled GEMMs on packed fp6 (e3m2 / e2m3) operands, kind::mxf8f6f4; the
// same tiles and variants as run_tile_mx.
kl_status run_tile_fp6(int32_t ab_type, int32_t c_type, int32_t variant, bool pair, kl::gemm::Problem const& pr,
                       cudaStream_t stream, kl::gemm::LaunchInfo* info, bool* handled);

}  // namespace kl::capi
