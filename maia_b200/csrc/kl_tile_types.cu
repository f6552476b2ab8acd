// Tile-kernel instantiations for the less common input/output types: f16 inputs (kind::f16 with
// f16 operands), e5m2 inputs (kind::f8f6f4, operand format 1), and fp8 inputs with an fp32 C.

#include <kl/gemm/gemm.hpp>

#include "kl_tile.cuh"

namespace kl::capi {

namespace {

using kl::gemm::TnConfig;

template <typename InT, typename OutT, int CG>
using Tile = TnConfig<InT, OutT, CG, 256, CG == 2 ? 6 : 4>;

template <typename InT, typename OutT>
kl_status run_pair_or_single(kl::gemm::Problem const& pr, bool pair, cudaStream_t stream, kl::gemm::LaunchInfo* info) {
  return pair ? run_cfg<Tile<InT, OutT, 2>>(pr, stream, info) : run_cfg<Tile<InT, OutT, 1>>(pr, stream, info);
}

}  // namespace

kl_status run_tile_types(int32_t ab, int32_t c, kl::gemm::Problem const& pr, bool pair, cudaStream_t stream,
                         kl::gemm::LaunchInfo* info, bool* handled) {
  *handled = true;
  if (ab == KL_F16 && c == KL_F16) return run_pair_or_single<kl::f16, kl::f16>(pr, pair, stream, info);
  if (ab == KL_F16 && c == KL_F32) return run_pair_or_single<kl::f16, float>(pr, pair, stream, info);
  if (ab == KL_E4M3 && c == KL_F32) return run_pair_or_single<kl::e4m3, float>(pr, pair, stream, info);
  if (ab == KL_E5M2 && c == KL_BF16) return run_pair_or_single<kl::e5m2, kl::bf16>(pr, pair, stream, info);
  if (ab == KL_E5M2 && c == KL_F32) return run_pair_or_single<kl::e5m2, float>(pr, pair, stream, info);
  *handled = false;
  return KL_ERR_NOT_SUPPORTED;
}

}  // namespace kl::capi
