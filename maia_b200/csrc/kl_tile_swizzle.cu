// Tile kernels whose operand tiles use the 64- or 32-byte swizzle: a stage still holds 128 bytes
// of K, as two (64 B) or four (32 B) swizzle-atom columns, each loaded by its own TMA box
// (TmaBox<Tile>::count boxes) and addressed by the MMAs through block_offset_16B.

#include <kl/gemm/gemm.hpp>

#include "kl_tile.cuh"

namespace kl::capi {

namespace {

using kl::gemm::TnConfig;

template <typename OutT, int CG, class Sw>
using Tile = TnConfig<kl::bf16, OutT, CG, 256, CG == 2 ? 6 : 4, false, false, false, Sw>;

template <typename OutT, class Sw>
kl_status run_pair_or_single(kl::gemm::Problem const& pr, bool pair, cudaStream_t stream, kl::gemm::LaunchInfo* info) {
  return pair ? run_cfg<Tile<OutT, 2, Sw>>(pr, stream, info) : run_cfg<Tile<OutT, 1, Sw>>(pr, stream, info);
}

}  // namespace

kl_status run_tile_swizzle(int32_t swizzle, int32_t ab, int32_t c, kl::gemm::Problem const& pr, bool pair,
                           cudaStream_t stream, kl::gemm::LaunchInfo* info, bool* handled) {
  *handled = true;
  if (ab == KL_BF16 && c == KL_BF16) {
    if (swizzle == 64) return run_pair_or_single<kl::bf16, kl::Swizzle64B>(pr, pair, stream, info);
    if (swizzle == 32) return run_pair_or_single<kl::bf16, kl::Swizzle32B>(pr, pair, stream, info);
  }
  if (ab == KL_BF16 && c == KL_F32) {
    if (swizzle == 64) return run_pair_or_single<float, kl::Swizzle64B>(pr, pair, stream, info);
    if (swizzle == 32) return run_pair_or_single<float, kl::Swizzle32B>(pr, pair, stream, info);
  }
  *handled = false;
  return KL_ERR_NOT_SUPPORTED;
}

}  // namespace kl::capi
