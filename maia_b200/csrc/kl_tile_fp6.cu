// Block-scaled tile kernels on packed fp6 operands (e3m2 / e2m3 with UE8M0 scales per 32
// K-elements, tcgen05.mma kind::mxf8f6f4.block_scale). The operands arrive through TMA's 16U6
// data type, which unpacks each 12 bytes of global memory into a 16-byte shared-memory slot, so
// the tiles, stage counts and MMAs are those of MXFP8.

#include <cuda_runtime.h>

#include <cstdint>

#include <kl/gemm/gemm.hpp>

#include "kl_tile.cuh"

namespace kl::capi {

kl_status run_tile_fp6(int32_t ab, int32_t c, int32_t variant, bool pair, kl::gemm::Problem const& pr,
                       cudaStream_t stream, kl::gemm::LaunchInfo* info, bool* handled) {
  using mx::run_mx;
  *handled = true;
  if (ab == KL_E3M2 && c == KL_BF16) return run_mx<kl::e3m2, kl::bf16>(variant, pair, pr, stream, info);
  if (ab == KL_E3M2 && c == KL_F32) return run_mx<kl::e3m2, float>(variant, pair, pr, stream, info);
  if (ab == KL_E2M3 && c == KL_BF16) return run_mx<kl::e2m3, kl::bf16>(variant, pair, pr, stream, info);
  if (ab == KL_E2M3 && c == KL_F32) return run_mx<kl::e2m3, float>(variant, pair, pr, stream, info);
  *handled = false;
  return KL_ERR_NOT_SUPPORTED;
}

}  // namespace kl::capi
