// Wide CTA-pair tiles: 256 x 512, two MMAs of N = 256 sharing every stage of A (TnConfig NSub = 2).
// Per MAC they bring 3/4 of the operand bytes of the 256 x 256 tiles from L2, which is what bounds
// the pair kernel when every SM runs at a high clock; their one accumulator fills TMEM, so the
// next tile waits for its drain.

#include <kl/gemm/gemm.hpp>

#include "kl_tile.cuh"

namespace kl::capi {

namespace {

using kl::gemm::TnConfig;

template <typename InT, typename OutT>
using WidePair = TnConfig<InT, OutT, 2, 256, 4, false, false, false, kl::Swizzle128B, 0, 2>;
using NarrowPairBf16 = TnConfig<kl::bf16, kl::bf16, 2, 256, 6>;  // the default pair kernel (kl_capi.cu)

// Share of the worker-waves a schedule keeps busy: tiles / (waves * workers).
double wave_fill(int tiles, int workers) {
  if (tiles <= 0 || workers <= 0) return 0.0;
  const long long waves = (tiles + workers - 1) / workers;
  return double(tiles) / double(waves * workers);
}

}  // namespace

bool wide_tiles_pay(int32_t ab, int32_t c, kl::gemm::Problem const& pr) {
  // Measured on B200 (bf16, back to back, same call): 8192 x 1024 x 8192 95.8 vs 100.3 us, 8192^3
  // 698 vs 706 us, both with the same wave fill on either tile; 8192 x 4096 375 vs 358 us (the wide
  // tiles fill fewer waves), 8192 x 2048 and 4096^3 equal or slower (the split tail already fills
  // their last wave). fp8 was slower on every shape measured, so only bf16 takes them.
  if (ab != KL_BF16 || c != KL_BF16) return false;
  if (pr.batch > 1 || pr.m_block_group != nullptr || pr.max_ctas > 0) return false;
  int dev = 0, wn = 0, ww = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (kl::gemm::detail::prepare_kernel<NarrowPairBf16>(dev, &wn) != cudaSuccess ||
      kl::gemm::detail::prepare_kernel<WidePair<kl::bf16, kl::bf16>>(dev, &ww) != cudaSuccess)
    return false;
  const kl::gemm::TnSchedule sn = kl::gemm::tn_schedule<NarrowPairBf16>(pr, wn);
  if (sn.sk_tiles > 0) return false;
  const kl::gemm::TnSchedule sw = kl::gemm::tn_schedule<WidePair<kl::bf16, kl::bf16>>(pr, ww);
  return wave_fill(sw.tiles, ww) >= wave_fill(sn.tiles, wn) - 1e-9;
}

kl_status run_tile_wide(int32_t ab, int32_t c, kl::gemm::Problem const& pr, cudaStream_t stream,
                        kl::gemm::LaunchInfo* info, bool* handled) {
  *handled = true;
  if (ab == KL_BF16 && c == KL_BF16) return run_cfg<WidePair<kl::bf16, kl::bf16>>(pr, stream, info);
  if (ab == KL_E4M3 && c == KL_BF16) return run_cfg<WidePair<kl::e4m3, kl::bf16>>(pr, stream, info);
  *handled = false;
  return KL_ERR_NOT_SUPPORTED;
}

}  // namespace kl::capi
