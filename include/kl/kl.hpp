#pragma once

// Umbrella header (kernel_lib/include/kl/kl.hpp:1-11): the descriptor and layout API. Device-side
// wrappers (mbarrier, cluster, TMA, tcgen05) live under <kl/arch/...> and the GEMM under
// <kl/gemm/...>; they are included separately because they need nvcc.

#include <kl/config.hpp>
#include <kl/types.hpp>

#include <kl/layout/gmem_tensor.hpp>
#include <kl/layout/smem_tile.hpp>
#include <kl/layout/tma_desc.hpp>
#include <kl/layout/umma_desc.hpp>
