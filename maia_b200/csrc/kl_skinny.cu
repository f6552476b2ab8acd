// Memory-bound small-M GEMM (decode shapes). Filled in below the dispatch helpers.

#include <cuda_runtime.h>

#include <kl/gemm/gemm.hpp>

#include "kl_internal.cuh"

namespace kl::capi {

int choose_algo(kl_gemm_desc const& d) {
  // A CTA pair needs at least 256 rows to fill its tile; below that one CTA per tile.
  return d.m >= 256 ? KL_ALGO_2CTA : KL_ALGO_1CTA;
}

kl_status skinny_workspace_size(kl_gemm_desc const& d, size_t* bytes) {
  (void)d;
  *bytes = 0;
  return fail(KL_ERR_NOT_SUPPORTED, "KL_ALGO_SKINNY is not built yet");
}

kl_status run_skinny(kl_gemm_desc const& d, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  (void)d;
  (void)workspace;
  (void)workspace_bytes;
  (void)stream;
  return fail(KL_ERR_NOT_SUPPORTED, "KL_ALGO_SKINNY is not built yet");
}

}  // namespace kl::capi
