// Block-scaled tile kernels: MXFP8 (e4m3 / e5m2, tcgen05.mma kind::mxf8f6f4.block_scale) and MXFP4
// (packed e2m1, kind::mxf4.block_scale.block32), UE8M0 scales per 32 K-elements; and the
// scale-factor repacking kernel.

#include <cuda_runtime.h>

#include <cstdint>

#include <kl/gemm/gemm.hpp>

#include "kl_tile.cuh"

namespace kl::capi {

namespace {

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

// One thread per 32-bit word of the blocked layout: the four K-group scales of one row. Padding
// (rows past `rows`, K-groups past `groups`) holds `pad`, a finite scale of 1 in the scale format
// (UE8M0 127, UE4M3 0x38): padded K-groups multiply zero-filled elements, which a NaN scale would
// turn into NaN.
__global__ void pack_scales_kernel(const uint8_t* __restrict__ src, long long rows, long long groups, long long ld,
                                   uint32_t* __restrict__ dst, long long k_blocks, long long words, uint32_t pad) {
  const long long w = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (w >= words) return;
  const long long atom = w >> 7;        // 128 words per 512-byte atom
  const int pos = int(w & 127);         // word inside the atom: (r % 32) * 4 + r / 32
  const long long rb = atom / k_blocks, kb = atom - rb * k_blocks;
  const long long row = rb * 128 + (pos & 3) * 32 + (pos >> 2);
  uint32_t v = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const long long g = kb * 4 + j;
    const uint32_t s = (row < rows && g < groups) ? src[row * ld + g] : pad;
    v |= s << (8 * j);
  }
  dst[w] = v;
}

}  // namespace

kl_status run_tile_mx(int32_t mode, int32_t ab, int32_t c, int32_t variant, bool pair, kl::gemm::Problem const& pr,
                      cudaStream_t stream, kl::gemm::LaunchInfo* info, bool* handled) {
  *handled = true;
  if (variant < 0 || variant > 3 || (variant == 3 && !pair))
    return fail(KL_ERR_INVALID_ARGUMENT,
                "block-scaled variant must be 0, 1 (256-column tiles), 2 (128) or, on a CTA pair, 3 (192)");
  if (mode == 2) {  // NVFP4: UE4M3 scales per 16 elements
    if (ab == KL_E2M1 && c == KL_BF16) return run_mx<kl::e2m1x2, kl::bf16, 16>(variant, pair, pr, stream, info);
    if (ab == KL_E2M1 && c == KL_F32) return run_mx<kl::e2m1x2, float, 16>(variant, pair, pr, stream, info);
    *handled = false;
    return KL_ERR_NOT_SUPPORTED;
  }
  if (ab == KL_E4M3 && c == KL_BF16) return run_mx<kl::e4m3, kl::bf16>(variant, pair, pr, stream, info);
  if (ab == KL_E4M3 && c == KL_F32) return run_mx<kl::e4m3, float>(variant, pair, pr, stream, info);
  if (ab == KL_E5M2 && c == KL_BF16) return run_mx<kl::e5m2, kl::bf16>(variant, pair, pr, stream, info);
  if (ab == KL_E5M2 && c == KL_F32) return run_mx<kl::e5m2, float>(variant, pair, pr, stream, info);
  if (ab == KL_E2M1 && c == KL_BF16) return run_mx<kl::e2m1x2, kl::bf16>(variant, pair, pr, stream, info);
  if (ab == KL_E2M1 && c == KL_F32) return run_mx<kl::e2m1x2, float>(variant, pair, pr, stream, info);
  *handled = false;
  return KL_ERR_NOT_SUPPORTED;
}

}  // namespace kl::capi

extern "C" {

int64_t kl_block_scale_bytes(int64_t rows, int64_t k, int32_t vec) {
  if (rows <= 0 || k <= 0 || (vec != 16 && vec != 32)) return 0;
  return ((rows + 127) / 128) * ((k + 4 * vec - 1) / (4 * vec)) * 512;
}

int64_t kl_mx_scale_bytes(int64_t rows, int64_t k) { return kl_block_scale_bytes(rows, k, 32); }

kl_status kl_pack_block_scales(const void* src, int64_t rows, int64_t k, int32_t vec, int64_t ld_src, void* dst,
                               void* stream) {
  using kl::capi::fail;
  if (vec != 16 && vec != 32) return fail(KL_ERR_INVALID_ARGUMENT, "kl_pack_block_scales: vec must be 16 or 32");
  if (rows < 0 || k < 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_pack_block_scales: negative extent");
  if (rows == 0 || k == 0) return KL_OK;
  const int64_t groups = (k + vec - 1) / vec;
  if (src == nullptr || dst == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "kl_pack_block_scales: null pointer");
  if (ld_src < groups) return fail(KL_ERR_INVALID_ARGUMENT, "kl_pack_block_scales: ld_src < ceil(k / vec)");
  if (reinterpret_cast<uintptr_t>(dst) % 16 != 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_pack_block_scales: dst must be 16-byte aligned");
  const int64_t k_blocks = (k + 4 * vec - 1) / (4 * vec);
  const int64_t words = kl_block_scale_bytes(rows, k, vec) / 4;
  const int threads = 256;
  const int64_t blocks = (words + threads - 1) / threads;
  if (blocks > INT32_MAX) return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_pack_scales: too large");
  kl::capi::pack_scales_kernel<<<unsigned(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), rows, groups, ld_src, static_cast<uint32_t*>(dst), k_blocks, words,
      vec == 16 ? 0x38u : 127u);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KL_OK : kl::capi::cuda_fail(e, "kl_pack_block_scales launch");
}

kl_status kl_mx_pack_scales(const void* src, int64_t rows, int64_t k, int64_t ld_src, void* dst, void* stream) {
  return kl_pack_block_scales(src, rows, k, 32, ld_src, dst, stream);
}

}  // extern "C"
