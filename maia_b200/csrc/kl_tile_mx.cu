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

// ---- MX quantisation (activations on the fly) -----------------------------------------------------
namespace kl::capi {
namespace {

// Two fp32 values rounded (nearest, ties to even, saturating) to e4m3 / e2m1, `lo` in the low
// byte / nibble.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
  uint16_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u16.u8 %0, t;\n\t}" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// One thread per (row, 32-element group) of the padded blocked layout: the group's UE8M0 scale
// 2^(floor(log2(amax)) - emax) (OCP MX v1.0) goes to its blocked position, the elements x * 2^-e
// (exact: a power of two) are rounded to the element format. Padding positions get scale 127.
template <typename XT, bool Fp4>
__global__ void mx_quantize_kernel(const XT* __restrict__ x, long long ldx, long long rows, long long groups,
                                   uint8_t* __restrict__ q, long long ldq_bytes, uint8_t* __restrict__ sf,
                                   long long k_blocks, long long rows_pad) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long groups_pad = k_blocks * 4;
  if (t >= rows_pad * groups_pad) return;
  const long long r = t / groups_pad, g = t - r * groups_pad;
  uint8_t* sfp = sf + ((r / 128) * k_blocks + g / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (g % 4);
  if (r >= rows || g >= groups) {
    *sfp = 127;
    return;
  }
  float v[32];
  const XT* src = x + r * ldx + g * 32;
  if constexpr (sizeof(XT) == 4) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 f = reinterpret_cast<const float4*>(src)[i];
      v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = reinterpret_cast<const uint4*>(src)[i];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
        v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
  }
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  constexpr int emax = Fp4 ? 2 : 8;  // exponent of the element format's largest normal value
  const int e = (amax > 0.0f ? ilogbf(amax) : 0) - emax;
  const int s = e + 127 < 0 ? 0 : e + 127 > 254 ? 254 : e + 127;
  *sfp = uint8_t(s);
  const float inv = ldexpf(1.0f, 127 - s);
  uint8_t* dst = q + r * ldq_bytes + g * (Fp4 ? 16 : 32);
  if constexpr (Fp4) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w[i] = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) w[i] |= cvt_e2m1x2(v[8 * i + 2 * j] * inv, v[8 * i + 2 * j + 1] * inv) << (8 * j);
    }
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      w[i] = cvt_e4m3x2(v[4 * i] * inv, v[4 * i + 1] * inv) | (cvt_e4m3x2(v[4 * i + 2] * inv, v[4 * i + 3] * inv) << 16);
    reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

}  // namespace
}  // namespace kl::capi

extern "C" kl_status kl_mx_quantize(const void* x, int32_t x_type, int64_t rows, int64_t k, int64_t ldx,
                                    int32_t q_type, void* q, int64_t ldq, void* scales, void* stream) {
  using kl::capi::fail;
  if (rows < 0 || k < 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: negative extent");
  if (rows == 0 || k == 0) return KL_OK;
  if (x == nullptr || q == nullptr || scales == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: null pointer");
  if (x_type != KL_F32 && x_type != KL_BF16) return fail(KL_ERR_NOT_SUPPORTED, "kl_mx_quantize: x must be f32 or bf16");
  if (q_type != KL_E4M3 && q_type != KL_E2M1) return fail(KL_ERR_NOT_SUPPORTED, "kl_mx_quantize: q must be e4m3 or e2m1");
  if (k % 32 != 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: k must be a multiple of 32");
  const int xb = x_type == KL_F32 ? 4 : 2;
  const bool fp4 = q_type == KL_E2M1;
  if (ldx < k || (ldx * xb) % 16 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: x must be 16-byte aligned with a 16-byte-multiple row pitch >= k");
  if (ldq < k || (fp4 && ldq % 32 != 0) || (!fp4 && ldq % 16 != 0) || reinterpret_cast<uintptr_t>(q) % 16 != 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: q must be 16-byte aligned with a 16-byte-multiple row pitch >= k");
  if (reinterpret_cast<uintptr_t>(scales) % 16 != 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: scales must be 16-byte aligned");
  const long long k_blocks = (k + 127) / 128, rows_pad = (rows + 127) / 128 * 128;
  const long long threads = rows_pad * k_blocks * 4;
  const long long blocks = (threads + 255) / 256;
  if (blocks > INT32_MAX) return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: too large");
  const long long ldq_bytes = fp4 ? ldq / 2 : ldq;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* qp = static_cast<uint8_t*>(q);
  auto* sp = static_cast<uint8_t*>(scales);
  if (x_type == KL_F32) {
    if (fp4)
      kl::capi::mx_quantize_kernel<float, true><<<unsigned(blocks), 256, 0, s>>>(
          static_cast<const float*>(x), ldx, rows, k / 32, qp, ldq_bytes, sp, k_blocks, rows_pad);
    else
      kl::capi::mx_quantize_kernel<float, false><<<unsigned(blocks), 256, 0, s>>>(
          static_cast<const float*>(x), ldx, rows, k / 32, qp, ldq_bytes, sp, k_blocks, rows_pad);
  } else {
    if (fp4)
      kl::capi::mx_quantize_kernel<uint16_t, true><<<unsigned(blocks), 256, 0, s>>>(
          static_cast<const uint16_t*>(x), ldx, rows, k / 32, qp, ldq_bytes, sp, k_blocks, rows_pad);
    else
      kl::capi::mx_quantize_kernel<uint16_t, false><<<unsigned(blocks), 256, 0, s>>>(
          static_cast<const uint16_t*>(x), ldx, rows, k / 32, qp, ldq_bytes, sp, k_blocks, rows_pad);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KL_OK : kl::capi::cuda_fail(e, "kl_mx_quantize launch");
}
