// Block-scaled tile kernels: MXFP8 (e4m3 / e5m2, tcgen05.mma kind::mxf8f6f4.block_scale) and MXFP4
// (packed e2m1, kind::mxf4.block_scale.block32), UE8M0 scales per 32 K-elements; and the
// scale-factor repacking kernel.

#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include <cuda_fp6.h>

#include <kl/gemm/gemm.hpp>

#include "kl_tile.cuh"

namespace kl::capi {

using mx::run_mx;

namespace {

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
  if (ab == KL_E3M2 || ab == KL_E2M3) return run_tile_fp6(ab, c, variant, pair, pr, stream, info, handled);
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

// Two fp32 values rounded (nearest, ties to even, saturating) to e4m3 / e2m1 / fp6, `lo` in the low
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
// fp6 (CUDA's fp6 conversion): each value in the low 6 bits of its byte.
template <int QT>
__device__ __forceinline__ uint32_t cvt_fp6x2(float lo, float hi) {
  return __nv_cvt_float2_to_fp6x2(make_float2(lo, hi), QT == KL_E3M2 ? __NV_E3M2 : __NV_E2M3, cudaRoundNearest);
}
// Element format constants: exponent of the largest normal value (OCP MX emax) and bytes per 32
// elements.
template <int QT>
inline constexpr int kQEmax = QT == KL_E4M3 ? 8 : QT == KL_E3M2 ? 4 : 2;
template <int QT>
inline constexpr int kQGroupBytes = QT == KL_E4M3 ? 32 : QT == KL_E2M1 ? 16 : 24;

// One thread per (row, 32-element group) of the padded blocked layout: the group's UE8M0 scale
// 2^(floor(log2(amax)) - emax) (OCP MX v1.0) goes to its blocked position, the elements x * 2^-e
// (exact: a power of two) are rounded to the element format. Padding positions get scale 127.
template <typename XT, int QT>
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
  const int e = (amax > 0.0f ? ilogbf(amax) : 0) - kQEmax<QT>;
  const int s = e + 127 < 0 ? 0 : e + 127 > 254 ? 254 : e + 127;
  *sfp = uint8_t(s);
  const float inv = ldexpf(1.0f, 127 - s);
  uint8_t* dst = q + r * ldq_bytes + g * kQGroupBytes<QT>;
  if constexpr (QT == KL_E3M2 || QT == KL_E2M3) {
    // 32 six-bit codes as one 192-bit little-endian stream: element i at bits [6i, 6i + 6).
    uint32_t w[6] = {0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const uint32_t pair = cvt_fp6x2<QT>(v[i] * inv, v[i + 1] * inv);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t c = (pair >> (8 * h)) & 63u;
        const int bit = 6 * (i + h), word = bit >> 5, off = bit & 31;
        w[word] |= c << off;
        if (off > 26) w[word + 1] |= c >> (32 - off);
      }
    }
    // 24 bytes at an 8-byte-aligned address (row pitches are multiples of 96 bytes).
    reinterpret_cast<uint2*>(dst)[0] = make_uint2(w[0], w[1]);
    reinterpret_cast<uint2*>(dst)[1] = make_uint2(w[2], w[3]);
    reinterpret_cast<uint2*>(dst)[2] = make_uint2(w[4], w[5]);
  } else if constexpr (QT == KL_E2M1) {
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

// ---- NVFP4 quantisation -----------------------------------------------------------------------

template <typename XT>
__device__ __forceinline__ float load_x(const XT* p) {
  if constexpr (sizeof(XT) == 4)
    return *p;
  else
    return __uint_as_float(uint32_t(*p) << 16);  // bf16 bits
}

// amax of |x| over the matrix, kept as float bits (non-negative floats order like their patterns):
// a grid-stride max per thread, a block max, one atomicMax per block into *out (zeroed before).
template <typename XT>
__global__ void amax_kernel(const XT* __restrict__ x, long long ldx, long long rows, long long k,
                            unsigned* __restrict__ out) {
  float m = 0.0f;
  const long long n = rows * k;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / k;
    m = fmaxf(m, fabsf(load_x(x + r * ldx + (i - r * k))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float warp_max[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) warp_max[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < int(blockDim.x >> 5) ? warp_max[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) atomicMax(out, __float_as_uint(m));
  }
}

// The per-tensor scale g = amax / (448 * 6) (1 for an all-zero x), in fp64 as every step below.
__device__ __forceinline__ double nv_global_scale(unsigned amax_bits) {
  const double amax = double(__uint_as_float(amax_bits));
  return amax > 0.0 ? amax / (448.0 * 6.0) : 1.0;
}

// One thread per (row, 16-element group) of the padded blocked layout (vec 16: K blocks of 64):
// scale s = e4m3(amax_group / (6 g)) (nearest, saturating; a UE4M3 byte), elements
// e2m1(x / (s g)) (0 where s = 0), packed two per byte, the first in the low nibble. Padding
// positions get scale 0x38 (1.0).
template <typename XT>
__global__ void nv_quantize_kernel(const XT* __restrict__ x, long long ldx, long long rows, long long groups,
                                   uint8_t* __restrict__ q, long long ldq_bytes, uint8_t* __restrict__ sf,
                                   long long k_blocks, long long rows_pad, const unsigned* __restrict__ amax_bits) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long groups_pad = k_blocks * 4;
  if (t >= rows_pad * groups_pad) return;
  const long long r = t / groups_pad, g = t - r * groups_pad;
  uint8_t* sfp = sf + ((r / 128) * k_blocks + g / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (g % 4);
  if (r >= rows || g >= groups) {
    *sfp = 0x38;
    return;
  }
  const double gs = nv_global_scale(*amax_bits);
  float v[16];
  const XT* src = x + r * ldx + g * 16;
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = load_x(src + i);
  float bmax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) bmax = fmaxf(bmax, fabsf(v[i]));
  const uint32_t sbits = cvt_e4m3x2(float(double(bmax) / (6.0 * gs)), 0.0f) & 0x7Fu;
  const uint32_t se = sbits >> 3, sm = sbits & 7u;  // the e4m3 value, exactly
  const double s = se == 0 ? ldexp(double(sm), -9) : ldexp(double(8 + sm), int(se) - 10);
  const double inv = s > 0.0 ? 1.0 / (s * gs) : 0.0;
  uint32_t w[2] = {0, 0};
#pragma unroll
  for (int j = 0; j < 8; ++j)
    w[j / 4] |= cvt_e2m1x2(float(double(v[2 * j]) * inv), float(double(v[2 * j + 1]) * inv)) << (8 * (j % 4));
  *reinterpret_cast<uint2*>(q + r * ldq_bytes + g * 8) = make_uint2(w[0], w[1]);
  *sfp = uint8_t(sbits);
}

// amax bits -> g, in place (one thread, after the quantisation has read the amax).
__global__ void nv_finish_kernel(unsigned* amax_then_g) {
  *reinterpret_cast<float*>(amax_then_g) = float(nv_global_scale(*amax_then_g));
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
  if (q_type != KL_E4M3 && q_type != KL_E2M1 && q_type != KL_E3M2 && q_type != KL_E2M3)
    return fail(KL_ERR_NOT_SUPPORTED, "kl_mx_quantize: q must be e4m3, e2m1, e3m2 or e2m3");
  if (k % 32 != 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: k must be a multiple of 32");
  const int xb = x_type == KL_F32 ? 4 : 2;
  const bool fp6 = q_type == KL_E3M2 || q_type == KL_E2M3;
  if (ldx < k || (ldx * xb) % 16 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: x must be 16-byte aligned with a 16-byte-multiple row pitch >= k");
  // Row pitch of q in bytes: e4m3 one per element, e2m1 two per byte, fp6 four per three bytes.
  const long long ldq_bytes = q_type == KL_E2M1 ? ldq / 2 : fp6 ? ldq / 4 * 3 : ldq;
  // Pitch granule, in elements: 16 bytes, or for fp6 96 bytes (128 elements, the GEMM's own rule).
  const long long ldq_unit = q_type == KL_E2M1 ? 32 : fp6 ? 128 : 16;
  if (ldq < k || ldq % ldq_unit != 0 || reinterpret_cast<uintptr_t>(q) % 16 != 0)
    return fail(KL_ERR_INVALID_ARGUMENT,
                fp6 ? "kl_mx_quantize: fp6 q must be 16-byte aligned with a row pitch >= k, a multiple of 128 elements"
                    : "kl_mx_quantize: q must be 16-byte aligned with a 16-byte-multiple row pitch >= k");
  if (reinterpret_cast<uintptr_t>(scales) % 16 != 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: scales must be 16-byte aligned");
  const long long k_blocks = (k + 127) / 128, rows_pad = (rows + 127) / 128 * 128;
  const long long threads = rows_pad * k_blocks * 4;
  const long long blocks = (threads + 255) / 256;
  if (blocks > INT32_MAX) return fail(KL_ERR_INVALID_ARGUMENT, "kl_mx_quantize: too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* qp = static_cast<uint8_t*>(q);
  auto* sp = static_cast<uint8_t*>(scales);
  auto launch = [&](auto const* xp, auto qt) {
    using XT = std::remove_cv_t<std::remove_pointer_t<decltype(xp)>>;
    kl::capi::mx_quantize_kernel<XT, decltype(qt)::value><<<unsigned(blocks), 256, 0, s>>>(
        xp, ldx, rows, k / 32, qp, ldq_bytes, sp, k_blocks, rows_pad);
  };
  auto by_q = [&](auto const* xp) {
    switch (q_type) {
      case KL_E4M3: launch(xp, std::integral_constant<int, KL_E4M3>{}); break;
      case KL_E2M1: launch(xp, std::integral_constant<int, KL_E2M1>{}); break;
      case KL_E3M2: launch(xp, std::integral_constant<int, KL_E3M2>{}); break;
      default: launch(xp, std::integral_constant<int, KL_E2M3>{}); break;
    }
  };
  if (x_type == KL_F32)
    by_q(static_cast<const float*>(x));
  else
    by_q(static_cast<const uint16_t*>(x));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KL_OK : kl::capi::cuda_fail(e, "kl_mx_quantize launch");
}

extern "C" kl_status kl_nv_quantize(const void* x, int32_t x_type, int64_t rows, int64_t k, int64_t ldx, void* q,
                                    int64_t ldq, void* scales, float* global_scale, void* stream) {
  using kl::capi::fail;
  if (rows < 0 || k < 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_nv_quantize: negative extent");
  if (rows == 0 || k == 0) return KL_OK;
  if (x == nullptr || q == nullptr || scales == nullptr || global_scale == nullptr)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_nv_quantize: null pointer");
  if (x_type != KL_F32 && x_type != KL_BF16) return fail(KL_ERR_NOT_SUPPORTED, "kl_nv_quantize: x must be f32 or bf16");
  if (k % 16 != 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_nv_quantize: k must be a multiple of 16");
  if (ldx < k) return fail(KL_ERR_INVALID_ARGUMENT, "kl_nv_quantize: ldx < k");
  if (ldq < k || ldq % 32 != 0 || reinterpret_cast<uintptr_t>(q) % 16 != 0)
    return fail(KL_ERR_INVALID_ARGUMENT,
                "kl_nv_quantize: q must be 16-byte aligned with a row pitch >= k, a multiple of 32 elements");
  if (reinterpret_cast<uintptr_t>(global_scale) % 4 != 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_nv_quantize: global_scale must be 4-byte aligned");
  const long long k_blocks = (k + 63) / 64, rows_pad = (rows + 127) / 128 * 128;
  const long long blocks = (rows_pad * k_blocks * 4 + 255) / 256;
  if (blocks > INT32_MAX) return fail(KL_ERR_INVALID_ARGUMENT, "kl_nv_quantize: too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* amax = reinterpret_cast<unsigned*>(global_scale);  // holds amax's bits until the last step
  cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(unsigned), s);
  if (e != cudaSuccess) return kl::capi::cuda_fail(e, "cudaMemsetAsync(amax)");
  auto* qp = static_cast<uint8_t*>(q);
  auto* sp = static_cast<uint8_t*>(scales);
  auto run = [&](auto const* xp) {
    using XT = std::remove_cv_t<std::remove_pointer_t<decltype(xp)>>;
    kl::capi::amax_kernel<XT><<<1184, 256, 0, s>>>(xp, ldx, rows, k, amax);
    kl::capi::nv_quantize_kernel<XT><<<unsigned(blocks), 256, 0, s>>>(xp, ldx, rows, k / 16, qp, ldq / 2, sp, k_blocks,
                                                                     rows_pad, amax);
  };
  if (x_type == KL_F32)
    run(static_cast<const float*>(x));
  else
    run(static_cast<const uint16_t*>(x));
  kl::capi::nv_finish_kernel<<<1, 1, 0, s>>>(amax);
  e = cudaGetLastError();
  return e == cudaSuccess ? KL_OK : kl::capi::cuda_fail(e, "kl_nv_quantize launch");
}
