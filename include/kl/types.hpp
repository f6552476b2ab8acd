#pragma once

// Element types. kernel_lib/include/kl/types.hpp:9-15 aliases CUTLASS's numeric types; kl for
// B200 aliases CUDA's own storage types instead, so no CUTLASS header is needed anywhere.

#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace kl {

using bf16 = __nv_bfloat16;
using f16 = __half;
using e4m3 = __nv_fp8_e4m3;
using e5m2 = __nv_fp8_e5m2;

// Width of one element in bits. Every type kl supports is a whole number of bytes.
template <typename T>
inline constexpr int bits_of = static_cast<int>(sizeof(T) * 8);

}  // namespace kl
