#pragma once

// Element types. kernel_lib/include/kl/types.hpp:9-15 aliases CUTLASS's numeric types; kl for
// B200 aliases CUDA's own storage types instead, so no CUTLASS header is needed anywhere.

#include <cstdint>
#include <type_traits>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace kl {

using bf16 = __nv_bfloat16;
using f16 = __half;
using e4m3 = __nv_fp8_e4m3;
using e5m2 = __nv_fp8_e5m2;

// Two e2m1 (fp4: 1 sign, 2 exponent bits with bias 1, 1 mantissa bit) values packed in one byte,
// the first in the low nibble. kl moves fp4 as these byte pairs: tiles, tensor maps and K extents
// of a packed operand count bytes, i.e. element pairs. (No counterpart in the reference, whose
// types stop at 8 bits.)
struct e2m1x2 {
  uint8_t bits;
};

// fp6 elements (OCP MX): e3m2 (1 sign, 3 exponent bits with bias 3, 2 mantissa bits, largest 28)
// and e2m3 (1 sign, 2 exponent bits with bias 1, 3 mantissa bits, largest 7.5); neither has an
// infinity or a NaN. In global memory they are packed, element i of a row at bits [6i, 6i + 6) of
// the row's bytes (least significant bit first: four elements in three bytes). TMA's 16U6 data
// type spreads each 16 elements (12 bytes) over a 16-byte slot of shared memory, so a shared-memory
// tile holds one element per byte, as for fp8: kernels and tiles use these one-byte types, and
// only tensor maps and transaction byte counts see the packing. (No counterpart in the reference.)
struct e3m2 {
  uint8_t bits;
};
struct e2m3 {
  uint8_t bits;
};
template <typename T>
inline constexpr bool is_fp6 = std::is_same_v<T, e3m2> || std::is_same_v<T, e2m3>;

// Width of one element (of one storage unit, for e2m1x2) in bits.
template <typename T>
inline constexpr int bits_of = static_cast<int>(sizeof(T) * 8);

}  // namespace kl
