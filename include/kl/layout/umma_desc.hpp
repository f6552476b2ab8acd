#pragma once

// UMMA (tcgen05.mma) operand descriptors.
//  - SmemDesc: the 64-bit shared-memory matrix descriptor. Field names and bit positions are the
//    ones kernel_lib/include/kl/layout/umma_desc.hpp:13 gets from CuTe's UMMA::SmemDescriptor, so
//    code that reads desc.start_address_ etc. keeps working.
//  - umma_desc(tile, k, row): descriptor of the k-th MMA K-slice of a K-major tile
//    (kernel_lib/include/kl/layout/umma_desc.hpp:31-47).
//  - mma_instr_desc<A, B, Acc, M, N>(): the 32-bit instruction descriptor
//    (kernel_lib/include/kl/layout/umma_desc.hpp:49-58), extended to M = 256 (cta_group::2).
// Every encoder is plain shifts, so they are constexpr and usable on the host.

#include <cassert>
#include <cstdint>
#include <type_traits>

#include <kl/config.hpp>
#include <kl/layout/smem_tile.hpp>
#include <kl/types.hpp>

namespace kl {

// Shared-memory layout codes of the descriptor's 3-bit layout field (bits 61..63).
enum class UmmaLayout : uint8_t {
  SWIZZLE_NONE = 0,
  SWIZZLE_128B_BASE32B = 1,
  SWIZZLE_128B = 2,
  SWIZZLE_64B = 4,
  SWIZZLE_32B = 6,
};

// 64-bit UMMA shared-memory descriptor. The union's field names and its lo / hi view follow CuTe's
// UMMA::SmemDescriptor (CUTLASS, Copyright (c) 2017 - 2025 NVIDIA CORPORATION & AFFILIATES, BSD-3-
// Clause licence), because callers of the reference read those names; the bit positions are the
// hardware's.
//   [0,14)  start address >> 4        [16,30) leading byte offset >> 4
//   [32,46) stride byte offset >> 4   [46,48) version (1 on sm_100)
//   [49,52) base offset               [52]    LBO mode
//   [61,64) layout (UmmaLayout)
union SmemDesc {
  uint64_t desc_ = 0;
  struct {
    uint16_t start_address_ : 14, : 2;
    uint16_t leading_byte_offset_ : 14, : 2;
    uint16_t stride_byte_offset_ : 14, version_ : 2;
    uint8_t : 1, base_offset_ : 3, lbo_mode_ : 1, : 3;
    uint8_t : 5, layout_type_ : 3;
  };
  struct {
    uint32_t lo;
    uint32_t hi;
  };

  KL_HOST_DEVICE constexpr operator uint64_t() const noexcept { return desc_; }
};
static_assert(sizeof(SmemDesc) == 8);

template <typename Sw>
KL_HOST_DEVICE constexpr UmmaLayout umma_layout() {
  if constexpr (Sw::bytes == 128) return UmmaLayout::SWIZZLE_128B;
  else if constexpr (Sw::bytes == 64) return UmmaLayout::SWIZZLE_64B;
  else if constexpr (Sw::bytes == 32) return UmmaLayout::SWIZZLE_32B;
  else return UmmaLayout::SWIZZLE_NONE;
}

// Pack the descriptor fields. Offsets are in bytes; the encoder drops the 4 low bits.
KL_HOST_DEVICE constexpr uint64_t encode_smem_desc(uint32_t start_bytes, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                                   UmmaLayout layout, uint32_t base_offset = 0) {
  return (uint64_t((start_bytes >> 4) & 0x3FFFu)) | (uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(base_offset & 7u) << 49) |
         (uint64_t(static_cast<uint8_t>(layout) & 7u) << 61);
}

// Elements of K that a single dense tcgen05.mma consumes: the instruction reads 32 bytes of every
// operand row whatever the kind (f16, tf32, f8f6f4, i8), so 16 for 16-bit types, 32 for 8-bit.
template <typename T>
inline constexpr int mma_k = 256 / bits_of<T>;

// MMAs needed to cover the K extent (the columns) of one operand tile.
template <SmemTileType Tile>
inline constexpr int num_k_blocks = Tile::cols / mma_k<typename Tile::value_type>;

namespace detail {

KL_HOST_DEVICE constexpr UmmaLayout umma_layout_rt(int swizzle_span) {
  return swizzle_span == 128 ? UmmaLayout::SWIZZLE_128B
         : swizzle_span == 64 ? UmmaLayout::SWIZZLE_64B
         : swizzle_span == 32 ? UmmaLayout::SWIZZLE_32B
                              : UmmaLayout::SWIZZLE_NONE;
}

// block_offset_16B with the tile as numbers.
KL_HOST_DEVICE constexpr uint32_t block_offset_16B_rt(int elem_bytes, int rows, int swizzle_span, int k_block, int row) {
  const int atom_elems = swizzle_span / elem_bytes;
  const int mma_k_elems = 32 / elem_bytes;
  return static_cast<uint32_t>(tile_offset(rows, atom_elems, row, k_block * mma_k_elems) * elem_bytes / 16);
}

// Descriptor of the first K-slice (rows [0, rows), K = 32 bytes) of a K-major tile at shared
// address `tile_addr`. Canonical K-major forms, in 16-byte units:
//   swizzled (32/64/128 B): ((8, n), 2) : ((Sw/16, SBO), 1)  -> LBO field 1, SBO = 8 rows * Sw bytes
//   no swizzle (interleave): ((8, n), 2) : ((1, SBO), LBO)   -> SBO = 8 rows * 16 B, LBO = rows * 16 B
KL_HOST_DEVICE constexpr uint64_t umma_desc_first_slice_rt(uint32_t tile_addr, int rows, int swizzle_span) {
  const UmmaLayout layout = umma_layout_rt(swizzle_span);
  const uint32_t sbo = 8u * uint32_t(swizzle_span);
  const uint32_t lbo = (layout == UmmaLayout::SWIZZLE_NONE) ? uint32_t(rows) * 16u : 16u;
  return encode_smem_desc(tile_addr, lbo, sbo, layout);
}

// Like CuTe's descriptor iterator, the K-slice offset is a 32-bit add on the low word: inside the
// shared-memory window the start address never carries into the LBO field.
KL_HOST_DEVICE constexpr uint64_t umma_desc_rt(uint32_t tile_addr, int elem_bytes, int rows, int swizzle_span,
                                               int k_block, int row) {
  const uint64_t d = umma_desc_first_slice_rt(tile_addr, rows, swizzle_span);
  const uint32_t lo = static_cast<uint32_t>(d) + block_offset_16B_rt(elem_bytes, rows, swizzle_span, k_block, row);
  return (d & 0xFFFFFFFF00000000ull) | lo;
}

// MN-major operands. The tile is stored K rows x MN columns (MN contiguous, SmemTile<T, K, MN, Sw>),
// atoms stacked down the K rows first, so a strip of one swizzle span of MN is contiguous over
// all K rows. Canonical MN-major swizzled form, in 16-byte units:
//   ((Sw/16, n), (8, k)) : ((1, LBO), (Sw/16, SBO))
// LBO = bytes between MN strips (K rows x Sw bytes; 0 when the operand is a single strip, as CuTe
// encodes an unused stride), SBO = bytes between 8-row K groups (8 x Sw bytes). The K-slice of one
// MMA (32 bytes of K = mma_k rows) starts mma_k rows further.
KL_HOST_DEVICE constexpr uint64_t umma_desc_mn_rt(uint32_t tile_addr, int elem_bytes, int k_rows, int swizzle_span,
                                                  int k_block, int mn_col, int mn_extent) {
  const UmmaLayout layout = umma_layout_rt(swizzle_span);
  const uint32_t lbo = mn_extent > swizzle_span / elem_bytes ? uint32_t(k_rows) * uint32_t(swizzle_span) : 0u;
  const uint32_t sbo = 8u * uint32_t(swizzle_span);
  const int atom_elems = swizzle_span / elem_bytes;
  const int mma_k_rows = 32 / elem_bytes;
  const uint32_t off = static_cast<uint32_t>(tile_offset(k_rows, atom_elems, k_block * mma_k_rows, mn_col) * elem_bytes);
  return encode_smem_desc(tile_addr + off, lbo, sbo, layout);
}

}  // namespace detail

// Descriptor of the k-th MMA K-slice of an MN-major tile (SmemTile<T, K rows, MN cols, Sw>, Sw a
// 32/64/128-byte swizzle) at shared address `tile_addr`, for the MN columns [mn_col, mn_col +
// mn_extent) one MMA reads (mn_col a multiple of the atom width; mn_extent 0 = all columns).
// No counterpart in the reference, whose descriptors are K-major only.
template <SmemTileType Tile>
KL_HOST_DEVICE constexpr SmemDesc umma_desc_mn_at(uint32_t tile_addr, int k_block = 0, int mn_col = 0,
                                                  int mn_extent = 0) {
  using T = typename Tile::value_type;
  static_assert(Tile::swizzle::bytes >= 32, "MN-major descriptors here cover the swizzled layouts");
  SmemDesc d;
  d.desc_ = detail::umma_desc_mn_rt(tile_addr, bits_of<T> / 8, Tile::rows, Tile::swizzle::bytes, k_block, mn_col,
                                    mn_extent > 0 ? mn_extent : Tile::cols);
  return d;
}

// Offset of the k-th MMA K-slice, starting at `row`, from the start of the tile, in 16-byte units,
// measured on the un-swizzled layout (the hardware applies the swizzle itself).
// (kernel_lib/include/kl/layout/umma_desc.hpp:22-29)
template <SmemTileType Tile>
KL_HOST_DEVICE constexpr uint32_t block_offset_16B(int k_block, int row = 0) {
  using T = typename Tile::value_type;
  return detail::block_offset_16B_rt(bits_of<T> / 8, Tile::rows, Tile::swizzle::bytes, k_block, row);
}

// Descriptor for the k-th MMA K-slice of a tile at shared address `tile_addr`, for rows
// [row, row + M or N). `row` lets one tile feed several MMAs along M or N; it must be a multiple of
// 8 so the slice starts on a swizzle-pattern boundary.
template <SmemTileType Tile>
KL_HOST_DEVICE constexpr SmemDesc umma_desc_at(uint32_t tile_addr, int k_block = 0, int row = 0) {
  using T = typename Tile::value_type;
  SmemDesc d;
  d.desc_ = detail::umma_desc_rt(tile_addr, bits_of<T> / 8, Tile::rows, Tile::swizzle::bytes, k_block, row);
  return d;
}

#if defined(__CUDACC__)
// (kernel_lib/include/kl/layout/umma_desc.hpp:35-47)
template <SmemTileType Tile>
KL_DEVICE SmemDesc umma_desc(Tile const& tile, int k_block = 0, int row = 0) {
  using T = typename Tile::value_type;
  static_assert(Tile::cols % mma_k<T> == 0, "tile K extent must be a multiple of the MMA K");
  assert(row % 8 == 0 && row < Tile::rows);
  return umma_desc_at<std::remove_cvref_t<Tile>>(tile.smem_u32(), k_block, row);
}
#endif

// Operand format codes of the instruction descriptor (bits 7..9 for A, 10..12 for B).
namespace detail {
template <typename T>
KL_HOST_DEVICE constexpr uint32_t umma_operand_format() {
  if constexpr (std::is_same_v<T, f16>) return 0;       // kind::f16
  else if constexpr (std::is_same_v<T, bf16>) return 1;  // kind::f16
  else if constexpr (std::is_same_v<T, float>) return 2; // kind::tf32 (fp32 storage read as tf32)
  else if constexpr (std::is_same_v<T, e4m3>) return 0;  // kind::f8f6f4
  else if constexpr (std::is_same_v<T, e5m2>) return 1;  // kind::f8f6f4
  else if constexpr (std::is_same_v<T, e2m3>) return 3;  // kind::f8f6f4 / mxf8f6f4
  else if constexpr (std::is_same_v<T, e3m2>) return 4;  // kind::f8f6f4 / mxf8f6f4
  else if constexpr (std::is_same_v<T, e2m1x2>) return 1;  // kind::mxf4 / mxf4nvf4 (packed e2m1)
  else if constexpr (std::is_same_v<T, uint8_t>) return 0;  // kind::i8
  else if constexpr (std::is_same_v<T, int8_t>) return 1;   // kind::i8
  else static_assert(sizeof(T) == 0, "no UMMA operand format for this element type");
}
template <typename T>
KL_HOST_DEVICE constexpr uint32_t umma_accum_format() {
  if constexpr (std::is_same_v<T, f16>) return 0;
  else if constexpr (std::is_same_v<T, float>) return 1;
  else if constexpr (std::is_same_v<T, int32_t>) return 2;
  else static_assert(sizeof(T) == 0, "no UMMA accumulator format for this type");
}
}  // namespace detail

// Major-ness of an operand in shared memory (bit 15 for A, 16 for B).
enum class UmmaMajor : uint32_t { K = 0, MN = 1 };

namespace detail {
// The instruction descriptor from format codes:
//   [4,6) accumulator format  [7,10) A format  [10,13) B format  [13] negate A  [14] negate B
//   [15] A major  [16] B major  [17,23) N >> 3  [24,29) M >> 4  [30,32) max shift (0)
KL_HOST_DEVICE constexpr uint32_t instr_desc_rt(uint32_t a_fmt, uint32_t b_fmt, uint32_t c_fmt, int m, int n,
                                                uint32_t a_major = 0, uint32_t b_major = 0) {
  return (c_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | (a_major << 15) | (b_major << 16) | (uint32_t(n >> 3) << 17) |
         (uint32_t(m >> 4) << 24);
}
}  // namespace detail

// 32-bit instruction descriptor for a dense tcgen05.mma. M = 64 or 128 issue with cta_group::1;
// M = 256 is a CTA pair (cta_group::2), which the reference's encoder rejects.
template <typename A, typename B, typename Acc, int M, int N, UmmaMajor AMajor = UmmaMajor::K,
          UmmaMajor BMajor = UmmaMajor::K>
KL_HOST_DEVICE constexpr uint32_t mma_instr_desc() {
  static_assert(M == 64 || M == 128 || M == 256, "tcgen05.mma supports M = 64, 128 (one CTA) or 256 (CTA pair)");
  static_assert(N <= 256 && N >= (M == 64 ? 8 : 16) && N % (M == 64 ? 8 : 16) == 0,
                "N must be a multiple of 8 (M=64) or 16 (M=128/256), at most 256");
  static_assert(bits_of<A> == bits_of<B>, "A and B of one MMA have the same element width");
  return detail::instr_desc_rt(detail::umma_operand_format<A>(), detail::umma_operand_format<B>(),
                               detail::umma_accum_format<Acc>(), M, N, static_cast<uint32_t>(AMajor),
                               static_cast<uint32_t>(BMajor));
}

namespace detail {
// Block-scaled form (kind::mxf8f6f4.block_scale): no accumulator-format field (fp32 always);
//   [4,6) B scale-factor id  [7,10) A format  [10,13) B format  [13] negate A  [14] negate B
//   [15] A major  [16] B major  [17,23) N >> 3  [23] scale format (1 = UE8M0)  [24,29) M >> 4
//   [29,31) A scale-factor id  [31] K size (0 = K32)
// The scale-factor ids pick the byte of each 32-bit TMEM scale word an MMA reads.
KL_HOST_DEVICE constexpr uint32_t instr_desc_block_scaled_rt(uint32_t a_fmt, uint32_t b_fmt, int m, int n,
                                                             uint32_t a_sf_id = 0, uint32_t b_sf_id = 0,
                                                             uint32_t a_major = 0, uint32_t b_major = 0) {
  return (b_sf_id << 4) | (a_fmt << 7) | (b_fmt << 10) | (a_major << 15) | (b_major << 16) |
         (uint32_t(n >> 3) << 17) | (1u << 23) | (uint32_t(m >> 4) << 24) | (a_sf_id << 29);
}
}  // namespace detail

// 32-bit instruction descriptor for a block-scaled 8-bit MMA (MXFP8: e4m3 / e5m2 operands, one
// UE8M0 scale per 32 K-elements), K-major operands, fp32 accumulate. No counterpart in the
// reference; the field layout is CuTe's InstrDescriptorBlockScaled.
template <typename A, typename B, int M, int N>
KL_HOST_DEVICE constexpr uint32_t mma_instr_desc_block_scaled(uint32_t a_sf_id = 0, uint32_t b_sf_id = 0) {
  static_assert(M == 128 || M == 256, "block-scaled tcgen05.mma: M = 128 (one CTA) or 256 (CTA pair)");
  static_assert(N <= 256 && N >= 16 && N % 16 == 0, "N must be a multiple of 16, at most 256");
  static_assert(bits_of<A> == 8 && bits_of<B> == 8, "block-scaled operands are 8-bit floats or packed fp4 pairs");
  static_assert(std::is_same_v<A, e2m1x2> == std::is_same_v<B, e2m1x2>, "fp4 (kind::mxf4) takes fp4 A and B");
  return detail::instr_desc_block_scaled_rt(detail::umma_operand_format<A>(), detail::umma_operand_format<B>(), M, N,
                                            a_sf_id, b_sf_id);
}

}  // namespace kl
