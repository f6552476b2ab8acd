#pragma once

// Swizzled shared-memory tiles: the layout every TMA box and UMMA descriptor in kl is derived from.
// Same contract as kernel_lib/include/kl/layout/smem_tile.hpp:12-84 (tags, atom, tile, concept),
// expressed as small constexpr functors instead of CuTe layout algebra.

#include <cstdint>
#include <type_traits>

#include <kl/config.hpp>
#include <kl/types.hpp>

namespace kl {

// Shared-memory swizzle modes, named by their span in bytes. `bits` is how many address bits the
// swizzle XORs: the 16-byte chunk index inside a span, bits [4, 4 + bits), is XORed with the row
// inside the 8-row pattern, bits [7, 7 + bits). (kernel_lib/include/kl/layout/smem_tile.hpp:12-28)
struct SwizzleNone {
  static constexpr int bytes = 16;
  static constexpr int bits = 0;
};
struct Swizzle32B {
  static constexpr int bytes = 32;
  static constexpr int bits = 1;
};
struct Swizzle64B {
  static constexpr int bytes = 64;
  static constexpr int bits = 2;
};
struct Swizzle128B {
  static constexpr int bytes = 128;
  static constexpr int bits = 3;
};

// The swizzle as a function of a byte address (or a byte offset from a pattern-aligned base).
template <typename Sw>
KL_HOST_DEVICE constexpr uint32_t swizzle_bytes(uint32_t byte_addr) {
  constexpr uint32_t mask = (1u << Sw::bits) - 1u;
  return byte_addr ^ (((byte_addr >> 7) & mask) << 4);
}

namespace detail {
// Runtime forms of the layout functions below (the C ABI and the typed templates share them).
KL_HOST_DEVICE constexpr int64_t tile_offset(int rows, int atom_elems, int row, int col) {
  return int64_t(col / atom_elems) * (int64_t(rows) * atom_elems) + int64_t(row) * atom_elems + col % atom_elems;
}
KL_HOST_DEVICE constexpr uint32_t swizzle_bytes_rt(int sw_bits, uint32_t byte_addr) {
  return byte_addr ^ (((byte_addr >> 7) & ((1u << sw_bits) - 1u)) << 4);
}
KL_HOST_DEVICE constexpr int64_t swizzled_tile_offset(int elem_bytes, int rows, int atom_elems, int sw_bits, int row,
                                                      int col) {
  const int64_t byte = tile_offset(rows, atom_elems, row, col) * elem_bytes;
  // The swizzle only touches address bits [4, 10); the rest pass through.
  const int64_t hi = byte & ~int64_t(1023);
  return (hi + swizzle_bytes_rt(sw_bits, static_cast<uint32_t>(byte & 1023))) / elem_bytes;
}
}  // namespace detail

// Un-swizzled element offset of (row, col) in a Rows x Cols tile built from 8-row x atom-wide
// atoms stacked down the rows first. Column strip j (atom_elems wide) is one contiguous block of
// Rows * atom_elems elements, i.e. exactly one TMA box. This is the layout the hardware sees
// before it applies the swizzle to addresses.
template <typename T, int Rows, int Cols, typename Sw>
struct TileOffset {
  static constexpr int atom_elems = Sw::bytes * 8 / bits_of<T>;
  KL_HOST_DEVICE constexpr int64_t operator()(int row, int col) const {
    return detail::tile_offset(Rows, atom_elems, row, col);
  }
};

// Swizzled layout of a Rows x Cols tile of T: (row, col) -> element offset from a base aligned to
// the swizzle pattern (8 rows x Sw::bytes). The swizzle acts on byte addresses, so any element
// width works; the alignment requirement is what SmemTile::alignment guarantees.
template <typename T, int Rows, int Cols, typename Sw>
struct SmemLayout {
  using value_type = T;
  using swizzle = Sw;
  static constexpr int rows = Rows;
  static constexpr int cols = Cols;

  // The un-swizzled part (the name follows the A o B composition convention: A = swizzle, B = offsets).
  KL_HOST_DEVICE constexpr TileOffset<T, Rows, Cols, Sw> layout_b() const { return {}; }

  KL_HOST_DEVICE constexpr int64_t operator()(int row, int col) const {
    return detail::swizzled_tile_offset(bits_of<T> / 8, Rows, Sw::bytes * 8 / bits_of<T>, Sw::bits, row, col);
  }
  KL_HOST_DEVICE static constexpr int64_t size() { return int64_t(Rows) * Cols; }
  KL_HOST_DEVICE static constexpr int64_t cosize() { return int64_t(Rows) * Cols; }
};

// One swizzle atom: 8 rows x Sw::bytes. (kernel_lib/include/kl/layout/smem_tile.hpp:30-37)
template <typename T, typename Sw>
using smem_atom = SmemLayout<T, 8, Sw::bytes * 8 / bits_of<T>, Sw>;

// Atoms tiled to (Rows, Cols), rows first. (kernel_lib/include/kl/layout/smem_tile.hpp:39-42)
template <typename T, int Rows, int Cols, typename Sw>
using smem_layout = SmemLayout<T, Rows, Cols, Sw>;

// A typed view of a tile's storage: t(row, col) is the element at that logical position.
template <typename T, typename Layout>
struct SmemTensor {
  T* ptr;
  KL_HOST_DEVICE constexpr T& operator()(int row, int col) const { return ptr[Layout{}(row, col)]; }
  KL_HOST_DEVICE constexpr T* data() const { return ptr; }
  KL_HOST_DEVICE static constexpr Layout layout() { return {}; }
};

// Rows x Cols elements of T in shared memory, each row's Cols elements contiguous and the 16-byte
// chunks of every 8-row group permuted by the swizzle Sw. Used for the operands of an MMA, whose
// rows are M (or N) and whose columns run along K. The storage is an aligned array inside the
// struct itself, so a kernel lays out its shared memory by declaring tiles as members. The member
// names follow kernel_lib/include/kl/layout/smem_tile.hpp:48-76.
template <typename T, int Rows, int Cols, typename Sw = Swizzle128B>
struct SmemTile {
  using value_type = T;
  using swizzle = Sw;
  using layout_type = smem_layout<T, Rows, Cols, Sw>;

  static constexpr int rows = Rows;
  static constexpr int cols = Cols;
  static constexpr int size = Rows * Cols;
  static constexpr int bytes = size * bits_of<T> / 8;
  // The swizzle pattern repeats every 8 rows of Sw::bytes; TMA wants at least 128 B.
  static constexpr int alignment = Sw::bytes * 8 < 128 ? 128 : Sw::bytes * 8;
  static constexpr int atom_elems = Sw::bytes * 8 / bits_of<T>;  // columns per swizzle atom

  static_assert(bits_of<T> >= 8, "sub-byte element types are not supported yet");
  static_assert(Cols % atom_elems == 0, "cols must be a multiple of the swizzle atom width");
  static_assert(Rows % 8 == 0, "rows must be a multiple of 8");

  alignas(alignment) unsigned char storage[bytes];

  KL_HOST_DEVICE T* data() { return reinterpret_cast<T*>(storage); }
  KL_HOST_DEVICE T const* data() const { return reinterpret_cast<T const*>(storage); }

  KL_HOST_DEVICE SmemTensor<T, layout_type> tensor() { return {data()}; }
  KL_HOST_DEVICE SmemTensor<T const, layout_type> tensor() const { return {data()}; }

#if defined(__CUDACC__)
  // 32-bit shared-window address of the tile (what TMA, mbarrier and UMMA descriptors take).
  KL_DEVICE uint32_t smem_u32() const { return static_cast<uint32_t>(__cvta_generic_to_shared(storage)); }
#endif
};

template <typename T>
inline constexpr bool is_smem_tile_v = false;
template <typename T, int R, int C, typename S>
inline constexpr bool is_smem_tile_v<SmemTile<T, R, C, S>> = true;

template <typename T>
concept SmemTileType = is_smem_tile_v<std::remove_cvref_t<T>>;

}  // namespace kl
