#pragma once

// TMA tensor-map builders. Same contract as kernel_lib/include/kl/layout/tma_desc.hpp:16-164:
// the same type and swizzle mapping, the same box geometry, the same validation (and messages)
// and the same arguments to cuTensorMapEncodeTiled, so the 128-byte maps are byte-identical.
// The driver entry point is resolved through the CUDA runtime, so users need not link libcuda.

#include <cuda.h>
#include <cuda_runtime_api.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <type_traits>

#include <kl/layout/gmem_tensor.hpp>
#include <kl/layout/smem_tile.hpp>
#include <kl/types.hpp>

namespace kl {

// Plain loads/stores only need the element size; real types matter for reducing stores and keep
// maps identical to the reference's. (kernel_lib/include/kl/layout/tma_desc.hpp:19-34)
template <typename T>
constexpr CUtensorMapDataType tma_dtype() {
  if constexpr (std::is_same_v<T, bf16>) {
    return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  } else if constexpr (std::is_same_v<T, f16>) {
    return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  } else if constexpr (std::is_same_v<T, float>) {
    return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  } else if constexpr (std::is_same_v<T, int32_t>) {
    return CU_TENSOR_MAP_DATA_TYPE_INT32;
  } else if constexpr (bits_of<T> == 8) {
    return CU_TENSOR_MAP_DATA_TYPE_UINT8;  // int8 / uint8 / fp8 move as raw bytes
  } else {
    static_assert(sizeof(T) == 0, "no TMA data type for this element type");
  }
}

// (kernel_lib/include/kl/layout/tma_desc.hpp:36-42)
template <typename Sw>
constexpr CUtensorMapSwizzle tma_swizzle() {
  if constexpr (Sw::bytes == 128) return CU_TENSOR_MAP_SWIZZLE_128B;
  else if constexpr (Sw::bytes == 64) return CU_TENSOR_MAP_SWIZZLE_64B;
  else if constexpr (Sw::bytes == 32) return CU_TENSOR_MAP_SWIZZLE_32B;
  else return CU_TENSOR_MAP_SWIZZLE_NONE;
}

// How a tile is covered by TMA boxes: one swizzle atom wide, at most 256 rows tall. Box i is
// column strip i / row_boxes, row block i % row_boxes, which walks storage front to back.
// (kernel_lib/include/kl/layout/tma_desc.hpp:44-74)
struct TmaBoxGeometry {
  int elem_bytes, rows;
  int inner, outer, col_boxes, row_boxes, count, bytes;
  KL_HOST_DEVICE constexpr int row(int i) const { return i % row_boxes * outer; }
  KL_HOST_DEVICE constexpr int col(int i) const { return i / row_boxes * inner; }
  // Byte offset of box i inside the tile (on the un-swizzled layout).
  KL_HOST_DEVICE constexpr uint32_t smem_offset(int i) const {
    return static_cast<uint32_t>(detail::tile_offset(rows, inner, row(i), col(i)) * elem_bytes);
  }
};

KL_HOST_DEVICE constexpr TmaBoxGeometry tma_box_geometry(int elem_bytes, int rows, int cols, int swizzle_span) {
  const int inner = swizzle_span / elem_bytes;  // the tile's atom width
  const int outer = rows < 256 ? rows : 256;
  const int col_boxes = cols / inner;
  const int row_boxes = rows / outer;
  return {elem_bytes, rows, inner, outer, col_boxes, row_boxes, col_boxes * row_boxes, inner * outer * elem_bytes};
}

template <SmemTileType Tile>
struct TmaBox {
  using T = typename Tile::value_type;
  static constexpr TmaBoxGeometry geometry =
      tma_box_geometry(bits_of<T> / 8, Tile::rows, Tile::cols, Tile::swizzle::bytes);
  static constexpr int inner = geometry.inner;
  static constexpr int outer = geometry.outer;
  static constexpr int col_boxes = geometry.col_boxes;
  static constexpr int row_boxes = geometry.row_boxes;
  static constexpr int count = geometry.count;
  static constexpr int bytes = geometry.bytes;

  static_assert(inner == Tile::atom_elems);
  static_assert(Tile::rows % outer == 0, "tiles taller than 256 rows must be a multiple of 256 rows");
  static_assert(inner <= 256 && outer <= 256, "TMA boxes are at most 256 along each dimension");
  static_assert(inner * bits_of<T> / 8 % 16 == 0, "a TMA box row must be a multiple of 16 bytes");
  static_assert(inner * bits_of<T> / 8 <= Tile::swizzle::bytes,
                "a swizzled TMA box row can't be wider than the swizzle span");

  // Position of box i's first element inside the tile, in elements. (Same formulas as
  // TmaBoxGeometry, written on the scalar members so device code can call them.)
  KL_HOST_DEVICE static constexpr int row(int i) { return i % row_boxes * outer; }
  KL_HOST_DEVICE static constexpr int col(int i) { return i / row_boxes * inner; }
  // Byte offset of box i inside the tile.
  KL_HOST_DEVICE static constexpr uint32_t smem_offset(int i) {
    return static_cast<uint32_t>(detail::tile_offset(Tile::rows, inner, row(i), col(i)) * (bits_of<T> / 8));
  }
};

struct TmaLoadTag {};
struct TmaStoreTag {};

// A tensor map for moving `Tile`s between shared memory and a rank-`Rank` global tensor.
// Pass it to kernels as `const __grid_constant__`. (kernel_lib/include/kl/layout/tma_desc.hpp:79-94)
template <SmemTileType Tile, typename Direction, int Rank = 2>
struct TmaDesc {
  using tile_type = Tile;
  using direction = Direction;
  static constexpr int rank = Rank;  // picks the TMA instruction (one coordinate per mode)
  CUtensorMap map;

  KL_HOST_DEVICE CUtensorMap const* get() const { return &map; }
};

template <SmemTileType Tile, int Rank = 2>
using TmaLoad = TmaDesc<Tile, TmaLoadTag, Rank>;
template <SmemTileType Tile, int Rank = 2>
using TmaStore = TmaDesc<Tile, TmaStoreTag, Rank>;

// Knobs the reference fixes. The defaults reproduce its maps exactly; kernels may ask for a
// different L2 promotion where a measurement says so.
struct TmaOptions {
  CUtensorMapL2promotion l2_promotion = CU_TENSOR_MAP_L2_PROMOTION_L2_128B;
};

namespace detail {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from whichever libcuda the CUDA runtime loaded (nullptr without a driver).
inline EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();  // do not leave a sticky runtime error behind
      return EncodeTiledFn{nullptr};
    }
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

[[noreturn]] inline void tma_fail(std::string const& what) {
  throw std::invalid_argument("kl::make_tma_desc: " + what);
}

}  // namespace detail

namespace detail {

// The body of make_tma_desc with the tile reduced to numbers: element type and width, swizzle and
// box. Dimensions and strides come outermost first, in elements, as in GmemTensor. Throws
// std::invalid_argument("kl::make_tma_desc: ...") exactly where the reference does.
inline void encode_tma_map(CUtensorMap* out, CUtensorMapDataType dtype, int elem_bytes, CUtensorMapSwizzle swizzle,
                           uint32_t box_inner, uint32_t box_outer, void const* gmem, int R, int64_t const* shape,
                           int64_t const* stride, TmaOptions const& opt) {
  if (R < 2 || R > 5) tma_fail("TMA tensors have 2 to 5 modes");
  // TMA lists dimensions innermost first and leaves the innermost stride implicit.
  uint64_t dims[5], strides[4];
  uint32_t box[5], elem_strides[5];
  for (int i = 0; i < R; ++i) {
    dims[i] = static_cast<uint64_t>(shape[R - 1 - i]);
    box[i] = i == 0 ? box_inner : i == 1 ? box_outer : 1;
    elem_strides[i] = 1;
  }
  for (int i = 1; i < R; ++i) strides[i - 1] = static_cast<uint64_t>(stride[R - 1 - i]) * elem_bytes;

  if (reinterpret_cast<uintptr_t>(gmem) % 16 != 0) tma_fail("global address must be 16-byte aligned");
  for (int i = 0; i < R; ++i)
    if (shape[i] < 1 || shape[i] > (int64_t(1) << 32)) tma_fail("extents must be in [1, 2^32]");
  for (int i = 0; i < R - 1; ++i)
    if (stride[i] <= 0 || strides[R - 2 - i] % 16 != 0 || strides[R - 2 - i] >= (uint64_t(1) << 40))
      tma_fail("outer strides must be positive multiples of 16 bytes, below 2^40 bytes");
  if (stride[R - 2] < shape[R - 1]) tma_fail("rows overlap: the row stride is smaller than cols");
  // The reference enforces this one at compile time through CuTe's static stride _1; a GmemTensor
  // built by row_major* always satisfies it, a hand-built one is checked here.
  if (stride[R - 1] != 1) tma_fail("the last mode must be contiguous (stride 1)");

  auto encode = tensor_map_encoder();
  if (encode == nullptr) tma_fail("cuTensorMapEncodeTiled is unavailable (no CUDA driver)");
  *out = CUtensorMap{};
  CUresult res = encode(out, dtype, static_cast<cuuint32_t>(R), const_cast<void*>(gmem), dims, strides, box,
                        elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, opt.l2_promotion,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res == CUDA_ERROR_NOT_SUPPORTED) tma_fail("the current device has no TMA (needs sm_90 or newer)");
  if (res != CUDA_SUCCESS) tma_fail("cuTensorMapEncodeTiled failed with CUresult " + std::to_string(int(res)));
}

// The same for packed fp6 (kl::e3m2 / kl::e2m3): TMA's 16U6_ALIGN16B data type reads 16 elements
// (12 bytes) of global memory into every 16-byte slot of shared memory. Shapes, strides and boxes
// count elements; the driver's rules for this type (cuTensorMapEncodeTiled, CUDA 12.8+): the base
// 32-byte aligned, the innermost extent a multiple of 128 elements, every stride a multiple of 32
// bytes (= 128 elements), the box 128 elements wide, and 128-byte swizzle (or none). A tile's x
// coordinate is then always a multiple of 128 elements (96 bytes).
inline void encode_tma_map_u6(CUtensorMap* out, CUtensorMapSwizzle swizzle, uint32_t box_inner, uint32_t box_outer,
                              void const* gmem, int R, int64_t const* shape, int64_t const* stride,
                              TmaOptions const& opt) {
  if (R < 2 || R > 5) tma_fail("TMA tensors have 2 to 5 modes");
  if (box_inner != 128) tma_fail("packed fp6 boxes are 128 elements wide");
  if (swizzle != CU_TENSOR_MAP_SWIZZLE_128B && swizzle != CU_TENSOR_MAP_SWIZZLE_NONE)
    tma_fail("packed fp6 tiles use 128-byte swizzle");
  if (reinterpret_cast<uintptr_t>(gmem) % 32 != 0) tma_fail("packed fp6: global address must be 32-byte aligned");
  if (shape[R - 1] % 128 != 0) tma_fail("packed fp6: the innermost extent must be a multiple of 128 elements");
  for (int i = 0; i < R - 1; ++i)
    if (stride[i] <= 0 || stride[i] % 128 != 0)
      tma_fail("packed fp6: outer strides must be positive multiples of 128 elements (32 bytes)");
  if (stride[R - 1] != 1) tma_fail("the last mode must be contiguous (stride 1)");
  if (stride[R - 2] < shape[R - 1]) tma_fail("rows overlap: the row stride is smaller than cols");
  uint64_t dims[5], strides[4];
  uint32_t box[5], elem_strides[5];
  for (int i = 0; i < R; ++i) {
    if (shape[i] < 1 || shape[i] > (int64_t(1) << 32)) tma_fail("extents must be in [1, 2^32]");
    dims[i] = static_cast<uint64_t>(shape[R - 1 - i]);
    box[i] = i == 0 ? box_inner : i == 1 ? box_outer : 1;
    elem_strides[i] = 1;
  }
  for (int i = 1; i < R; ++i) {
    strides[i - 1] = static_cast<uint64_t>(stride[R - 1 - i]) * 3 / 4;  // 6 bits per element
    if (strides[i - 1] >= (uint64_t(1) << 40)) tma_fail("outer strides must be below 2^40 bytes");
  }
  auto encode = tensor_map_encoder();
  if (encode == nullptr) tma_fail("cuTensorMapEncodeTiled is unavailable (no CUDA driver)");
  *out = CUtensorMap{};
  CUresult res = encode(out, CU_TENSOR_MAP_DATA_TYPE_16U6_ALIGN16B, static_cast<cuuint32_t>(R), const_cast<void*>(gmem),
                        dims, strides, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, opt.l2_promotion,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) tma_fail("cuTensorMapEncodeTiled failed with CUresult " + std::to_string(int(res)));
}

}  // namespace detail

// Describe a global tensor for TMA (build it with kl::row_major / row_major_strided). The last mode
// is contiguous: TMA can't transpose, so global memory is row-major like the tile. The last two
// modes are the tile's (rows, cols); outer modes (batch, heads, ...) get a box of 1.
// Validation and the driver call follow kernel_lib/include/kl/layout/tma_desc.hpp:100-154.
template <SmemTileType Tile, typename Direction, typename G, int R>
TmaDesc<Tile, Direction, R> make_tma_desc(GmemTensor<G, R> const& g, TmaOptions const& opt = {}) {
  using T = typename Tile::value_type;
  using Box = TmaBox<Tile>;
  static_assert(std::is_same_v<std::remove_cv_t<G>, T>, "the global tensor's element type must match the tile's");
  static_assert(R >= 2 && R <= 5, "TMA tensors have 2 to 5 modes");
  static_assert(!(std::is_same_v<Direction, TmaStoreTag> && std::is_const_v<G>), "a TMA store needs a non-const tensor");
  TmaDesc<Tile, Direction, R> desc{};
  if constexpr (is_fp6<T>) {
    static_assert(std::is_same_v<Direction, TmaLoadTag>, "packed fp6 tensors are read-only here");
    detail::encode_tma_map_u6(&desc.map, tma_swizzle<typename Tile::swizzle>(), Box::inner, Box::outer, g.ptr, R,
                              g.shape, g.stride, opt);
  } else {
    detail::encode_tma_map(&desc.map, tma_dtype<T>(), bits_of<T> / 8, tma_swizzle<typename Tile::swizzle>(),
                           Box::inner, Box::outer, g.ptr, R, g.shape, g.stride, opt);
  }
  return desc;
}

template <SmemTileType Tile, typename G, int R>
TmaLoad<Tile, R> make_tma_load(GmemTensor<G, R> const& g, TmaOptions const& opt = {}) {
  return make_tma_desc<Tile, TmaLoadTag>(g, opt);
}

template <SmemTileType Tile, typename G, int R>
TmaStore<Tile, R> make_tma_store(GmemTensor<G, R> const& g, TmaOptions const& opt = {}) {
  return make_tma_desc<Tile, TmaStoreTag>(g, opt);
}

}  // namespace kl
