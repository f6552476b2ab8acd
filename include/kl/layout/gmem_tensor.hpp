#pragma once

// Row-major views of global memory. Same construction API as
// kernel_lib/include/kl/layout/gmem_tensor.hpp:13-32 (row_major, row_major_strided); the result is a
// kl-owned GmemTensor (pointer + int64 extents and strides, outermost mode first) instead of a
// CuTe tensor.

#include <cstdint>
#include <type_traits>

#include <kl/config.hpp>

namespace kl {

// A rank-R strided view whose last mode is contiguous (stride 1), the only layout TMA can move
// without transposing. Extents and strides are in elements, outermost mode first.
template <typename T, int R>
struct GmemTensor {
  static_assert(R >= 1, "a tensor needs at least one mode");
  using element_type = T;
  using value_type = std::remove_cv_t<T>;
  static constexpr int rank = R;

  T* ptr = nullptr;
  int64_t shape[R] = {};
  int64_t stride[R] = {};

  KL_HOST_DEVICE T* data() const { return ptr; }
  KL_HOST_DEVICE int64_t size(int mode) const { return shape[mode]; }
};

// A compact row-major tensor: the last mode is contiguous, extents listed outermost first, as
// shapes are usually written: row_major(a, M, K), row_major(q, B, H, S, D).
template <typename T, typename... Extents>
KL_HOST_DEVICE GmemTensor<T, int(sizeof...(Extents))> row_major(T* ptr, Extents... extents) {
  static_assert(sizeof...(Extents) >= 1, "row_major needs at least one extent");
  constexpr int R = int(sizeof...(Extents));
  GmemTensor<T, R> g;
  g.ptr = ptr;
  const int64_t ext[R] = {static_cast<int64_t>(extents)...};
  int64_t s = 1;
  for (int i = R - 1; i >= 0; --i) {
    g.shape[i] = ext[i];
    g.stride[i] = s;
    s *= ext[i];
  }
  return g;
}

// A (rows x cols) row-major matrix whose rows are `row_stride` elements apart (row_stride >= cols).
// Example: a fused QKV projection writes [tokens, 3*d]; Q, K and V are column slices:
//   auto k = row_major_strided(qkv + d, tokens, d, 3 * d);
// (For TMA each slice must start 16-byte aligned: d a multiple of 8 for bf16.)
template <typename T>
KL_HOST_DEVICE GmemTensor<T, 2> row_major_strided(T* ptr, int64_t rows, int64_t cols, int64_t row_stride) {
  GmemTensor<T, 2> g;
  g.ptr = ptr;
  g.shape[0] = rows;
  g.shape[1] = cols;
  g.stride[0] = row_stride;
  g.stride[1] = 1;
  return g;
}

}  // namespace kl
