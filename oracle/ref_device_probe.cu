// GPU-side reference probes, compiled from the reference's OWN headers (kernel_lib/include/kl)
// against CUTLASS/CuTe 4.5.0 into oracle/_ref/libkl_ref.so. TEST INFRASTRUCTURE ONLY: the GPU
// tests load it to compare libkl_b200.so's descriptors and tensor maps with the reference's.
//
//  kl_ref_umma_descs  -- the reference's device kl::umma_desc for every (row block, k-block) of a
//                        tile at a real shared address, plus CuTe's own iterator-based descriptor
//                        (the comparison kernel_lib/tests/unit/test_umma_desc.cu:18-39 makes).
//  kl_ref_tma_desc    -- the reference's kl::make_tma_load map for a row-major tensor, and CuTe's
//                        make_tma_copy map for the same memory (test_tma_desc.cu:24-29).
//  kl_ref_tma_error   -- the reference's error message for an invalid global layout
//                        (test_tma_desc.cu:97-118).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

#include <cute/atom/copy_traits_sm90_tma.hpp>
#include <cute/tensor.hpp>
#include <kl/kl.hpp>

namespace {

template <int BlockRows, typename Tile>
__device__ uint64_t cute_desc(Tile const& tile, int m, int k) {
  using T = typename Tile::value_type;
  auto part = cute::zipped_divide(tile.tensor(), cute::Shape<cute::Int<BlockRows>, cute::Int<kl::mma_k<T>>>{});
  auto descs = cute::make_tensor<cute::UMMA::smem_desc<cute::UMMA::Major::K>>(part);
  return descs(0, cute::make_coord(m, k));
}

template <typename Tile, int BlockRows>
__global__ void desc_kernel(uint64_t* kl_out, uint64_t* ref_out, uint32_t* base_out) {
  extern __shared__ __align__(1024) unsigned char smem[];
  auto& tile = *reinterpret_cast<Tile*>(smem);
  constexpr int nk = kl::num_k_blocks<Tile>;
  for (int m = 0; m < Tile::rows / BlockRows; ++m)
    for (int k = 0; k < nk; ++k) {
      kl_out[m * nk + k] = kl::umma_desc(tile, k, m * BlockRows);
      ref_out[m * nk + k] = cute_desc<BlockRows>(tile, m, k);
    }
  *base_out = tile.smem_u32();
}

template <typename Tile, int BlockRows>
int run_desc(uint64_t* h_kl, uint64_t* h_ref, uint32_t* h_base, int* count) {
  constexpr int n = (Tile::rows / BlockRows) * kl::num_k_blocks<Tile>;
  uint64_t *d_kl = nullptr, *d_ref = nullptr;
  uint32_t* d_base = nullptr;
  if (cudaMalloc(&d_kl, n * 8) || cudaMalloc(&d_ref, n * 8) || cudaMalloc(&d_base, 4)) return 1;
  constexpr int smem = sizeof(Tile);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(desc_kernel<Tile, BlockRows>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  desc_kernel<Tile, BlockRows><<<1, 1, smem>>>(d_kl, d_ref, d_base);
  int rc = cudaDeviceSynchronize() != cudaSuccess;
  if (!rc) {
    cudaMemcpy(h_kl, d_kl, n * 8, cudaMemcpyDeviceToHost);
    cudaMemcpy(h_ref, d_ref, n * 8, cudaMemcpyDeviceToHost);
    cudaMemcpy(h_base, d_base, 4, cudaMemcpyDeviceToHost);
    *count = n;
  }
  cudaFree(d_kl);
  cudaFree(d_ref);
  cudaFree(d_base);
  return rc;
}

template <typename Tile>
int tma_maps(void* gmem, int64_t rows, int64_t cols, void* kl_map, void* cute_map) {
  using T = typename Tile::value_type;
  T* p = static_cast<T*>(gmem);
  auto g = kl::row_major(p, rows, cols);
  auto ours = kl::make_tma_load<Tile>(g);
  std::memcpy(kl_map, &ours.map, sizeof(CUtensorMap));
  if (cute_map) {
    if constexpr (Tile::rows <= 256) {
      auto theirs = cute::make_tma_copy(cute::SM90_TMA_LOAD{}, g, typename Tile::layout_type{});
      std::memcpy(cute_map, theirs.get_tma_descriptor(), sizeof(CUtensorMap));
    } else {
      std::memset(cute_map, 0, sizeof(CUtensorMap));
    }
  }
  return 0;
}

}  // namespace

// Cases shared with tests/test_descriptors_gpu.py (same numbering).
extern "C" int kl_ref_umma_descs(int c, uint64_t* h_kl, uint64_t* h_ref, uint32_t* base, int* count) {
  using kl::SmemTile;
  switch (c) {
    case 0: return run_desc<SmemTile<kl::bf16, 128, 64>, 128>(h_kl, h_ref, base, count);
    case 1: return run_desc<SmemTile<kl::bf16, 256, 64>, 256>(h_kl, h_ref, base, count);
    case 2: return run_desc<SmemTile<kl::bf16, 128, 128>, 128>(h_kl, h_ref, base, count);
    case 3: return run_desc<SmemTile<kl::bf16, 128, 64, kl::Swizzle64B>, 128>(h_kl, h_ref, base, count);
    case 4: return run_desc<SmemTile<kl::bf16, 128, 32, kl::Swizzle32B>, 128>(h_kl, h_ref, base, count);
    case 5: return run_desc<SmemTile<int8_t, 128, 128>, 128>(h_kl, h_ref, base, count);
    case 6: return run_desc<SmemTile<kl::e4m3, 128, 128>, 128>(h_kl, h_ref, base, count);
    case 7: return run_desc<SmemTile<float, 128, 32>, 128>(h_kl, h_ref, base, count);
    case 8: return run_desc<SmemTile<kl::bf16, 256, 64>, 128>(h_kl, h_ref, base, count);
    case 9: return run_desc<SmemTile<kl::bf16, 512, 64>, 256>(h_kl, h_ref, base, count);
    case 10: return run_desc<SmemTile<kl::bf16, 128, 128>, 64>(h_kl, h_ref, base, count);
    case 11: return run_desc<SmemTile<kl::bf16, 256, 64, kl::Swizzle64B>, 128>(h_kl, h_ref, base, count);
    case 12: return run_desc<SmemTile<int8_t, 256, 128>, 128>(h_kl, h_ref, base, count);
    case 13: return run_desc<SmemTile<kl::e4m3, 256, 128>, 128>(h_kl, h_ref, base, count);
    default: return 2;
  }
}

extern "C" int kl_ref_tma_desc(int c, void* gmem, int64_t rows, int64_t cols, void* kl_map, void* cute_map) {
  using kl::SmemTile;
  try {
    switch (c) {
      case 0: return tma_maps<SmemTile<kl::bf16, 128, 64>>(gmem, rows, cols, kl_map, cute_map);
      case 1: return tma_maps<SmemTile<kl::bf16, 256, 64>>(gmem, rows, cols, kl_map, cute_map);
      case 2: return tma_maps<SmemTile<int8_t, 128, 128>>(gmem, rows, cols, kl_map, cute_map);
      case 3: return tma_maps<SmemTile<kl::bf16, 128, 128>>(gmem, rows, cols, kl_map, cute_map);
      case 4: return tma_maps<SmemTile<kl::bf16, 128, 32, kl::Swizzle64B>>(gmem, rows, cols, kl_map, cute_map);
      case 5: return tma_maps<SmemTile<kl::bf16, 128, 16, kl::Swizzle32B>>(gmem, rows, cols, kl_map, cute_map);
      case 6: return tma_maps<SmemTile<kl::bf16, 128, 8, kl::SwizzleNone>>(gmem, rows, cols, kl_map, cute_map);
      case 7: return tma_maps<SmemTile<kl::bf16, 512, 64>>(gmem, rows, cols, kl_map, cute_map);
      case 8: return tma_maps<SmemTile<kl::e4m3, 128, 128>>(gmem, rows, cols, kl_map, cute_map);
      case 9: return tma_maps<SmemTile<float, 32, 32>>(gmem, rows, cols, kl_map, cute_map);
      case 10: return tma_maps<SmemTile<kl::bf16, 32, 64>>(gmem, rows, cols, kl_map, cute_map);
      default: return 2;
    }
  } catch (std::exception const&) {
    return 3;
  }
}

// Batched rank-3 case of test_tma_desc.cu:72-83: (B, M, K) row-major, 128x64 bf16 tile.
extern "C" int kl_ref_tma_desc_batched(void* gmem, int64_t b, int64_t m, int64_t k, void* kl_map, void* cute_map) {
  auto* p = static_cast<kl::bf16*>(gmem);
  using Tile = kl::SmemTile<kl::bf16, 128, 64>;
  auto ours = kl::make_tma_load<Tile>(kl::row_major(p, b, m, k));
  std::memcpy(kl_map, &ours.map, sizeof(CUtensorMap));
  auto ref = cute::make_tensor(cute::make_gmem_ptr(p), cute::make_shape(m, k, b), cute::make_stride(k, cute::_1{}, m * k));
  auto theirs = cute::make_tma_copy(cute::SM90_TMA_LOAD{}, ref, typename Tile::layout_type{});
  std::memcpy(cute_map, theirs.get_tma_descriptor(), sizeof(CUtensorMap));
  return 0;
}

// Rank-4 and rank-5 tensors (two or three outer modes), row-major: the reference's
// make_tma_load<bf16 128x64>(row_major(p, extents...)) and CuTe's make_tma_copy of the same tensor
// with the outer modes last (the order CuTe tiles in).
extern "C" int kl_ref_tma_desc_rank(void* gmem, int rank, const int64_t* e, void* kl_map, void* cute_map) {
  auto* p = static_cast<kl::bf16*>(gmem);
  using Tile = kl::SmemTile<kl::bf16, 128, 64>;
  if (rank == 4) {
    auto ours = kl::make_tma_load<Tile>(kl::row_major(p, e[0], e[1], e[2], e[3]));
    std::memcpy(kl_map, &ours.map, sizeof(CUtensorMap));
    const int64_t mk = e[2] * e[3];
    auto ref = cute::make_tensor(cute::make_gmem_ptr(p), cute::make_shape(e[2], e[3], e[1], e[0]),
                                 cute::make_stride(e[3], cute::_1{}, mk, mk * e[1]));
    auto theirs = cute::make_tma_copy(cute::SM90_TMA_LOAD{}, ref, typename Tile::layout_type{});
    std::memcpy(cute_map, theirs.get_tma_descriptor(), sizeof(CUtensorMap));
    return 0;
  }
  if (rank == 5) {
    auto ours = kl::make_tma_load<Tile>(kl::row_major(p, e[0], e[1], e[2], e[3], e[4]));
    std::memcpy(kl_map, &ours.map, sizeof(CUtensorMap));
    const int64_t mk = e[3] * e[4];
    auto ref = cute::make_tensor(cute::make_gmem_ptr(p), cute::make_shape(e[3], e[4], e[2], e[1], e[0]),
                                 cute::make_stride(e[4], cute::_1{}, mk, mk * e[2], mk * e[2] * e[1]));
    auto theirs = cute::make_tma_copy(cute::SM90_TMA_LOAD{}, ref, typename Tile::layout_type{});
    std::memcpy(cute_map, theirs.get_tma_descriptor(), sizeof(CUtensorMap));
    return 0;
  }
  return 1;
}

// The reference's message for make_tma_load<bf16 128x64> on (ptr, rows, cols, row_stride), or "".
extern "C" int kl_ref_tma_error(void* gmem, int64_t rows, int64_t cols, int64_t row_stride, char* msg, int cap) {
  using Tile = kl::SmemTile<kl::bf16, 128, 64>;
  msg[0] = 0;
  try {
    (void)kl::make_tma_load<Tile>(kl::row_major_strided(static_cast<kl::bf16*>(gmem), rows, cols, row_stride));
  } catch (std::invalid_argument const& e) {
    std::strncpy(msg, e.what(), cap - 1);
    msg[cap - 1] = 0;
    return 1;
  }
  return 0;
}
