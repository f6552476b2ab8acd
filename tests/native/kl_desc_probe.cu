// Test helper (not part of libkl_b200.so): evaluates kl's device-side descriptor code,
// kl::umma_desc(tile, k_block, row) from <kl/layout/umma_desc.hpp>, on a tile at a real shared
// address, so the GPU tests can compare it with the reference's device code
// (oracle/_ref/libkl_ref.so, case numbers shared with oracle/ref_device_probe.cu).
#include <cuda_runtime.h>

#include <cstdint>

#include <kl/kl.hpp>

namespace {

template <typename Tile, int BlockRows>
__global__ void desc_kernel(uint64_t* out, uint32_t* base_out) {
  extern __shared__ __align__(1024) unsigned char smem[];
  auto& tile = *reinterpret_cast<Tile*>(smem);
  constexpr int nk = kl::num_k_blocks<Tile>;
  for (int m = 0; m < Tile::rows / BlockRows; ++m)
    for (int k = 0; k < nk; ++k) out[m * nk + k] = kl::umma_desc(tile, k, m * BlockRows);
  *base_out = tile.smem_u32();
}

template <typename Tile, int BlockRows>
int run(uint64_t* h_out, uint32_t* h_base, int* count) {
  constexpr int n = (Tile::rows / BlockRows) * kl::num_k_blocks<Tile>;
  uint64_t* d_out = nullptr;
  uint32_t* d_base = nullptr;
  if (cudaMalloc(&d_out, n * 8) != cudaSuccess || cudaMalloc(&d_base, 4) != cudaSuccess) return 1;
  constexpr int smem = sizeof(Tile);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(desc_kernel<Tile, BlockRows>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  desc_kernel<Tile, BlockRows><<<1, 1, smem>>>(d_out, d_base);
  int rc = cudaDeviceSynchronize() != cudaSuccess;
  if (!rc) {
    cudaMemcpy(h_out, d_out, n * 8, cudaMemcpyDeviceToHost);
    cudaMemcpy(h_base, d_base, 4, cudaMemcpyDeviceToHost);
    *count = n;
  }
  cudaFree(d_out);
  cudaFree(d_base);
  return rc;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int kl_test_umma_descs(int c, uint64_t* out, uint32_t* base,
                                                                          int* count) {
  using kl::SmemTile;
  switch (c) {
    case 0: return run<SmemTile<kl::bf16, 128, 64>, 128>(out, base, count);
    case 1: return run<SmemTile<kl::bf16, 256, 64>, 256>(out, base, count);
    case 2: return run<SmemTile<kl::bf16, 128, 128>, 128>(out, base, count);
    case 3: return run<SmemTile<kl::bf16, 128, 64, kl::Swizzle64B>, 128>(out, base, count);
    case 4: return run<SmemTile<kl::bf16, 128, 32, kl::Swizzle32B>, 128>(out, base, count);
    case 5: return run<SmemTile<int8_t, 128, 128>, 128>(out, base, count);
    case 6: return run<SmemTile<kl::e4m3, 128, 128>, 128>(out, base, count);
    case 7: return run<SmemTile<float, 128, 32>, 128>(out, base, count);
    case 8: return run<SmemTile<kl::bf16, 256, 64>, 128>(out, base, count);
    case 9: return run<SmemTile<kl::bf16, 512, 64>, 256>(out, base, count);
    case 10: return run<SmemTile<kl::bf16, 128, 128>, 64>(out, base, count);
    case 11: return run<SmemTile<kl::bf16, 256, 64, kl::Swizzle64B>, 128>(out, base, count);
    case 12: return run<SmemTile<int8_t, 256, 128>, 128>(out, base, count);
    case 13: return run<SmemTile<kl::e4m3, 256, 128>, 128>(out, base, count);
    default: return 2;
  }
}
