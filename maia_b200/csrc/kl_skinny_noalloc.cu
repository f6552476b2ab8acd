// kl_gemm_skinny_noalloc: the memory-bound small-M GEMM (gemm_skinny_kernel) with its scratch in a
// fixed array of device memory that belongs to this library, so the call itself allocates nothing.
//
// Who needs it: a caller that cannot allocate device memory at call time and cannot hand the
// library a workspace either. Typical cases are plugin interfaces of inference runtimes, where the
// host framework owns every device buffer and only passes a kernel its input and output tensors,
// and serving loops that have a no-allocation rule after warm-up so that no request ever waits on
// (or fails in) the allocator. kl_gemm would allocate its workspace on first use; kl_gemm_ws needs
// the caller to own one. This entry point needs neither.
//
// The price: the array below (16 MiB) is reserved on every GPU that loads libkl_b200.so, for the
// life of the process, and it bounds the problem size: at most 524288 rows of B, and at most
// 16 MiB - 64 KiB of fp32 partial sums, i.e. (ceil(N/128) + #SMs - 1) * token_tile * 512 bytes
// (N = 28672 on 148 SMs: up to 64 tokens per call).

#include <cuda_runtime.h>

#include <atomic>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>

#include <kl/gemm/gemm.hpp>
#include <kl/gemm/skinny_kernel.cuh>
#include <kl_gemm.h>

#include "kl_internal.cuh"

namespace {

using namespace kl::gemm;

// Layout of the scratch array: arrival tickets first, at a fixed size (16 bytes per 128 rows of B,
// room for N <= 4096 * 128 = 524288), then the fp32 partial-sum slots. Because the ticket region
// never moves, no call's partial sums land where another shape's tickets live.
constexpr size_t kScratchBytes = size_t(16) << 20;  // 16 MiB in total
constexpr size_t kTicketBytes = size_t(64) << 10;   // 64 KiB
constexpr size_t kSlotBytes = kScratchBytes - kTicketBytes;
constexpr int kMaxWeightTiles = int(kTicketBytes / 16);

// Device-resident scratch. In host code this name is only a stand-in for the symbol: its device
// address comes from cudaGetSymbolAddress below and is what the kernel receives.
static __device__ __align__(256) unsigned char kl_noalloc_scratch[kScratchBytes];

template <typename InT, typename OutT, int Tok>
using Skinny = SkinnyConfig<InT, OutT, Tok, (Tok == 16 ? 11 : Tok == 32 ? 10 : Tok == 64 ? 8 : Tok == 128 ? 6 : 4)>;

// Device address of kl_noalloc_scratch, per device. Cleared by kl_release_workspaces, so that a
// caller who resets a device (which unloads the module holding the array) can look it up again.
std::mutex g_mutex;
unsigned char* g_scratch[64] = {};

// Once per device, with that device current: resolve the array's device address. No allocation
// happens here (the array exists since the library was loaded).
kl_status setup_device(int dev, unsigned char** out) {
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, kl_noalloc_scratch);
    if (e != cudaSuccess) return kl::capi::cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_scratch[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_scratch[dev];
  return KL_OK;
}

// Encodes the tensor maps first (they can reject the call), then queues the ticket clear and the
// kernel: a rejected call leaves nothing on the stream.
template <class Cfg>
kl_status launch(kl_gemm_desc const& d, int n_tiles, int k_blocks, int grid, unsigned char* scratch,
                 cudaStream_t stream) {
  using InT = typename Cfg::in_type;
  int* status = nullptr;
  kl_status s = kl::capi::device_status_ptr(&status);
  if (s != KL_OK) return s;
  static std::atomic<int> configured[64];  // per device; idempotent, so concurrent first calls are fine
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return kl::capi::fail(KL_ERR_NOT_SUPPORTED, "device index above 63");
  if (!configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_skinny_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(Cfg::kSmemBytes));
    if (e != cudaSuccess) return kl::capi::cuda_fail(e, "cudaFuncSetAttribute(no-alloc skinny)");
    configured[dev].store(1, std::memory_order_release);
  }
  SkinnyParams p{};
  p.map_w = kl::make_tma_load<typename Cfg::WTile>(kl::row_major_strided(static_cast<InT const*>(d.b), d.n, d.k, d.ldb)).map;
  p.map_x = kl::make_tma_load<typename Cfg::XTile>(kl::row_major_strided(static_cast<InT const*>(d.a), d.m, d.k, d.lda)).map;
  SkinnyArgs& a = p.args;
  a.m = int(d.m);
  a.n = int(d.n);
  a.k = int(d.k);
  a.n_tiles = n_tiles;
  a.k_blocks = k_blocks;
  a.total_units = (long long)n_tiles * k_blocks;
  a.grid = grid;
  a.alpha = d.alpha;
  a.scale_a = d.scale_a;
  a.scale_b = d.scale_b;
  a.c = d.c;
  a.ldc = d.ldc;
  a.tickets = reinterpret_cast<int*>(scratch);
  a.slots = reinterpret_cast<float*>(scratch + kTicketBytes);
  a.status = status;
  a.timeout_ns = kl::capi::wait_timeout_ns();
  a.prefetch = d.prefetch > 0 ? d.prefetch : d.prefetch < 0 ? 0 : kDefaultPrefetchSkinny;
  a.c_reduce = d.c_reduce;
  // The arrival tickets this call uses must start at zero. The kernel re-arms them when it
  // finishes, but a kernel stopped by a timed-out wait would leave them mid-count, and the array
  // keeps whatever the last call left; so clear them on the stream, ahead of the kernel. The
  // partial-sum slots need no clearing: each is written before it is read.
  cudaError_t e = cudaMemsetAsync(scratch, 0, size_t(n_tiles) * 16, stream);
  if (e != cudaSuccess) return kl::capi::cuda_fail(e, "cudaMemsetAsync(no-alloc tickets)");
  gemm_skinny_kernel<Cfg><<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(p);
  e = cudaGetLastError();
  return e == cudaSuccess ? KL_OK : kl::capi::cuda_fail(e, "no-alloc skinny launch");
}

template <typename InT, typename OutT>
kl_status dispatch(kl_gemm_desc const& d, int tok, int n_tiles, int k_blocks, int grid, unsigned char* scratch,
                   cudaStream_t stream) {
  switch (tok) {
    case 16: return launch<Skinny<InT, OutT, 16>>(d, n_tiles, k_blocks, grid, scratch, stream);
    case 32: return launch<Skinny<InT, OutT, 32>>(d, n_tiles, k_blocks, grid, scratch, stream);
    case 64: return launch<Skinny<InT, OutT, 64>>(d, n_tiles, k_blocks, grid, scratch, stream);
    case 128: return launch<Skinny<InT, OutT, 128>>(d, n_tiles, k_blocks, grid, scratch, stream);
    default: return launch<Skinny<InT, OutT, 256>>(d, n_tiles, k_blocks, grid, scratch, stream);
  }
}

}  // namespace

namespace kl::capi {
void forget_noalloc_scratch() {
  std::lock_guard<std::mutex> lock(g_mutex);
  for (auto& p : g_scratch) p = nullptr;
}
}  // namespace kl::capi

extern "C" kl_status kl_gemm_skinny_noalloc(const kl_gemm_desc* d, void* stream_ptr) {
  using kl::capi::fail;
  if (d == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null descriptor");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (d->algo != KL_ALGO_AUTO && d->algo != KL_ALGO_SKINNY)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_skinny_noalloc runs the skinny kernel only (algo AUTO or SKINNY)");
  if (d->m <= 0 || d->n <= 0 || d->k <= 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_skinny_noalloc: m, n and k must be positive");
  if (d->m > 256) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_skinny_noalloc: at most 256 rows of A");
  if (d->batch > 1) return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_skinny_noalloc: one problem per call");
  if (d->m_block_group != nullptr || d->block_scale != 0)
    return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_skinny_noalloc: plain (not grouped, not block-scaled) GEMMs only");
  if (d->a_major != 0 || d->b_major != 0 || (d->swizzle != 0 && d->swizzle != 128))
    return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_skinny_noalloc: K-major operands with the 128-byte swizzle only");
  if (d->c_reduce != 0 && d->c_reduce != 1)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_skinny_noalloc: c_reduce must be 0 (store) or 1 (add)");
  if (d->n > INT32_MAX || d->k > INT32_MAX)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_skinny_noalloc: extents must fit in 32 bits");
  if (d->a == nullptr || d->b == nullptr || d->c == nullptr)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_skinny_noalloc: null A, B or C");
  if (d->ldc < d->n) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_skinny_noalloc: ldc < n");
  if (reinterpret_cast<uintptr_t>(d->c) % (d->c_type == KL_F32 ? 4 : 2) != 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_skinny_noalloc: C is not aligned to its element size");
  // Variant 2 (two 128-row weight boxes per stage) has no no-alloc build; 0 and 1 both name the
  // one-box kernel that kl_gemm runs for them.
  if (d->variant != 0 && d->variant != 1)
    return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_skinny_noalloc: variant must be 0 or 1");
  const bool bf16_bf16 = d->ab_type == KL_BF16 && d->c_type == KL_BF16;
  const bool bf16_f32 = d->ab_type == KL_BF16 && d->c_type == KL_F32;
  const bool e4m3_bf16 = d->ab_type == KL_E4M3 && d->c_type == KL_BF16;
  if (!bf16_bf16 && !bf16_f32 && !e4m3_bf16)
    return fail(KL_ERR_NOT_SUPPORTED,
                "kl_gemm_skinny_noalloc supports (A/B, C) = (bf16, bf16), (bf16, f32), (e4m3, bf16)");

  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return kl::capi::cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(KL_ERR_NOT_SUPPORTED, "device index above 63");
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return kl::capi::cuda_fail(e, "cudaDeviceGetAttribute");

  // The same plan as the allocating path: 128-row weight tiles, 128-byte K-blocks, one unit range
  // per CTA, token tile rounded up to 16 or a multiple of 32.
  const int elem = d->ab_type == KL_E4M3 ? 1 : 2;
  const int tok = d->m <= 16 ? 16 : d->m <= 32 ? 32 : d->m <= 64 ? 64 : d->m <= 128 ? 128 : 256;
  const int n_tiles = int((d->n + 127) / 128);
  const int k_blocks = int((d->k + 128 / elem - 1) / (128 / elem));
  const long long total = (long long)n_tiles * k_blocks;
  const int cap = d->max_ctas > 0 ? std::min(d->max_ctas, sms) : skinny_default_ctas(sms);
  const int grid = int(std::min<long long>(cap, total));
  const size_t slots = size_t(n_tiles + grid - 1) * size_t(tok) * 128 * sizeof(float);
  if (n_tiles > kMaxWeightTiles)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_skinny_noalloc: B has " + std::to_string(d->n) +
                                             " rows; the fixed scratch holds counters for at most " +
                                             std::to_string(kMaxWeightTiles * 128));
  if (slots > kSlotBytes)
    return fail(KL_ERR_INVALID_ARGUMENT,
                "kl_gemm_skinny_noalloc: needs " + std::to_string(slots) + " bytes of partial sums (" +
                    std::to_string(n_tiles) + " weight tiles, " + std::to_string(tok) +
                    "-token tile); the fixed scratch has " + std::to_string(kSlotBytes) +
                    " (use kl_gemm / kl_gemm_ws, or fewer tokens per call)");

  unsigned char* scratch = nullptr;
  kl_status s = setup_device(dev, &scratch);
  if (s != KL_OK) return s;
  try {
    if (bf16_bf16) return dispatch<kl::bf16, kl::bf16>(*d, tok, n_tiles, k_blocks, grid, scratch, stream);
    if (bf16_f32) return dispatch<kl::bf16, float>(*d, tok, n_tiles, k_blocks, grid, scratch, stream);
    return dispatch<kl::e4m3, kl::bf16>(*d, tok, n_tiles, k_blocks, grid, scratch, stream);
  } catch (std::invalid_argument const& ex) {
    return fail(KL_ERR_INVALID_ARGUMENT, ex.what());
  }
}
