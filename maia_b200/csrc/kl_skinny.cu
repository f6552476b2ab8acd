// KL_ALGO_SKINNY: dispatch, workspace sizing and launch of the memory-bound small-M kernel
// (include/kl/gemm/skinny_kernel.cuh).

#include <cuda_runtime.h>

#include <atomic>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>

#include <kl/gemm/gemm.hpp>
#include <kl/gemm/skinny_kernel.cuh>

#include "kl_internal.cuh"

namespace kl::capi {

namespace {

using namespace kl::gemm;

constexpr size_t kAlign = 256;
constexpr int kDefaultSkinnySub = 1;
size_t round_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

int token_tile(int64_t m) { return m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 128 : 256; }

// Stages that fit next to the tile sizes (weights 16 KB per 128-row box, activations tok x 128 B
// per stage) in ~200 KB of shared memory.
constexpr int skinny_stages(int tok, int sub) {
  return sub == 1 ? (tok == 16 ? 11 : tok == 32 ? 10 : tok == 64 ? 8 : tok == 128 ? 6 : 4)
                  : (tok <= 32 ? 6 : tok == 64 ? 5 : 4);
}
template <typename InT, typename OutT, int Tok, int Sub>
using Skinny = SkinnyConfig<InT, OutT, Tok, skinny_stages(Tok, Sub), Sub>;

// Block-scaled (SfVec V): the bf16/fp8 stage counts, fewer where the scale atoms (512 bytes per 128
// rows and atom along K) push a stage past the ~200 KB budget. (A 216 KB budget, one stage more at
// 16, 32 and 128 tokens, measured the same on B200: MXFP8 16 tokens 40.9 vs 41.0 us.)
constexpr int skinny_mx_stages(int tok, bool fp4, int vec) {
  const int atoms_k = (fp4 ? 256 : 128) / (4 * vec);
  const int stage = 16384 + tok * 128 + 512 * atoms_k * (1 + (tok + 127) / 128);
  const int fit = 204800 / stage;
  return fit < skinny_stages(tok, 1) ? fit : skinny_stages(tok, 1);
}
template <typename InT, typename OutT, int Tok, int V>
using SkinnyMx = SkinnyConfig<InT, OutT, Tok, skinny_mx_stages(Tok, std::is_same_v<InT, kl::e2m1x2>, V), 1, V>;

struct Plan {
  int tok = 0;
  int sub = 1;  // 128-row weight boxes per tile
  int n_tiles = 0, k_blocks = 0, grid = 0;
  long long total = 0;
  size_t ticket_bytes = 0, slot_bytes = 0;
};

kl_status make_plan(kl_gemm_desc const& d, Plan* p) {
  if (d.m > 256) return fail(KL_ERR_INVALID_ARGUMENT, "KL_ALGO_SKINNY handles at most 256 rows of A");
  if (d.m <= 0 || d.n <= 0 || d.k <= 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: m, n and k must be positive");
  if (d.n > INT32_MAX || d.k > INT32_MAX) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: extents must fit in 32 bits");
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  // Elements per 128-byte K-block: 64 (16-bit), 128 (8-bit, and fp6 whose tiles hold a byte per
  // element), 256 (packed fp4).
  const bool one_byte = d.ab_type == KL_E4M3 || d.ab_type == KL_E5M2 || d.ab_type == KL_E3M2 || d.ab_type == KL_E2M3;
  const int block_k = d.ab_type == KL_E2M1 ? 256 : one_byte ? 128 : 64;
  if (d.block_scale != 0 && d.m > 128)
    return fail(KL_ERR_INVALID_ARGUMENT, "KL_ALGO_SKINNY with block scaling handles at most 128 rows of A");
  p->tok = token_tile(d.m);
  p->sub = d.variant == 2 ? 2 : d.variant == 1 ? 1 : kDefaultSkinnySub;
  if (d.block_scale != 0) p->sub = 1;
  if (p->sub == 2 && p->tok > 128) p->sub = 1;  // two 256-token accumulators would not fit in TMEM
  if (d.variant < 0 || d.variant > 2) return fail(KL_ERR_INVALID_ARGUMENT, "KL_ALGO_SKINNY variant must be 0, 1 or 2");
  p->n_tiles = int((d.n + 128 * p->sub - 1) / (128 * p->sub));
  p->k_blocks = int((d.k + block_k - 1) / block_k);
  p->total = (long long)p->n_tiles * p->k_blocks;
  // Packed fp6 brings 3/4 of fp8's bytes per shared-memory stage (the 16U6 tiles hold a byte per
  // element), so a latency-bound weight stream keeps fewer bytes in flight per CTA: at 16 tokens it
  // runs on every SM. Measured on B200 (N = 28672, K = 8192, MXFP6): 16 tokens 36.6 us with 148
  // CTAs vs 40.8 us with 112; 64 tokens 43.2 us both; 128 tokens 112 CTAs ahead (47.3 vs 53.3 us).
  const bool fp6 = d.ab_type == KL_E3M2 || d.ab_type == KL_E2M3;
  int cap = d.max_ctas > 0 ? std::min(d.max_ctas, sms) : (fp6 && d.m <= 16) ? sms : skinny_default_ctas(sms);
  p->grid = int(std::min<long long>(cap, p->total));
  p->ticket_bytes = round_up(size_t(p->n_tiles) * 4 * sizeof(int));
  p->slot_bytes = size_t(p->n_tiles + p->grid - 1) * size_t(p->tok) * 128 * p->sub * sizeof(float);
  return KL_OK;
}

template <class Cfg>
kl_status launch(kl_gemm_desc const& d, Plan const& pl, void* ws, cudaStream_t stream) {
  using InT = typename Cfg::in_type;
  int* status = nullptr;
  kl_status s = device_status_ptr(&status);
  if (s != KL_OK) return s;
  static std::atomic<int> configured[64];  // per device; idempotent, so concurrent first calls are fine
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_skinny_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(Cfg::kSmemBytes));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(skinny)");
    configured[dev].store(1, std::memory_order_release);
  }
  SkinnyParams p{};
  // Packed fp4: K and the pitches count elements, the maps bytes.
  constexpr int64_t pack = Cfg::kFp4 ? 2 : 1;
  if (d.k % pack != 0 || d.lda % pack != 0 || d.ldb % pack != 0)
    throw std::invalid_argument("kl::gemm: packed fp4 needs even K and leading dimensions");
  p.map_w = make_tma_load<typename Cfg::WTile>(
                row_major_strided(static_cast<InT const*>(d.b), d.n, d.k / pack, d.ldb / pack)).map;
  p.map_x = make_tma_load<typename Cfg::XTile>(
                row_major_strided(static_cast<InT const*>(d.a), d.m, d.k / pack, d.lda / pack)).map;
  if constexpr (Cfg::kMx) {
    if (d.sfa == nullptr || d.sfb == nullptr) throw std::invalid_argument("kl::gemm: block scaling needs scales of A and B");
    const int64_t kb = (d.k + 4 * Cfg::kSfVecSize - 1) / (4 * Cfg::kSfVecSize);
    auto sf_map = [&](CUtensorMap* map, void const* ptr, int64_t rows) {
      const int64_t shape[3] = {(rows + 127) / 128, kb, 128};
      const int64_t stride[3] = {kb * 128, 128, 1};
      kl::detail::encode_tma_map(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, CU_TENSOR_MAP_SWIZZLE_NONE, 128,
                                 uint32_t(Cfg::kSfAtomsK), ptr, 3, shape, stride, TmaOptions{});
    };
    sf_map(&p.map_sfw, d.sfb, d.n);
    sf_map(&p.map_sfx, d.sfa, d.m);
  }
  if (d.ldc < d.n) throw std::invalid_argument("kl_gemm: ldc < n");
  if (reinterpret_cast<uintptr_t>(d.c) % (d.c_type == KL_F32 ? 4 : 2) != 0)
    throw std::invalid_argument("kl_gemm: C is not aligned to its element size");
  SkinnyArgs& a = p.args;
  a.m = int(d.m);
  a.n = int(d.n);
  a.k = int(d.k);
  a.n_tiles = pl.n_tiles;
  a.k_blocks = pl.k_blocks;
  a.total_units = pl.total;
  a.grid = pl.grid;
  a.alpha = d.alpha;
  a.scale_a = d.scale_a;
  a.scale_b = d.scale_b;
  a.c = d.c;
  a.ldc = d.ldc;
  a.tickets = static_cast<int*>(ws);
  a.slots = reinterpret_cast<float*>(static_cast<char*>(ws) + pl.ticket_bytes);
  a.status = status;
  a.timeout_ns = wait_timeout_ns();
  a.prefetch = d.prefetch > 0 ? d.prefetch : d.prefetch < 0 ? 0 : kDefaultPrefetchSkinny;
  a.c_reduce = d.c_reduce;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(unsigned(pl.grid), 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  if (d.launch_overlap >= 0) {  // programmatic dependent launch (the kernel waits before any global access)
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_skinny_kernel<Cfg>, p);
  return e == cudaSuccess ? KL_OK : cuda_fail(e, "skinny launch");
}

template <typename InT, typename OutT>
kl_status dispatch_tok(kl_gemm_desc const& d, Plan const& pl, void* ws, cudaStream_t stream) {
  if (pl.sub == 2) {
    switch (pl.tok) {
      case 16: return launch<Skinny<InT, OutT, 16, 2>>(d, pl, ws, stream);
      case 32: return launch<Skinny<InT, OutT, 32, 2>>(d, pl, ws, stream);
      case 64: return launch<Skinny<InT, OutT, 64, 2>>(d, pl, ws, stream);
      default: return launch<Skinny<InT, OutT, 128, 2>>(d, pl, ws, stream);
    }
  }
  switch (pl.tok) {
    case 16: return launch<Skinny<InT, OutT, 16, 1>>(d, pl, ws, stream);
    case 32: return launch<Skinny<InT, OutT, 32, 1>>(d, pl, ws, stream);
    case 64: return launch<Skinny<InT, OutT, 64, 1>>(d, pl, ws, stream);
    case 128: return launch<Skinny<InT, OutT, 128, 1>>(d, pl, ws, stream);
    default: return launch<Skinny<InT, OutT, 256, 1>>(d, pl, ws, stream);
  }
}

template <typename InT, typename OutT, int V>
kl_status dispatch_tok_mx(kl_gemm_desc const& d, Plan const& pl, void* ws, cudaStream_t stream) {
  switch (pl.tok) {
    case 16: return launch<SkinnyMx<InT, OutT, 16, V>>(d, pl, ws, stream);
    case 32: return launch<SkinnyMx<InT, OutT, 32, V>>(d, pl, ws, stream);
    case 64: return launch<SkinnyMx<InT, OutT, 64, V>>(d, pl, ws, stream);
    default: return launch<SkinnyMx<InT, OutT, 128, V>>(d, pl, ws, stream);
  }
}

// Library-owned workspace for kl_gemm (no caller workspace): one per device, grown on demand.
// Layout per call: tickets in [0, ticket_bytes), slots after them. A call leaves its own ticket
// range at zero but writes slots right after it, so a later call with more weight tiles (a longer
// ticket range) would find slot data where it expects zero tickets: `clean` tracks the prefix
// known to hold only zero tickets, and the gap is cleared on the stream before such a call.
// Calls that overlap on one device share the buffer.
struct DeviceWorkspace {
  void* ptr = nullptr;
  size_t bytes = 0;
  size_t clean = 0;
  bool dirty = false;
};
std::mutex g_ws_mutex;
DeviceWorkspace g_ws[64];

kl_status library_workspace(size_t need, size_t tickets, cudaStream_t stream, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(KL_ERR_NOT_SUPPORTED, "device index above 63");
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  DeviceWorkspace& w = g_ws[dev];
  if (w.bytes < need) {
    if (w.ptr) {
      e = cudaDeviceSynchronize();  // the old buffer may still be in use
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
      cudaFree(w.ptr);
      w.ptr = nullptr;
      w.bytes = 0;
    }
    e = cudaMalloc(&w.ptr, need);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(skinny workspace)");
    e = cudaMemset(w.ptr, 0, need);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(skinny workspace)");
    w.bytes = need;
    w.clean = need;
  } else if (w.dirty) {
    e = cudaMemset(w.ptr, 0, w.bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(skinny workspace)");
    w.clean = w.bytes;
  }
  w.dirty = false;
  if (tickets > w.clean) {
    e = cudaMemsetAsync(static_cast<char*>(w.ptr) + w.clean, 0, tickets - w.clean, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(skinny tickets)");
  }
  w.clean = tickets;  // this call writes slots from here on
  *out = w.ptr;
  return KL_OK;
}

}  // namespace

kl_status release_skinny_workspaces() {
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  for (int dev = 0; dev < 64; ++dev) {
    DeviceWorkspace& w = g_ws[dev];
    if (w.ptr == nullptr) continue;
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();  // no launch may still use it
    if (e == cudaSuccess) e = cudaFree(w.ptr);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "kl_release_workspaces (skinny)");
    w = DeviceWorkspace{};
  }
  return KL_OK;
}

void mark_workspace_dirty(int device) {
  if (device < 0 || device >= 64) return;
  tile_workspaces_mark_dirty(device);
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  g_ws[device].dirty = true;
}

int choose_algo(kl_gemm_desc const& d) {
  // A CTA pair needs at least 256 rows to fill its tile. Below that the weights dominate traffic.
  // Measured on B200 at N = 28672, K = 8192 (bf16): the stream-K skinny kernel reads 6.23 TB/s at
  // 64 rows (the one-CTA tile kernel 5.90), but at 128 rows its MMAs no longer hide behind the
  // stream and the one-CTA tile kernel (112 weight bands of 256 rows) is ahead, 5.88 vs 5.68 TB/s.
  // fp8 halves the MMA work per byte, so it stays on the skinny kernel up to 128 rows.
  if (d.block_scale != 0) {
    // Block-scaled decode shapes (MXFP8 / MXFP6 / MXFP4 / NVFP4 weights, bf16 C) stream on the
    // skinny kernel up to 128 rows.
    const bool mx_8_6 = d.ab_type == KL_E4M3 || d.ab_type == KL_E3M2 || d.ab_type == KL_E2M3;
    const bool bs_skinny = d.c_type == KL_BF16 && (d.ab_type == KL_E2M1 || (mx_8_6 && d.block_scale == 1));
    if (bs_skinny && d.m <= 128 && d.m_block_group == nullptr) return KL_ALGO_SKINNY;
    return d.m >= 256 ? KL_ALGO_2CTA : KL_ALGO_1CTA;
  }
  const bool bf16_skinny = d.ab_type == KL_BF16 && (d.c_type == KL_BF16 || d.c_type == KL_F32);
  const bool fp8_skinny = d.ab_type == KL_E4M3 && d.c_type == KL_BF16;
  if ((bf16_skinny && d.m <= 64) || (fp8_skinny && d.m <= 128)) return KL_ALGO_SKINNY;
  return d.m >= 256 ? KL_ALGO_2CTA : KL_ALGO_1CTA;
}

kl_status skinny_workspace_size(kl_gemm_desc const& d, size_t* bytes) {
  Plan pl;
  kl_status s = make_plan(d, &pl);
  if (s != KL_OK) return s;
  *bytes = pl.ticket_bytes + pl.slot_bytes;
  return KL_OK;
}

kl_status run_skinny(kl_gemm_desc const& d, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  Plan pl;
  kl_status s = make_plan(d, &pl);
  if (s != KL_OK) return s;
  const size_t need = pl.ticket_bytes + pl.slot_bytes;
  void* ws = workspace;
  if (ws == nullptr) {
    s = library_workspace(need, pl.ticket_bytes, stream, &ws);
    if (s != KL_OK) return s;
  } else if (workspace_bytes < need) {
    return fail(KL_ERR_INVALID_ARGUMENT,
                "kl_gemm_ws: workspace of " + std::to_string(workspace_bytes) + " bytes, need " + std::to_string(need));
  } else if (reinterpret_cast<uintptr_t>(ws) % 16 != 0) {
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_ws: workspace must be 16-byte aligned");
  }
  if (d.block_scale == 1) {
    if (d.ab_type == KL_E4M3 && d.c_type == KL_BF16) return dispatch_tok_mx<kl::e4m3, kl::bf16, 32>(d, pl, ws, stream);
    if (d.ab_type == KL_E2M1 && d.c_type == KL_BF16) return dispatch_tok_mx<kl::e2m1x2, kl::bf16, 32>(d, pl, ws, stream);
    if (d.ab_type == KL_E3M2 && d.c_type == KL_BF16) return dispatch_tok_mx<kl::e3m2, kl::bf16, 32>(d, pl, ws, stream);
    if (d.ab_type == KL_E2M3 && d.c_type == KL_BF16) return dispatch_tok_mx<kl::e2m3, kl::bf16, 32>(d, pl, ws, stream);
    return fail(KL_ERR_NOT_SUPPORTED,
                "KL_ALGO_SKINNY with MX scales supports (A/B, C) = (e4m3, bf16), (e3m2, bf16), (e2m3, bf16), (e2m1, bf16)");
  }
  if (d.block_scale == 2) {
    if (d.ab_type == KL_E2M1 && d.c_type == KL_BF16) return dispatch_tok_mx<kl::e2m1x2, kl::bf16, 16>(d, pl, ws, stream);
    return fail(KL_ERR_NOT_SUPPORTED, "KL_ALGO_SKINNY with NVFP4 scales supports (A/B, C) = (e2m1, bf16)");
  }
  if (d.ab_type == KL_BF16 && d.c_type == KL_BF16) return dispatch_tok<kl::bf16, kl::bf16>(d, pl, ws, stream);
  if (d.ab_type == KL_BF16 && d.c_type == KL_F32) return dispatch_tok<kl::bf16, float>(d, pl, ws, stream);
  if (d.ab_type == KL_E4M3 && d.c_type == KL_BF16) return dispatch_tok<kl::e4m3, kl::bf16>(d, pl, ws, stream);
  return fail(KL_ERR_NOT_SUPPORTED, "KL_ALGO_SKINNY supports (A/B, C) = (bf16, bf16), (bf16, f32), (e4m3, bf16)");
}

}  // namespace kl::capi
