// C ABI of libkl_b200.so (declared in include/kl_gemm.h): GEMM dispatch, device status word,
// and the runtime forms of the kl descriptor encoders.

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>

#include <cstdint>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>

#include <kl/gemm/gemm.hpp>
#include <kl/kl.hpp>
#include <kl_gemm.h>

#include "kl_internal.cuh"
#include "kl_tile.cuh"

namespace {

thread_local std::string g_last_error;
unsigned long long g_timeout_ns = 2000000000ull;

}  // namespace

// Timeout bits of every kl kernel on this device land here.
__device__ int kl_device_status_word;

namespace kl::capi {

kl_status fail(kl_status s, std::string const& msg) {
  g_last_error = msg;
  return s;
}

kl_status cuda_fail(cudaError_t e, char const* where) {
  return fail(KL_ERR_CUDA, std::string(where) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

unsigned long long wait_timeout_ns() { return g_timeout_ns; }

kl_status device_status_ptr(int** out) {
  static std::atomic<int*> cache[64];  // per device; the same address whoever looks it up first
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(KL_ERR_NOT_SUPPORTED, "device index above 63");
  int* p = cache[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, kl_device_status_word);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    p = static_cast<int*>(addr);
    cache[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return KL_OK;
}

}  // namespace kl::capi

using kl::capi::cuda_fail;
using kl::capi::fail;

namespace {

using namespace kl::gemm;

// The instantiated kernels: (inputs, output, CTA group, tile N, stages).
using Bf16Bf16_1 = TnConfig<kl::bf16, kl::bf16, 1, 256, 4>;
using Bf16F32_1 = TnConfig<kl::bf16, float, 1, 256, 4>;
using E4m3Bf16_1 = TnConfig<kl::e4m3, kl::bf16, 1, 256, 4>;
using Bf16Bf16_2 = TnConfig<kl::bf16, kl::bf16, 2, 256, 6>;
using Bf16F32_2 = TnConfig<kl::bf16, float, 2, 256, 6>;
using E4m3Bf16_2 = TnConfig<kl::e4m3, kl::bf16, 2, 256, 6>;

template <class Cfg>
kl_status run(Problem const& pr, cudaStream_t stream, LaunchInfo* info = nullptr) {
  return kl::capi::run_cfg<Cfg>(pr, stream, info);
}

// MN-major operands (A and/or B stored transposed), bf16 -> bf16.
template <bool AMn, bool BMn>
using Bf16Mn_1 = TnConfig<kl::bf16, kl::bf16, 1, 256, 4, false, AMn, BMn>;
template <bool AMn, bool BMn>
using Bf16Mn_2 = TnConfig<kl::bf16, kl::bf16, 2, 256, 6, false, AMn, BMn>;

kl_status run_mn(Problem const& pr, bool pair, bool a_mn, bool b_mn, cudaStream_t stream, LaunchInfo* info) {
  if (a_mn && b_mn) return pair ? run<Bf16Mn_2<true, true>>(pr, stream, info) : run<Bf16Mn_1<true, true>>(pr, stream, info);
  if (a_mn) return pair ? run<Bf16Mn_2<true, false>>(pr, stream, info) : run<Bf16Mn_1<true, false>>(pr, stream, info);
  return pair ? run<Bf16Mn_2<false, true>>(pr, stream, info) : run<Bf16Mn_1<false, true>>(pr, stream, info);
}

// Whether a CTA-pair request runs on the 256 x 512 tiles: asked for (variant 4), or the library's
// choice for variant 0. Block-scaled, MN-major and 64 / 32-byte-swizzle requests never do.
bool takes_wide_tiles(kl_gemm_desc const& d, Problem const& pr) {
  if (d.block_scale != 0 || d.a_major == 1 || d.b_major == 1 || (d.swizzle != 0 && d.swizzle != 128)) return false;
  return d.variant == 4 || (d.variant == 0 && kl::capi::wide_tiles_pay(d.ab_type, d.c_type, pr));
}

// The tile kernel for a request: by operand majors, operand swizzle and (A/B, C) types. Throws
// std::invalid_argument from the tensor-map builders, like launch_tn.
kl_status run_tile(kl_gemm_desc const& d, Problem const& pr, bool pair, cudaStream_t stream, LaunchInfo* info,
                   char const* who) {
  const bool a_mn = d.a_major == 1, b_mn = d.b_major == 1;
  if (d.block_scale != 0) {
    if (d.block_scale != 1 && d.block_scale != 2)
      return fail(KL_ERR_INVALID_ARGUMENT, std::string(who) + ": block_scale must be 0, 1 (MX) or 2 (NVFP4)");
    if (a_mn || b_mn || (d.swizzle != 0 && d.swizzle != 128) || pr.batch > 1)
      return fail(KL_ERR_NOT_SUPPORTED, std::string(who) + ": block-scaled GEMMs take K-major operands, 128-byte swizzle, batch 1");
    bool handled = false;
    kl_status s = kl::capi::run_tile_mx(d.block_scale, d.ab_type, d.c_type, d.variant, pair, pr, stream, info, &handled);
    if (handled) return s;
    return fail(KL_ERR_NOT_SUPPORTED, std::string(who) + (d.block_scale == 2
                                                              ? ": NVFP4 takes e2m1 inputs with bf16 or f32 C"
                                                              : ": MX takes e4m3, e5m2, e3m2, e2m3 or e2m1 inputs with bf16 or f32 C"));
  }
  const int32_t sw = d.swizzle == 0 ? 128 : d.swizzle;
  if (sw != 128 && sw != 64 && sw != 32)
    return fail(KL_ERR_INVALID_ARGUMENT, std::string(who) + ": swizzle must be 0 (default), 128, 64 or 32 bytes");
  if (a_mn || b_mn) {
    if (d.ab_type != KL_BF16 || d.c_type != KL_BF16 || sw != 128)
      return fail(KL_ERR_NOT_SUPPORTED,
                  std::string(who) + ": MN-major operands are built for bf16 inputs, bf16 C and the 128-byte swizzle");
    return run_mn(pr, pair, a_mn, b_mn, stream, info);
  }
  bool handled = false;
  kl_status s = KL_OK;
  if (sw != 128) {
    s = kl::capi::run_tile_swizzle(sw, d.ab_type, d.c_type, pr, pair, stream, info, &handled);
    if (handled) return s;
    return fail(KL_ERR_NOT_SUPPORTED, std::string(who) + ": 64- and 32-byte operand swizzle take bf16 inputs and bf16 or f32 C");
  }
  if (pair && takes_wide_tiles(d, pr)) {
    // 256 x 512 tiles: asked for, or the library default where they measured faster
    s = kl::capi::run_tile_wide(d.ab_type, d.c_type, pr, stream, info, &handled);
    if (handled) return s;
    return fail(KL_ERR_NOT_SUPPORTED, std::string(who) + ": 256 x 512 tiles (variant 4) take (bf16, bf16) or (e4m3, bf16)");
  }
  if (d.ab_type == KL_BF16 && d.c_type == KL_BF16)
    return pair ? run<Bf16Bf16_2>(pr, stream, info) : run<Bf16Bf16_1>(pr, stream, info);
  if (d.ab_type == KL_BF16 && d.c_type == KL_F32)
    return pair ? run<Bf16F32_2>(pr, stream, info) : run<Bf16F32_1>(pr, stream, info);
  if (d.ab_type == KL_E4M3 && d.c_type == KL_BF16)
    return pair ? run<E4m3Bf16_2>(pr, stream, info) : run<E4m3Bf16_1>(pr, stream, info);
  s = kl::capi::run_tile_types(d.ab_type, d.c_type, pr, pair, stream, info, &handled);
  if (handled) return s;
  return fail(KL_ERR_NOT_SUPPORTED,
              std::string(who) + ": supported (A/B, C) types are (bf16, bf16), (bf16, f32), (f16, f16), (f16, f32), "
                                 "(e4m3, bf16), (e4m3, f32), (e5m2, bf16), (e5m2, f32)");
}

// Problem fields shared by every entry point.
Problem problem_of(kl_gemm_desc const& d) {
  Problem pr;
  pr.m = d.m;
  pr.n = d.n;
  pr.k = d.k;
  pr.a = d.a;
  pr.lda = d.lda;
  pr.b = d.b;
  pr.ldb = d.ldb;
  pr.c = d.c;
  pr.ldc = d.ldc;
  pr.alpha = d.alpha;
  pr.scale_a = d.scale_a;
  pr.scale_b = d.scale_b;
  pr.group_m = d.group_m;
  pr.max_ctas = d.max_ctas;
  pr.prefetch = d.prefetch;
  pr.batch = d.batch > 1 ? d.batch : 1;
  pr.stride_a = d.stride_a;
  pr.stride_b = d.stride_b;
  pr.stride_c = d.stride_c;
  pr.c_reduce = d.c_reduce;
  pr.sfa = d.sfa;
  pr.sfb = d.sfb;
  pr.groups = d.groups;
  pr.m_block_group = d.m_block_group;
  pr.stream_k = d.stream_k;
  pr.overlap_launch = d.launch_overlap >= 0;
  return pr;
}

// Probe buffer for kl_gemm_clock_probe: one per device, 4 words per CTA, allocated on first use.
unsigned long long* g_probe[64] = {};

int elem_bytes_of(int32_t t) {
  switch (t) {
    case KL_BF16:
    case KL_F16:
      return 2;
    case KL_E4M3:
    case KL_E5M2:
    case KL_E3M2:  // packed fp6: one byte per element in shared memory
    case KL_E2M3:
    case KL_I8:
    case KL_U8:
      return 1;
    case KL_F32:
    case KL_I32:
      return 4;
    default:
      return 0;
  }
}

kl_status check_tile(int32_t elem_bytes, int32_t rows, int32_t cols, int32_t span) {
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4) return fail(KL_ERR_INVALID_ARGUMENT, "elem_bytes must be 1, 2 or 4");
  if (span != 16 && span != 32 && span != 64 && span != 128)
    return fail(KL_ERR_INVALID_ARGUMENT, "swizzle_span must be 16, 32, 64 or 128");
  const int atom = span / elem_bytes;
  if (rows <= 0 || rows % 8 != 0) return fail(KL_ERR_INVALID_ARGUMENT, "rows must be a positive multiple of 8");
  if (cols <= 0 || cols % atom != 0) return fail(KL_ERR_INVALID_ARGUMENT, "cols must be a multiple of the swizzle atom width");
  return KL_OK;
}

// The kernel family kl_gemm runs for `d`: desc->algo, or KL_ALGO_AUTO resolved. m-grouped GEMMs
// run on the tile kernels (the one-CTA kernel takes any 128-row grouping; the CTA pair needs groups
// padded to 256 rows, since it reads the group of each tile's first block, so it runs only when
// asked for); batched, MN-major and non-default-swizzle problems on the tile kernels; the rest by
// the size rule of choose_algo.
kl_status resolve_algo(kl_gemm_desc const& d, int* out) {
  const int64_t batch = d.batch > 1 ? d.batch : 1;
  const bool a_mn = d.a_major == 1, b_mn = d.b_major == 1;
  const bool default_swizzle = d.swizzle == 0 || d.swizzle == 128;
  int algo = d.algo;
  if (d.m_block_group != nullptr) {
    if (algo != KL_ALGO_AUTO && algo != KL_ALGO_1CTA && algo != KL_ALGO_2CTA)
      return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm: m-grouped GEMMs run on the tile kernels (KL_ALGO_1CTA / 2CTA)");
    if (batch > 1 || a_mn || b_mn)
      return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm: m-grouped GEMMs take K-major operands, batch 1");
    if (algo == KL_ALGO_AUTO) algo = KL_ALGO_1CTA;
  }
  if (algo == KL_ALGO_AUTO && d.block_scale != 0)
    algo = kl::capi::choose_algo(d);
  else if (algo == KL_ALGO_AUTO)
    algo = (batch > 1 || a_mn || b_mn || !default_swizzle) ? (d.m >= 256 ? KL_ALGO_2CTA : KL_ALGO_1CTA)
                                                           : kl::capi::choose_algo(d);
  *out = algo;
  return KL_OK;
}

}  // namespace

extern "C" {

int32_t kl_version(void) { return 100; }

kl_status kl_gemm_resolve_algo(const kl_gemm_desc* d, int32_t* algo) {
  if (d == nullptr || algo == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null argument");
  if (d->m <= 0 || d->n <= 0 || d->k <= 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_resolve_algo: empty problem");
  int a = KL_ALGO_AUTO;
  kl_status s = resolve_algo(*d, &a);
  if (s == KL_OK) *algo = a;
  return s;
}

kl_status kl_gemm_resolve_tile(const kl_gemm_desc* d, int32_t* tile_m, int32_t* tile_n) {
  if (d == nullptr || tile_m == nullptr || tile_n == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null argument");
  if (d->m <= 0 || d->n <= 0 || d->k <= 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_resolve_tile: empty problem");
  int a = KL_ALGO_AUTO;
  kl_status s = resolve_algo(*d, &a);
  if (s != KL_OK) return s;
  const bool mx = d->block_scale != 0;
  if (a == KL_ALGO_SKINNY) {
    *tile_m = 0;  // stream-K over the weight rows: no fixed C tile
    *tile_n = 0;
  } else if (a == KL_ALGO_1CTA) {
    *tile_m = 128;
    *tile_n = (mx && d->variant == 2) ? 128 : 256;
  } else {
    *tile_m = 256;
    *tile_n = mx ? (d->variant == 2 ? 128 : d->variant == 3 ? 192 : 256) : 256;
    if (!mx) {
      int count = 0;
      if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        (void)cudaGetLastError();
        return fail(KL_ERR_CUDA, "kl_gemm_resolve_tile: no CUDA device (the CTA-pair choice reads its SM count)");
      }
      if (takes_wide_tiles(*d, problem_of(*d))) *tile_n = 512;
    }
  }
  return KL_OK;
}

kl_status kl_release_workspaces(void) {
  kl::capi::forget_noalloc_scratch();
  kl_status s = kl::capi::release_tile_workspaces();
  if (s != KL_OK) return s;
  return kl::capi::release_skinny_workspaces();
}

const char* kl_last_error(void) { return g_last_error.c_str(); }

void kl_set_wait_timeout_ns(uint64_t ns) { g_timeout_ns = ns; }

kl_status kl_gemm_workspace_size(const kl_gemm_desc* d, size_t* bytes) {
  if (d == nullptr || bytes == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null argument");
  *bytes = 0;
  if (d->algo == KL_ALGO_SKINNY) return kl::capi::skinny_workspace_size(*d, bytes);
  return KL_OK;
}

kl_status kl_gemm_ws(const kl_gemm_desc* d, void* workspace, size_t workspace_bytes, void* stream_ptr) {
  if (d == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null descriptor");
  g_last_error.clear();
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (d->m < 0 || d->n < 0 || d->k < 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: negative extent");
  if (d->c_reduce != 0 && d->c_reduce != 1) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: c_reduce must be 0 (store) or 1 (add)");
  if (d->m == 0 || d->n == 0) return KL_OK;
  if (d->c == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: null C");
  const int c_bytes = elem_bytes_of(d->c_type);
  const int64_t batch = d->batch > 1 ? d->batch : 1;
  if (d->k == 0) {
    // An empty sum: C = 0, or C unchanged when adding into it.
    if (d->ldc < d->n) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: ldc < n");
    if (d->c_reduce) return KL_OK;
    for (int64_t i = 0; i < batch; ++i) {
      cudaError_t e = cudaMemset2DAsync(static_cast<char*>(d->c) + size_t(i) * d->stride_c * c_bytes,
                                        size_t(d->ldc) * c_bytes, 0, size_t(d->n) * c_bytes, size_t(d->m), stream);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemset2DAsync");
    }
    return KL_OK;
  }
  if (d->a == nullptr || d->b == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: null A or B");

  const Problem pr = problem_of(*d);
  const bool a_mn = d->a_major == 1, b_mn = d->b_major == 1;
  if ((d->a_major != 0 && !a_mn) || (d->b_major != 0 && !b_mn))
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: a_major / b_major must be 0 (K) or 1 (MN)");
  const bool default_swizzle = d->swizzle == 0 || d->swizzle == 128;
  if (d->launch_overlap < -1 || d->launch_overlap > 1)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: launch_overlap must be -1, 0 or 1");
  if (d->stream_k < -1 || d->stream_k > 1) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: stream_k must be -1, 0 or 1");
  int algo = KL_ALGO_AUTO;
  kl_status rs = resolve_algo(*d, &algo);
  if (rs != KL_OK) return rs;
  if (algo == KL_ALGO_SKINNY && batch > 1) return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm: KL_ALGO_SKINNY is not batched");
  if (algo == KL_ALGO_SKINNY && (a_mn || b_mn))
    return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm: KL_ALGO_SKINNY takes K-major operands");
  if (algo == KL_ALGO_SKINNY && !default_swizzle)
    return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm: KL_ALGO_SKINNY uses the 128-byte swizzle");
  try {
    if (algo == KL_ALGO_SKINNY) return kl::capi::run_skinny(*d, workspace, workspace_bytes, stream);
    if (algo != KL_ALGO_1CTA && algo != KL_ALGO_2CTA) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm: unknown algo");
    return run_tile(*d, pr, algo == KL_ALGO_2CTA, stream, nullptr, "kl_gemm");
  } catch (std::invalid_argument const& ex) {
    return fail(KL_ERR_INVALID_ARGUMENT, ex.what());
  } catch (std::exception const& ex) {
    return fail(KL_ERR_CUDA, ex.what());
  }
}

kl_status kl_gemm(const kl_gemm_desc* d, void* stream) { return kl_gemm_ws(d, nullptr, 0, stream); }

kl_status kl_gemm_gather(const kl_gemm_desc* d, void* const* peer_c, int32_t n_peers, void* stream_ptr) {
  if (d == nullptr || (n_peers > 0 && peer_c == nullptr)) return fail(KL_ERR_INVALID_ARGUMENT, "null argument");
  if (n_peers < 0 || n_peers > kMaxPeers) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather: 0 to 7 peers");
  g_last_error.clear();
  if (d->m < 0 || d->n < 0 || d->k < 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather: negative extent");
  if (d->m == 0 || d->n == 0) return KL_OK;  // an empty shard: nothing to compute or send
  if (d->k == 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather: k must be positive");
  if (d->a == nullptr || d->b == nullptr || d->c == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather: null A, B or C");
  for (int q = 0; q < n_peers; ++q)
    if (peer_c[q] == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather: null peer C");
  int algo = d->algo;
  if (algo == KL_ALGO_AUTO || algo == KL_ALGO_SKINNY)  // m-grouped: the pair needs 256-row groups, so ask for it
    algo = (d->m >= 256 && d->m_block_group == nullptr) ? KL_ALGO_2CTA : KL_ALGO_1CTA;
  if (algo != KL_ALGO_1CTA && algo != KL_ALGO_2CTA) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather: unknown algo");
  if (d->c_reduce != 0 && d->c_reduce != 1)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather: c_reduce must be 0 (store) or 1 (add)");
  Problem pr = problem_of(*d);
  pr.peer_c = peer_c;
  pr.n_peers = n_peers;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  try {
    return run_tile(*d, pr, algo == KL_ALGO_2CTA, stream, nullptr, "kl_gemm_gather");
  } catch (std::invalid_argument const& ex) {
    return fail(KL_ERR_INVALID_ARGUMENT, ex.what());
  } catch (std::exception const& ex) {
    return fail(KL_ERR_CUDA, ex.what());
  }
}

kl_status kl_gemm_gather_multicast(const kl_gemm_desc* d, void* mc_c, void* stream_ptr) {
  if (d == nullptr || mc_c == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null argument");
  g_last_error.clear();
  if (d->m < 0 || d->n < 0 || d->k < 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather_multicast: negative extent");
  if (d->m == 0 || d->n == 0) return KL_OK;  // an empty shard: nothing to compute or send
  if (d->k == 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather_multicast: k must be positive");
  if (d->a == nullptr || d->b == nullptr || d->c == nullptr)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather_multicast: null A, B or C");
  if (d->c_reduce != 0) return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_gather_multicast: C = result only (c_reduce 0)");
  if (d->batch > 1) return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_gather_multicast: one problem per call");
  int algo = d->algo;
  if (algo == KL_ALGO_AUTO || algo == KL_ALGO_SKINNY)
    algo = (d->m >= 256 && d->m_block_group == nullptr) ? KL_ALGO_2CTA : KL_ALGO_1CTA;
  if (algo != KL_ALGO_1CTA && algo != KL_ALGO_2CTA)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_gather_multicast: unknown algo");
  Problem pr = problem_of(*d);
  pr.mc_c = mc_c;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  try {
    return run_tile(*d, pr, algo == KL_ALGO_2CTA, stream, nullptr, "kl_gemm_gather_multicast");
  } catch (std::invalid_argument const& ex) {
    return fail(KL_ERR_INVALID_ARGUMENT, ex.what());
  } catch (std::exception const& ex) {
    return fail(KL_ERR_CUDA, ex.what());
  }
}

kl_status kl_ipc_get_handle(const void* dev_ptr, void* handle, int64_t* offset) {
  if (dev_ptr == nullptr || handle == nullptr || offset == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null argument");
  // The handle names the whole allocation that contains dev_ptr (a caching allocator hands out
  // pieces of larger allocations), so the importer also needs dev_ptr's offset inside it.
  using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static AddressRangeFn range = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return AddressRangeFn{nullptr};
    return reinterpret_cast<AddressRangeFn>(p);
  }();
  if (range == nullptr) return fail(KL_ERR_NOT_SUPPORTED, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail(KL_ERR_INVALID_ARGUMENT, "kl_ipc_get_handle: not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
  std::memcpy(handle, &h, sizeof(h));
  *offset = int64_t(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return KL_OK;
}

kl_status kl_ipc_open_handle(const void* handle, void** dev_ptr) {
  if (dev_ptr == nullptr || handle == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return KL_OK;
}

kl_status kl_ipc_close(void* dev_ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? KL_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

kl_status kl_gemm_clock_probe(const kl_gemm_desc* d, uint64_t* out, int32_t out_words, int32_t* ctas, void* stream_ptr) {
  if (d == nullptr || out == nullptr || ctas == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null argument");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  int algo = d->algo == KL_ALGO_AUTO ? kl::capi::choose_algo(*d) : d->algo;
  if (algo != KL_ALGO_1CTA && algo != KL_ALGO_2CTA)
    return fail(KL_ERR_NOT_SUPPORTED, "kl_gemm_clock_probe: tile kernels only (1CTA / 2CTA)");
  if (d->m <= 0 || d->n <= 0 || d->k <= 0) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_clock_probe: empty problem");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(KL_ERR_NOT_SUPPORTED, "device index above 63");
  if (g_probe[dev] == nullptr) {
    e = cudaMalloc(&g_probe[dev], 4096 * 4 * sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(clock probe)");
  }
  Problem pr = problem_of(*d);
  pr.clock_probe = g_probe[dev];
  LaunchInfo info;
  kl_status s = KL_OK;
  try {
    s = run_tile(*d, pr, algo == KL_ALGO_2CTA, stream, &info, "kl_gemm_clock_probe");
  } catch (std::invalid_argument const& ex) {
    return fail(KL_ERR_INVALID_ARGUMENT, ex.what());
  } catch (std::exception const& ex) {
    return fail(KL_ERR_CUDA, ex.what());
  }
  if (s != KL_OK) return s;
  if (info.grid > 4096 || 4 * info.grid > out_words) return fail(KL_ERR_INVALID_ARGUMENT, "kl_gemm_clock_probe: output too small");
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  e = cudaMemcpy(out, g_probe[dev], size_t(4) * info.grid * sizeof(uint64_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(clock probe)");
  *ctas = info.grid;
  return KL_OK;
}

kl_status kl_read_status(int32_t* bits, int32_t clear) {
  int* status = nullptr;
  kl_status s = kl::capi::device_status_ptr(&status);
  if (s != KL_OK) return s;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpy(&v, status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status)");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpy(status, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status clear)");
  }
  if (bits) *bits = v;
  if (v != 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) kl::capi::mark_workspace_dirty(dev);
  }
  if (v != 0) return fail(KL_ERR_TIMEOUT, "a device-side wait timed out (status bits " + std::to_string(v) + ")");
  return KL_OK;
}

kl_status kl_probe_wait_timeout(uint64_t timeout_ns, void* stream) {
  int* status = nullptr;
  kl_status s = kl::capi::device_status_ptr(&status);
  if (s != KL_OK) return s;
  return kl::capi::launch_wait_probe(status, timeout_ns, static_cast<cudaStream_t>(stream));
}

kl_status kl_smem_tile_offset(int32_t elem_bytes, int32_t rows, int32_t cols, int32_t span, int32_t row, int32_t col,
                              int64_t* swizzled, int64_t* plain) {
  kl_status s = check_tile(elem_bytes, rows, cols, span);
  if (s != KL_OK) return s;
  if (row < 0 || row >= rows || col < 0 || col >= cols) return fail(KL_ERR_INVALID_ARGUMENT, "(row, col) outside the tile");
  int sw_bits = span == 128 ? 3 : span == 64 ? 2 : span == 32 ? 1 : 0;
  const int atom = span / elem_bytes;
  if (plain) *plain = kl::detail::tile_offset(rows, atom, row, col);
  if (swizzled) *swizzled = kl::detail::swizzled_tile_offset(elem_bytes, rows, atom, sw_bits, row, col);
  return KL_OK;
}

kl_status kl_tma_box_geometry(int32_t elem_bytes, int32_t rows, int32_t cols, int32_t span, kl_tma_box* out) {
  kl_status s = check_tile(elem_bytes, rows, cols, span);
  if (s != KL_OK) return s;
  if (out == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null output");
  const auto g = kl::tma_box_geometry(elem_bytes, rows, cols, span);
  if (rows % g.outer != 0) return fail(KL_ERR_INVALID_ARGUMENT, "tiles taller than 256 rows must be a multiple of 256 rows");
  *out = kl_tma_box{g.inner, g.outer, g.col_boxes, g.row_boxes, g.count, g.bytes};
  return KL_OK;
}

kl_status kl_tma_box_position(int32_t elem_bytes, int32_t rows, int32_t cols, int32_t span, int32_t box, int32_t* row,
                              int32_t* col, uint32_t* smem_offset) {
  kl_tma_box geo;
  kl_status s = kl_tma_box_geometry(elem_bytes, rows, cols, span, &geo);
  if (s != KL_OK) return s;
  if (box < 0 || box >= geo.count) return fail(KL_ERR_INVALID_ARGUMENT, "box index out of range");
  const auto g = kl::tma_box_geometry(elem_bytes, rows, cols, span);
  if (row) *row = g.row(box);
  if (col) *col = g.col(box);
  if (smem_offset) *smem_offset = g.smem_offset(box);
  return KL_OK;
}

kl_status kl_umma_smem_desc(int32_t elem_bytes, int32_t rows, int32_t cols, int32_t span, uint32_t tile_addr,
                            int32_t k_block, int32_t row, uint64_t* out) {
  kl_status s = check_tile(elem_bytes, rows, cols, span);
  if (s != KL_OK) return s;
  if (out == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null output");
  const int mma_k = 32 / elem_bytes;
  if (cols % mma_k != 0) return fail(KL_ERR_INVALID_ARGUMENT, "tile K extent must be a multiple of the MMA K");
  if (k_block < 0 || k_block >= cols / mma_k) return fail(KL_ERR_INVALID_ARGUMENT, "k_block out of range");
  if (row < 0 || row % 8 != 0 || row >= rows) return fail(KL_ERR_INVALID_ARGUMENT, "row must be a multiple of 8 inside the tile");
  *out = kl::detail::umma_desc_rt(tile_addr, elem_bytes, rows, span, k_block, row);
  return KL_OK;
}

kl_status kl_umma_smem_desc_mn(int32_t elem_bytes, int32_t k_rows, int32_t mn_cols, int32_t span, uint32_t tile_addr,
                               int32_t k_block, int32_t mn_col, int32_t mn_extent, uint64_t* out) {
  kl_status s = check_tile(elem_bytes, k_rows, mn_cols, span);
  if (s != KL_OK) return s;
  if (out == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null output");
  if (span < 32) return fail(KL_ERR_NOT_SUPPORTED, "MN-major descriptors cover the 32/64/128-byte swizzles");
  const int mma_k_rows = 32 / elem_bytes;
  if (k_rows % mma_k_rows != 0) return fail(KL_ERR_INVALID_ARGUMENT, "tile K extent must be a multiple of the MMA K");
  if (k_block < 0 || k_block >= k_rows / mma_k_rows) return fail(KL_ERR_INVALID_ARGUMENT, "k_block out of range");
  const int atom = span / elem_bytes;
  if (mn_col < 0 || mn_col % atom != 0 || mn_col >= mn_cols)
    return fail(KL_ERR_INVALID_ARGUMENT, "mn_col must be a multiple of the atom width inside the tile");
  if (mn_extent <= 0) mn_extent = mn_cols - mn_col;
  *out = kl::detail::umma_desc_mn_rt(tile_addr, elem_bytes, k_rows, span, k_block, mn_col, mn_extent);
  return KL_OK;
}

kl_status kl_mma_instr_desc_major(int32_t a_type, int32_t b_type, int32_t acc_type, int32_t m, int32_t n,
                                  int32_t a_major, int32_t b_major, uint32_t* out) {
  if ((a_major != 0 && a_major != 1) || (b_major != 0 && b_major != 1))
    return fail(KL_ERR_INVALID_ARGUMENT, "major must be 0 (K) or 1 (MN)");
  kl_status s = kl_mma_instr_desc(a_type, b_type, acc_type, m, n, out);
  if (s != KL_OK) return s;
  *out |= (uint32_t(a_major) << 15) | (uint32_t(b_major) << 16);
  return KL_OK;
}

kl_status kl_mma_instr_desc_block_scaled(int32_t a_type, int32_t b_type, int32_t scale_type, int32_t m, int32_t n,
                                         int32_t a_sf_id, int32_t b_sf_id, uint32_t* out) {
  if (out == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null output");
  // Operand formats: kind::mxf8f6f4 e4m3 = 0, e5m2 = 1, e2m3 = 3, e3m2 = 4; kind::mxf4 / mxf4nvf4
  // e2m1 = 1.
  auto fmt = [](int32_t t) {
    switch (t) {
      case KL_E4M3: return 0;
      case KL_E5M2:
      case KL_E2M1: return 1;
      case KL_E2M3: return 3;
      case KL_E3M2: return 4;
      default: return -1;
    }
  };
  const int fa = fmt(a_type), fb = fmt(b_type);
  if (fa < 0 || fb < 0)
    return fail(KL_ERR_INVALID_ARGUMENT, "block-scaled operands must be e4m3, e5m2, e3m2, e2m3 or e2m1");
  if ((a_type == KL_E2M1) != (b_type == KL_E2M1)) return fail(KL_ERR_INVALID_ARGUMENT, "e2m1 takes e2m1 A and B");
  if (scale_type != KL_UE8M0 && scale_type != KL_UE4M3)
    return fail(KL_ERR_INVALID_ARGUMENT, "scale_type must be KL_UE8M0 or KL_UE4M3");
  if (scale_type == KL_UE4M3 && a_type != KL_E2M1)
    return fail(KL_ERR_INVALID_ARGUMENT, "UE4M3 scales go with e2m1 operands (kind::mxf4nvf4)");
  if (m != 128 && m != 256) return fail(KL_ERR_INVALID_ARGUMENT, "block-scaled M must be 128 or 256");
  if (n < 16 || n > 256 || n % 16 != 0) return fail(KL_ERR_INVALID_ARGUMENT, "N must be a multiple of 16 in [16, 256]");
  if (a_sf_id < 0 || a_sf_id > 3 || b_sf_id < 0 || b_sf_id > 3)
    return fail(KL_ERR_INVALID_ARGUMENT, "scale-factor ids are 0 to 3");
  *out = kl::detail::instr_desc_block_scaled_rt(uint32_t(fa), uint32_t(fb), m, n, uint32_t(a_sf_id), uint32_t(b_sf_id));
  if (scale_type == KL_UE4M3) *out &= ~(1u << 23);  // scale format bit: 1 = UE8M0, 0 = UE4M3
  return KL_OK;
}

kl_status kl_mma_instr_desc(int32_t a_type, int32_t b_type, int32_t acc_type, int32_t m, int32_t n, uint32_t* out) {
  if (out == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null output");
  auto operand = [](int32_t t, int* kind) -> int {
    switch (t) {
      case KL_F16: *kind = 0; return 0;
      case KL_BF16: *kind = 0; return 1;
      case KL_F32: *kind = 1; return 2;  // tf32
      case KL_E4M3: *kind = 2; return 0;
      case KL_E5M2: *kind = 2; return 1;
      case KL_E2M3: *kind = 2; return 3;
      case KL_E3M2: *kind = 2; return 4;
      case KL_U8: *kind = 3; return 0;
      case KL_I8: *kind = 3; return 1;
      default: return -1;
    }
  };
  int ka = -1, kb = -1;
  const int fa = operand(a_type, &ka), fb = operand(b_type, &kb);
  if (fa < 0 || fb < 0) return fail(KL_ERR_INVALID_ARGUMENT, "no UMMA operand format for this type");
  if (ka != kb) return fail(KL_ERR_INVALID_ARGUMENT, "A and B must belong to the same MMA kind");
  int fc = acc_type == KL_F16 ? 0 : acc_type == KL_F32 ? 1 : acc_type == KL_I32 ? 2 : -1;
  if (fc < 0) return fail(KL_ERR_INVALID_ARGUMENT, "no UMMA accumulator format for this type");
  if (m != 64 && m != 128 && m != 256) return fail(KL_ERR_INVALID_ARGUMENT, "M must be 64, 128 or 256");
  const int step = m == 64 ? 8 : 16;
  if (n < step || n > 256 || n % step != 0) return fail(KL_ERR_INVALID_ARGUMENT, "N must be a multiple of 8 (M=64) or 16, at most 256");
  *out = kl::detail::instr_desc_rt(uint32_t(fa), uint32_t(fb), uint32_t(fc), m, n);
  return KL_OK;
}

kl_status kl_make_tma_desc(int32_t dtype, int32_t tile_rows, int32_t tile_cols, int32_t span, int32_t is_store,
                           const void* gmem, int32_t rank, const int64_t* shape, const int64_t* stride, void* map_out) {
  (void)is_store;  // loads and stores encode identically
  const int eb = elem_bytes_of(dtype);
  if (eb == 0) return fail(KL_ERR_INVALID_ARGUMENT, "unknown dtype");
  kl_status s = check_tile(eb, tile_rows, tile_cols, span);
  if (s != KL_OK) return s;
  if (map_out == nullptr || shape == nullptr || stride == nullptr) return fail(KL_ERR_INVALID_ARGUMENT, "null argument");
  const auto g = kl::tma_box_geometry(eb, tile_rows, tile_cols, span);
  if (tile_rows % g.outer != 0) return fail(KL_ERR_INVALID_ARGUMENT, "tiles taller than 256 rows must be a multiple of 256 rows");
  CUtensorMapDataType t;
  switch (dtype) {
    case KL_BF16: t = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case KL_F16: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case KL_F32: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    case KL_I32: t = CU_TENSOR_MAP_DATA_TYPE_INT32; break;
    default: t = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
  }
  CUtensorMapSwizzle sw = span == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                        : span == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                        : span == 32  ? CU_TENSOR_MAP_SWIZZLE_32B
                                      : CU_TENSOR_MAP_SWIZZLE_NONE;
  try {
    CUtensorMap map;
    if (dtype == KL_E3M2 || dtype == KL_E2M3)  // packed fp6 in global memory: a 16U6 map
      kl::detail::encode_tma_map_u6(&map, sw, uint32_t(g.inner), uint32_t(g.outer), gmem, rank, shape, stride,
                                    kl::TmaOptions{});
    else
      kl::detail::encode_tma_map(&map, t, eb, sw, uint32_t(g.inner), uint32_t(g.outer), gmem, rank, shape, stride,
                                 kl::TmaOptions{});
    std::memcpy(map_out, &map, sizeof(CUtensorMap));
  } catch (std::invalid_argument const& ex) {
    return fail(KL_ERR_INVALID_ARGUMENT, ex.what());
  }
  return KL_OK;
}

}  // extern "C"
