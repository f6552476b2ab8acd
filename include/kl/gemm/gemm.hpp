#pragma once

// Host-side launchers for the kl GEMM kernels (C++ API; the C ABI in kl_gemm.h wraps these).
// No counterpart in the reference: kernel_lib stops at the descriptor encoders.

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <stdexcept>
#include <type_traits>

#include <kl/gemm/gemm_kernel.cuh>
#include <kl/kl.hpp>

namespace kl::gemm {

struct Problem {
  int64_t m = 0, n = 0, k = 0;
  const void* a = nullptr;
  int64_t lda = 0;
  const void* b = nullptr;
  int64_t ldb = 0;
  void* c = nullptr;
  int64_t ldc = 0;
  float alpha = 1.0f;
  const float* scale_a = nullptr;
  const float* scale_b = nullptr;
  int group_m = 0;   // 0 = default for the config
  int max_ctas = 0;  // 0 = every SM
  int prefetch = 0;  // L2 prefetch distance in K-blocks: 0 = default, < 0 = off
  // Programmatic dependent launch: true lets this launch start its prologue while the kernel before
  // it on the stream finishes (the kernel waits for that kernel's results before reading memory).
  bool overlap_launch = true;
  unsigned long long* clock_probe = nullptr;  // device [4 * grid]: per CTA clock64/globaltimer at start and end
  // Peer copies of C (same shape and pitch, in other GPUs' memory, already mapped into this
  // process): the epilogue TMA-stores every tile there too. Not with the direct-store epilogue.
  void* const* peer_c = nullptr;
  int n_peers = 0;
  // NVLink multicast address of C (the same element (0, 0) and pitch as `c`, in a buffer bound to a
  // multicast object on every GPU): the epilogue writes every tile there once with multimem stores
  // instead of TMA-storing it to `c` and the peers. One problem, C = result, no peer copies; base,
  // pitch and width of C multiples of 16 bytes.
  void* mc_c = nullptr;
  // Batched GEMM: `batch` independent problems, A/B/C matrix b at a/b/c + b * stride_*.
  int64_t batch = 1;
  int64_t stride_a = 0, stride_b = 0, stride_c = 0;  // elements
  // 0: C = result. 1: C += result: on an fp32 C by TMA reducing stores (the add happens in the TMA
  // unit, also on every peer copy of C); on a bf16 / f16 C the epilogue reads this GPU's C, adds in
  // fp32 and stores the sum (rounded once) to C and its peer copies. Not with the direct-store
  // epilogue.
  int c_reduce = 0;
  // Block scaling (configs with kMx: MXFP8 / MXFP4 with UE8M0 scales per 32 K-elements, NVFP4 with
  // UE4M3 scales per 16): scales of A and B in the 128 x 4 blocked layout, ceil(rows / 128) x
  // ceil(K / (4 * vec)) atoms of 512 bytes, row-block major.
  const void* sfa = nullptr;
  const void* sfb = nullptr;
  // m-grouped GEMM: `groups` B matrices [groups, N, K] (stride_b elements apart); A [M, K] and
  // C [M, N] are single matrices whose 128-row blocks each use the B named by m_block_group[block]
  // (device, ceil(M / 128) entries; -1 = padding, computed with B = 0). CTA-pair configs use the
  // group of each 256-row tile's first block, so there blocks 2i and 2i + 1 must agree.
  int groups = 0;
  const int* m_block_group = nullptr;
  // Split tail (see tn_schedule): 0 = where the last wave would leave workers idle, 1 = always
  // (tests), -1 = never. It needs a workspace (kTnStreamKWorkspaceBytes, its first
  // kTnStreamKTicketBytes zeroed before the first launch; launches keep them zero); without one the
  // launch is data-parallel.
  int stream_k = 0;
  void* sk_workspace = nullptr;
  size_t sk_workspace_bytes = 0;
};

// Split-tail workspace: tickets first (zero between launches), then one fp32 slot of one CTA's
// 128 x 256 accumulator per CTA of every tail piece (up to 4 pieces for each of 148 one-CTA workers
// or 74 pairs on a B200).
inline constexpr size_t kTnStreamKTicketBytes = 64 * 1024;
inline constexpr size_t kTnStreamKSlotCtas = 4 * 148;
inline constexpr size_t kTnStreamKWorkspaceBytes = kTnStreamKTicketBytes + kTnStreamKSlotCtas * 128 * 256 * 4;

// How a launch deals its tiles. The persistent workers take whole tiles t, t + W, ...; when that
// leaves the last wave short (R = tiles mod W of W workers busy, as N-sharding does: an 8192 x 2048
// shard of 256 x 256 tiles is 256 tiles on 74 CTA pairs, R = 34), the R tail tiles are each cut
// into s equal K-ranges (s = 2..4, at most one per K-block) and the R s pieces dealt round-robin in
// range-major order, before the whole tiles: the tail then takes ceil(R s / W) / s of a wave plus the
// traffic of its partial sums instead of one wave. s is the one that minimises that, used when it
// saves at least a tenth of a wave (R = 34, W = 74, K 8192: s = 2; R = 54: no split, the four
// ranges it would need cost more in partial sums than the quarter wave they save); stream_k = 1
// always splits (s >= 2) where there is a K to split.
struct TnSchedule {
  int tiles = 0;
  int workers = 0;
  int sk_tiles = 0, sk_split = 1;
  size_t ticket_bytes = 0, slot_bytes = 0;
};

template <class Cfg>
TnSchedule tn_schedule(Problem const& pr, int max_workers) {
  TnSchedule s;
  const long long tiles_m = (pr.m + Cfg::kTileM - 1) / Cfg::kTileM, tiles_n = (pr.n + Cfg::kTileN - 1) / Cfg::kTileN;
  const long long tiles = tiles_m * tiles_n * (pr.batch > 1 ? pr.batch : 1);
  if (tiles <= 0 || tiles > INT32_MAX) return s;
  s.tiles = int(tiles);
  int cap = max_workers;
  if (pr.max_ctas > 0) cap = std::min(cap, std::max(1, pr.max_ctas / Cfg::kCtaGroup));
  s.workers = std::min(s.tiles, cap);
  if (pr.stream_k < 0 || cap <= 0) return s;
  if constexpr (Cfg::kNSub > 1) return s;  // wide tiles: whole tiles only
  const int W = cap, T = s.tiles;
  int R = T % W;
  if (R == 0 && pr.stream_k > 0) R = W;  // forced: split the last full wave
  if (R == 0) return s;
  const long long pack = Cfg::kFp4 ? 2 : 1;
  const long long k_blocks = (pr.k / pack + Cfg::kBlockK - 1) / Cfg::kBlockK;
  // The tail's time in waves of whole tiles, for s K-ranges per tile: ceil(R s / W) / s of MMA
  // work, plus the fp32 partial sums (written once and read once, 2 x R s CtaGroup 128 BlockN x 4
  // bytes, at ~6 TB/s) over one tile's MMA time at the power-capped ~1.4 GHz. Measured on B200
  // (8192 x 8192 bf16 A, 256 x 256 tiles on 74 pairs, K 8192): R 34 x 2 ranges 139.6 us vs 155.5
  // whole (the model: 0.63 of a wave); R 54 x 4 ranges 88 us vs 83 whole (the model: 1.15).
  const double tensor_flop_per_clk = sizeof(typename Cfg::in_type) == 2 ? 8192.0 : Cfg::kFp4 ? 32768.0 : 16384.0;
  const double tile_s = 2.0 * Cfg::kTileM * Cfg::kTileN * double(k_blocks * Cfg::kBlockK * pack) /
                        (tensor_flop_per_clk * Cfg::kCtaGroup * 1.4e9);
  int best = 1;
  double best_cost = 1.0;
  for (int sp = 2; sp <= 4 && sp <= k_blocks; ++sp) {
    if (size_t(R) * sp * Cfg::kCtaGroup > kTnStreamKSlotCtas) break;
    const double fixup_s = 2.0 * R * sp * Cfg::kCtaGroup * 128.0 * Cfg::kTileN * 4.0 / 6.0e12;
    const double cost = double((R * sp + W - 1) / W) / sp + fixup_s / tile_s;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = sp;
    }
  }
  if (pr.stream_k > 0 && best == 1 && k_blocks >= 2 && size_t(R) * 2 * Cfg::kCtaGroup <= kTnStreamKSlotCtas) best = 2;
  if (best == 1 || (pr.stream_k == 0 && best_cost > 0.9)) return s;
  const size_t tickets = size_t(R) * Cfg::kCtaGroup * Cfg::kEpiWarps * sizeof(int);
  const size_t slots = size_t(R) * best * Cfg::kCtaGroup * 128 * Cfg::kTileN * sizeof(float);
  if (tickets > kTnStreamKTicketBytes || kTnStreamKTicketBytes + slots > kTnStreamKWorkspaceBytes) return s;
  s.workers = T > W ? W : std::min(W, R * best);
  s.sk_tiles = R;
  s.sk_split = best;
  s.ticket_bytes = tickets;
  s.slot_bytes = slots;
  return s;
}

// Library defaults for the knobs a Problem leaves at 0.
inline constexpr int kDefaultPrefetchTn = 0;

struct LaunchInfo {
  int grid = 0;
  int tiles = 0;
  int cluster = 1;
};

namespace detail {

// Per-device caches below are filled on first use from whichever host thread gets there; the
// values are the same whoever computes them, and atomics keep concurrent first calls race-free.
inline int sm_count(int device) {
  static std::atomic<int> cache[64];
  if (device < 0 || device >= 64) return 0;
  int n = cache[device].load(std::memory_order_acquire);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    cache[device].store(n, std::memory_order_release);
  }
  return n;
}

template <class Cfg>
inline cudaError_t prepare_kernel(int device, int* max_workers) {
  // Per device: opt in to the shared-memory size and ask how many CTA groups fit at once.
  static std::atomic<int> workers[64];
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  if (workers[device].load(std::memory_order_acquire) == 0) {
    auto kernel = gemm_tn_kernel<Cfg>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg::kSmemBytes));
    if (e != cudaSuccess) return e;
    int n = 0;
    if constexpr (Cfg::kCtaGroup == 1) {
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, Cfg::kThreads, Cfg::kSmemBytes);
      if (e != cudaSuccess) return e;
      n *= sm_count(device);
    } else {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
      if (e != cudaSuccess) return e;
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = Cfg::kCtaGroup;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(Cfg::kCtaGroup * sm_count(device), 1, 1);
      cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
      cfg.dynamicSmemBytes = Cfg::kSmemBytes;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
      if (e != cudaSuccess) return e;
    }
    if (n <= 0) return cudaErrorInvalidConfiguration;
    workers[device].store(n, std::memory_order_release);
  }
  *max_workers = workers[device].load(std::memory_order_acquire);
  return cudaSuccess;
}

}  // namespace detail

// Queue C = alpha * A . B^T with the persistent tcgen05 kernel `Cfg` on `stream`. Throws
// std::invalid_argument (bad layout, from the tensor-map builder) and returns CUDA errors.
template <class Cfg>
cudaError_t launch_tn(Problem const& pr, int* status, unsigned long long timeout_ns, cudaStream_t stream,
                      LaunchInfo* info = nullptr) {
  using InT = typename Cfg::in_type;
  using OutT = typename Cfg::out_type;
  if (pr.m <= 0 || pr.n <= 0 || pr.k <= 0) throw std::invalid_argument("kl::gemm: m, n and k must be positive");
  if (pr.m > INT32_MAX || pr.n > INT32_MAX || pr.k > INT32_MAX)
    throw std::invalid_argument("kl::gemm: extents must fit in 32 bits");

  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  int max_workers = 0;
  e = detail::prepare_kernel<Cfg>(device, &max_workers);
  if (e != cudaSuccess) return e;

  if (pr.batch < 1 || pr.batch > 65535) throw std::invalid_argument("kl::gemm: batch must be in [1, 65535]");
  TnParams p{};
  // A batched problem is a rank-3 tensor (batch, rows, cols) per operand; one problem is rank 2.
  auto matrix = [&](auto* ptr, int64_t rows, int64_t cols, int64_t ld, int64_t bstride) {
    GmemTensor<std::remove_pointer_t<decltype(ptr)>, 3> g;
    g.ptr = ptr;
    g.shape[0] = pr.batch;
    g.shape[1] = rows;
    g.shape[2] = cols;
    g.stride[0] = bstride;
    g.stride[1] = ld;
    g.stride[2] = 1;
    return g;
  };
  // A K-major operand is stored [rows, K]; an MN-major one [K, rows].
  // Packed fp4 operands: K, leading dimensions and batch strides arrive in elements and are moved as
  // bytes (element pairs).
  constexpr int64_t kPack = Cfg::kFp4 ? 2 : 1;
  if (pr.k % kPack != 0 || pr.lda % kPack != 0 || pr.ldb % kPack != 0 || pr.stride_a % kPack != 0 ||
      pr.stride_b % kPack != 0)
    throw std::invalid_argument("kl::gemm: packed fp4 needs even K, leading dimensions and batch strides");
  const int64_t ku = pr.k / kPack, lda = pr.lda / kPack, ldb = pr.ldb / kPack;
  const int64_t a_rows = Cfg::kAMn ? ku : pr.m, a_cols = Cfg::kAMn ? pr.m : ku;
  const int64_t b_rows = Cfg::kBMn ? ku : pr.n, b_cols = Cfg::kBMn ? pr.n : ku;
  const bool grouped = pr.m_block_group != nullptr;
  if (grouped) {
    if (Cfg::kAMn || Cfg::kBMn || pr.batch > 1)
      throw std::invalid_argument("kl::gemm: m-grouped GEMMs take K-major operands, batch 1");
    if (pr.groups < 1 || pr.groups > 65535) throw std::invalid_argument("kl::gemm: groups must be in [1, 65535]");
  }
  if (grouped) {
    p.map_a = make_tma_load<typename Cfg::ATile>(row_major_strided(static_cast<InT const*>(pr.a), a_rows, a_cols, lda)).map;
    GmemTensor<InT const, 3> gb;
    gb.ptr = static_cast<InT const*>(pr.b);
    gb.shape[0] = pr.groups;
    gb.shape[1] = b_rows;
    gb.shape[2] = b_cols;
    gb.stride[0] = pr.stride_b / kPack;
    gb.stride[1] = ldb;
    gb.stride[2] = 1;
    p.map_b = make_tma_load<typename Cfg::BTile>(gb).map;
    p.map_c = make_tma_store<typename Cfg::CBox>(row_major_strided(static_cast<OutT*>(pr.c), pr.m, pr.n, pr.ldc)).map;
  } else if (pr.batch > 1) {
    p.map_a = make_tma_load<typename Cfg::ATile>(
                  matrix(static_cast<InT const*>(pr.a), a_rows, a_cols, lda, pr.stride_a / kPack)).map;
    p.map_b = make_tma_load<typename Cfg::BTile>(
                  matrix(static_cast<InT const*>(pr.b), b_rows, b_cols, ldb, pr.stride_b / kPack)).map;
    p.map_c = make_tma_store<typename Cfg::CBox>(matrix(static_cast<OutT*>(pr.c), pr.m, pr.n, pr.ldc, pr.stride_c)).map;
  } else {
    p.map_a = make_tma_load<typename Cfg::ATile>(row_major_strided(static_cast<InT const*>(pr.a), a_rows, a_cols, lda)).map;
    p.map_b = make_tma_load<typename Cfg::BTile>(row_major_strided(static_cast<InT const*>(pr.b), b_rows, b_cols, ldb)).map;
    p.map_c = make_tma_store<typename Cfg::CBox>(row_major_strided(static_cast<OutT*>(pr.c), pr.m, pr.n, pr.ldc)).map;
  }
  if (pr.n_peers < 0 || pr.n_peers > kMaxPeers) throw std::invalid_argument("kl::gemm: at most 7 peer copies of C");
  if (pr.n_peers > 0 && Cfg::kDirectStore)
    throw std::invalid_argument("kl::gemm: peer stores need the TMA-store epilogue");
  if (pr.c_reduce != 0 && pr.c_reduce != 1) throw std::invalid_argument("kl::gemm: c_reduce must be 0 (store) or 1 (add)");
  if (pr.c_reduce && Cfg::kDirectStore)
    throw std::invalid_argument("kl::gemm: reducing stores need the TMA-store epilogue");
  for (int q = 0; q < pr.n_peers; ++q) {
    auto* pc = static_cast<OutT*>(pr.peer_c[q]);
    p.map_peer[q] = pr.batch > 1 ? make_tma_store<typename Cfg::CBox>(matrix(pc, pr.m, pr.n, pr.ldc, pr.stride_c)).map
                                 : make_tma_store<typename Cfg::CBox>(row_major_strided(pc, pr.m, pr.n, pr.ldc)).map;
  }
  p.n_peers = pr.n_peers;
  if (pr.mc_c != nullptr) {
    if (Cfg::kDirectStore || pr.c_reduce != 0 || pr.batch > 1 || pr.n_peers > 0)
      throw std::invalid_argument(
          "kl::gemm: multicast C takes the staged epilogue, one problem, C = result and no peer copies");
    if (reinterpret_cast<uintptr_t>(pr.mc_c) % 16 != 0 || (pr.ldc * int64_t(sizeof(OutT))) % 16 != 0 ||
        (pr.n * int64_t(sizeof(OutT))) % 16 != 0)
      throw std::invalid_argument("kl::gemm: multicast C needs its base, pitch and width in multiples of 16 bytes");
  }

  TnArgs& a = p.args;
  a.m = int(pr.m);
  a.n = int(pr.n);
  a.k = int(ku);
  a.tiles_m = int((pr.m + Cfg::kTileM - 1) / Cfg::kTileM);
  a.tiles_n = int((pr.n + Cfg::kTileN - 1) / Cfg::kTileN);
  a.k_blocks = int((ku + Cfg::kBlockK - 1) / Cfg::kBlockK);
  // Default raster group: 8 tile-rows for the CTA pair, 16 for one CTA; per-tensor fp8 pairs take 16
  // once there are 32 or more tile columns (measured on B200, fp8 16384 x N x 8192: N = 16384 1419 vs
  // 1444 us, N = 8192 715 vs 725; N = 4096 and 2048 equal or faster with 8).
  // 256 x 512 pair tiles take 16 too (8192^3 bf16 under ncu: DRAM 0.969 GB per launch vs 1.031 with
  // 8, 673 vs 678 us).
  int group_default = Cfg::kCtaGroup == 2 ? 8 : 16;
  if constexpr (Cfg::kCtaGroup == 2 && Cfg::kIsF8 && !Cfg::kMx)
    if (a.tiles_n >= 32) group_default = 16;
  if constexpr (Cfg::kNSub > 1) group_default = 16;
  a.group_m = pr.group_m > 0 ? pr.group_m : group_default;
  a.group_m = std::min(a.group_m, a.tiles_m);
  a.alpha = pr.alpha;
  a.scale_a = pr.scale_a;
  a.scale_b = pr.scale_b;
  a.status = status;
  a.timeout_ns = timeout_ns;
  a.prefetch = pr.prefetch > 0 ? pr.prefetch : pr.prefetch < 0 ? 0 : kDefaultPrefetchTn;
  a.c = pr.c;
  a.ldc = pr.ldc;
  a.clock_probe = pr.clock_probe;
  a.batch = int(pr.batch);
  a.batch_stride_c = pr.stride_c;
  a.c_reduce = pr.c_reduce;
  a.m_block_group = pr.m_block_group;
  a.mc_c = pr.mc_c;
  if constexpr (Cfg::kMx) {
    if (pr.sfa == nullptr || pr.sfb == nullptr) throw std::invalid_argument("kl::gemm: block scaling needs scales of A and B");
    if (pr.batch > 1) throw std::invalid_argument("kl::gemm: block-scaled GEMMs are not batched");
    // The blocked scale arrays as [row blocks][K blocks][128 words of 4 bytes]; a box is the
    // kSfAtomsK atoms of one stage (K blocks of 4 * kSfVec elements).
    const int64_t kb = (pr.k + 4 * Cfg::kSfVec - 1) / (4 * Cfg::kSfVec);  // K blocks of 4 scales
    auto sf_map = [&](CUtensorMap* map, void const* ptr, int64_t row_blocks) {
      const int64_t shape[3] = {row_blocks, kb, 128};
      const int64_t stride[3] = {kb * 128, 128, 1};
      kl::detail::encode_tma_map(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, CU_TENSOR_MAP_SWIZZLE_NONE, 128,
                                 uint32_t(Cfg::kSfAtomsK), ptr, 3, shape, stride, TmaOptions{});
    };
    // m-grouped: B's scales are the groups' blocked arrays back to back, ceil(N / 128) row blocks
    // each.
    const int64_t nb = (pr.n + 127) / 128;
    sf_map(&p.map_sfa, pr.sfa, (pr.m + 127) / 128);
    sf_map(&p.map_sfb, pr.sfb, grouped ? nb * pr.groups : nb);
    a.sfb_group_blocks = grouped ? int(nb) : 0;
  }

  const long long all_tiles = (long long)a.tiles_m * a.tiles_n * a.batch;
  if (all_tiles > INT32_MAX) throw std::invalid_argument("kl::gemm: too many tiles");
  const int tiles = int(all_tiles);
  if (pr.stream_k < -1 || pr.stream_k > 1) throw std::invalid_argument("kl::gemm: stream_k must be -1, 0 or 1");
  TnSchedule sch = tn_schedule<Cfg>(pr, max_workers);
  if (sch.sk_tiles > 0 && (pr.sk_workspace == nullptr || pr.sk_workspace_bytes < kTnStreamKWorkspaceBytes)) {
    Problem dp = pr;  // no workspace: every tile whole
    dp.stream_k = -1;
    sch = tn_schedule<Cfg>(dp, max_workers);
  }
  const int workers = sch.workers;
  a.sk_tiles = sch.sk_tiles;
  a.sk_split = sch.sk_split;
  a.sk_tickets = sch.sk_tiles > 0 ? static_cast<int*>(pr.sk_workspace) : nullptr;
  a.sk_slots = sch.sk_tiles > 0 ? reinterpret_cast<float*>(static_cast<char*>(pr.sk_workspace) + kTnStreamKTicketBytes)
                                : nullptr;
  if (sch.sk_tiles > 0) a.prefetch = 0;  // the L2 prefetch follows the data-parallel tile order only

  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  unsigned n_attr = 0;
  cfg.gridDim = dim3(unsigned(workers * Cfg::kCtaGroup), 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  if constexpr (Cfg::kCtaGroup > 1) {
    attr[n_attr].id = cudaLaunchAttributeClusterDimension;
    attr[n_attr].val.clusterDim.x = Cfg::kCtaGroup;
    attr[n_attr].val.clusterDim.y = 1;
    attr[n_attr].val.clusterDim.z = 1;
    ++n_attr;
  }
  if (pr.overlap_launch) {
    attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n_attr].val.programmaticStreamSerializationAllowed = 1;
    ++n_attr;
  }
  cfg.attrs = n_attr > 0 ? attr : nullptr;
  cfg.numAttrs = n_attr;
  if (info) {
    info->grid = workers * Cfg::kCtaGroup;
    info->tiles = tiles;
    info->cluster = Cfg::kCtaGroup;
  }
  return cudaLaunchKernelEx(&cfg, gemm_tn_kernel<Cfg>, p);
}

}  // namespace kl::gemm
