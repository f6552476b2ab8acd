#pragma once

// Memory-bound GEMM for few rows of A (decode-shaped: C[M,N] = A[M,K] . B[N,K]^T with M <= 256
// tokens and a large weight matrix B). No counterpart in the reference: kernel_lib ships the
// descriptor encoders this kernel is built from, but no kernel.
//
// The operands are swapped so that the weights fill the 128-row UMMA M dimension and the tokens
// are the UMMA N dimension (N = TokPad, a multiple of 16): D^T[n, tok] = B[n, :] . A[tok, :]^T.
// Every weight byte is read from HBM exactly once. To keep all SMs streaming the same number of
// bytes, the flattened space of (128-row weight tile, 64-wide K-block) units is cut into one
// contiguous range per CTA (stream-K): a CTA walks its range tile by tile, accumulating in TMEM.
// A tile whose K-blocks all fall in one CTA is written straight to C. A tile shared by several
// CTAs is reduced through a workspace: each contributor stores its fp32 partial in its own slot,
// and the contributor that finishes last (a per-tile atomic ticket) sums the slots in fixed order
// (deterministic), writes C and re-arms the ticket for the next call. Nothing waits on another
// CTA, so there is no inter-CTA spin.
//
// Roles as in gemm_kernel.cuh: warp 0 TMA producer (weights streamed with an L2 evict-first hint,
// the small activation tile with evict-last), warp 1 MMA issuer, warps 2..5 epilogue.
//
// Block-scaled inputs (SfVec 32: MXFP8 / MXFP4, 16: NVFP4) work as in the tile kernels: each unit
// brings the scale atoms of its 128 weight rows (the MMA's A) and of the tokens (the MMA's B) with
// the K-block, and the MMA thread copies them into TMEM ahead of the block-scaled MMAs.

#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdint>

#include <kl/arch/cluster.hpp>
#include <kl/arch/griddep.hpp>
#include <kl/arch/mbarrier.hpp>
#include <kl/arch/tcgen05.hpp>
#include <kl/arch/tma.hpp>
#include <kl/gemm/gemm_kernel.cuh>
#include <kl/kl.hpp>

namespace kl::gemm {

template <typename InT, typename OutT, int TokPad, int Stages, int WSub = 1, int SfVec = 0>
struct SkinnyConfig {
  using in_type = InT;
  using out_type = OutT;
  static constexpr int kThreads = 192;
  static constexpr int kSub = WSub;                        // 128-row weight boxes per tile
  static constexpr int kTileW = 128 * WSub;                // weight rows per tile
  static constexpr int kTok = TokPad;                      // UMMA N
  static constexpr int kBlockK = 128 / int(sizeof(InT));   // one 128-byte swizzle span
  static constexpr int kUmmaK = 32 / int(sizeof(InT));
  static constexpr int kStages = Stages;
  static constexpr int kNumAcc = 2;
  static constexpr int kAccCols = TokPad * WSub;           // one accumulator: WSub blocks of TokPad columns
  // Block scales: atoms along K per stage, token atoms (128 tokens each), MMAs per atom, bytes.
  static constexpr int kSfVecSize = SfVec;
  static constexpr bool kMx = SfVec != 0;
  static constexpr bool kNv = SfVec == 16;
  static constexpr bool kFp4 = std::is_same_v<InT, e2m1x2>;
  // Packed fp6 (e3m2 / e2m3): TMA's 16U6 type gives each element a shared-memory byte, so the tiles
  // are fp8's; transactions count the packed bytes (3/4 of the tiles).
  static constexpr bool kFp6 = is_fp6<InT>;
  static constexpr int kSfAtomsK = kMx ? (kFp4 ? 256 : 128) / (4 * SfVec) : 0;
  static constexpr int kXAtoms = kMx ? (TokPad + 127) / 128 : 0;
  static constexpr int kMmasPerSfAtom = kMx ? 4 / kSfAtomsK : 1;
  static constexpr uint32_t kSfIdStep = 4u / uint32_t(kMmasPerSfAtom);
  static constexpr uint32_t kSfwBytes = 512u * kSfAtomsK * WSub;
  static constexpr uint32_t kSfxBytes = 512u * kSfAtomsK * kXAtoms;
  static constexpr int kSfwCol = kAccCols * kNumAcc;       // TMEM columns of the weights' and tokens' scales
  static constexpr int kSfxCol = kSfwCol + 4 * kSfAtomsK * WSub;
  static constexpr int kTmemUsed = kAccCols * kNumAcc + 4 * kSfAtomsK * (WSub + kXAtoms);
  static constexpr int kTmemCols = (kTmemUsed <= 32) ? 32 : (kTmemUsed <= 64) ? 64 : (kTmemUsed <= 128) ? 128
                                 : (kTmemUsed <= 256) ? 256 : 512;
  using WTile = SmemTile<InT, 128, kBlockK>;               // one UMMA M = 128 box
  using XTile = SmemTile<InT, kTok, kBlockK>;
  static constexpr uint32_t kWBoxBytes = WTile::bytes;
  static constexpr uint32_t kWBytes = WTile::bytes * WSub;
  static constexpr uint32_t kXBytes = XTile::bytes;
  static constexpr uint32_t kStageTx = (kFp6 ? (kWBytes + kXBytes) / 4 * 3 : kWBytes + kXBytes) + kSfwBytes + kSfxBytes;
  static constexpr uint32_t kOffW = 0;
  static constexpr uint32_t kOffX = kStages * kWBytes;
  static constexpr uint32_t kOffSfw = kOffX + kStages * kXBytes;
  static constexpr uint32_t kOffSfx = kOffSfw + kStages * kSfwBytes;
  static constexpr uint32_t kOffBar = kOffSfx + kStages * kSfxBytes;
  static constexpr uint32_t kNumBars = 2 * kStages + 2 * kNumAcc + 1;
  static constexpr uint32_t kOffSlot = kOffBar + 8 * kNumBars;
  static constexpr uint32_t kSmemBytes = kOffSlot + 16 + 1024;
  static constexpr bool kIsF8 = sizeof(InT) == 1;
  static constexpr uint32_t idesc() {
    if constexpr (kNv)  // scale format bit 23: 0 = UE4M3
      return mma_instr_desc_block_scaled<InT, InT, 128, kTok>() & ~(1u << 23);
    else if constexpr (kMx)
      return mma_instr_desc_block_scaled<InT, InT, 128, kTok>();
    else
      return mma_instr_desc<InT, InT, float, 128, kTok>();
  }
  static constexpr uint32_t kIdesc = idesc();

  static_assert(WSub == 1 || WSub == 2, "one or two 128-row weight boxes per tile");
  static_assert(kTmemUsed <= 512, "two accumulators (and the scales) must fit in TMEM");
  static_assert(SfVec == 0 || SfVec == 32 || (SfVec == 16 && kFp4), "scales per 32 elements, or per 16 for fp4");
  static_assert(!kFp4 || kMx, "packed fp4 operands are block-scaled");
  static_assert(!kFp6 || SfVec == 32, "fp6 operands are MX block-scaled (kind::mxf8f6f4)");
  static_assert(TokPad == 16 || (TokPad % 32 == 0 && TokPad <= 256), "token tile: 16 or a multiple of 32 up to 256");
  static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
  static_assert(kWBytes % 1024 == 0 && kXBytes % 1024 == 0, "stages keep 1 KB alignment");
};

struct SkinnyArgs {
  int m, n, k;            // C[m, n], m = tokens
  int n_tiles, k_blocks;  // weight tiles (of kTileW rows) and K-blocks per tile
  long long total_units;  // n_tiles * k_blocks
  int grid;               // CTAs (each owns one contiguous unit range)
  float alpha;
  const float* scale_a;
  const float* scale_b;
  void* c;                // C, row-major [m, ldc]
  long long ldc;
  int* tickets;           // [n_tiles][4] arrival counters, zero between calls
  float* slots;           // [n_tiles + grid - 1][TokPad][tile rows] fp32 partials
  int* status;
  unsigned long long timeout_ns;
  int prefetch;           // L2 prefetch distance for weight tiles, in units (0 = off)
  int c_reduce;           // 0: C = result; 1: C += result
};

struct SkinnyParams {
  CUtensorMap map_w;  // B [N, K], box {kBlockK, 128} (kSub boxes per tile)
  CUtensorMap map_x;  // A [M, K], box {kBlockK, TokPad}
  CUtensorMap map_sfw;  // block scales of B and A (blocked arrays as [row blocks, K blocks, 128] words)
  CUtensorMap map_sfx;
  SkinnyArgs args;
};

// Library default L2 prefetch distance of the skinny kernel, in K-blocks (0 = off). Measured on
// B200 at the decode shapes: prefetching 8-64 K-blocks ahead only lowered throughput.
inline constexpr int kDefaultPrefetchSkinny = 0;

// CTAs the skinny kernel streams with by default: three quarters of the SMs, rounded up to a
// multiple of 8 (112 on a 148-SM B200). Measured on B200 (N = 28672, K = 8192): 112 CTAs read
// 6.34 TB/s at 16 tokens against 5.64 TB/s with all 148; 56-104 and 120-148 were all slower.
// More concurrent weight streams than that only add contention in the memory system.
KL_HOST_DEVICE constexpr int skinny_default_ctas(int sms) { return ((sms * 3 / 4) + 7) / 8 * 8; }

// The CTA whose unit range contains unit f, for ranges [floor(i*T/G), floor((i+1)*T/G)).
KL_HOST_DEVICE int cta_of_unit(long long f, long long total, int grid) {
  return int(((f + 1) * grid + total - 1) / total) - 1;
}
KL_HOST_DEVICE long long unit_range_start(int cta, long long total, int grid) { return (long long)cta * total / grid; }

#if defined(__CUDACC__)

KL_DEVICE void st_global_b16(void* p, uint16_t v) {
  asm volatile("st.global.b16 [%0], %1;" ::"l"(p), "h"(v) : "memory");
}

// C[j0 + q][col] = alpha * r[q] for the tokens q < W that exist (one C column per thread: a warp
// writes 32 consecutive columns of each token row). With args.c_reduce the result is added to C
// in fp32 and rounded once; exactly one thread writes each element, so the read-modify-write needs
// no atomics.
template <typename OutT, int W>
KL_DEVICE void store_c_column(SkinnyArgs const& args, const uint32_t (&r)[32], int j0, int col, float alpha) {
#pragma unroll
  for (int q = 0; q < W; ++q) {
    const int j = j0 + q;
    if (j < args.m) {
      const float v = __uint_as_float(r[q]) * alpha;
      if constexpr (sizeof(OutT) == 2) {
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(args.c) + (long long)j * args.ldc + col;
        __nv_bfloat16 h = __float2bfloat16_rn(args.c_reduce ? __bfloat162float(*dst) + v : v);
        st_global_b16(dst, *reinterpret_cast<uint16_t*>(&h));
      } else {
        float* dst = static_cast<float*>(args.c) + (long long)j * args.ldc + col;
        *dst = args.c_reduce ? *dst + v : v;
      }
    }
  }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1) gemm_skinny_kernel(const __grid_constant__ SkinnyParams p) {
#if defined(KL_ARCH_SM100)
  using OutT = typename Cfg::out_type;
  constexpr int S = Cfg::kStages;
  constexpr int TOK = Cfg::kTok;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t w_smem = base + Cfg::kOffW;
  const uint32_t x_smem = base + Cfg::kOffX;
  const uint32_t sfw_smem = base + Cfg::kOffSfw;
  const uint32_t sfx_smem = base + Cfg::kOffSfx;
  const uint32_t bar0 = base + Cfg::kOffBar;
  const uint32_t tmem_slot = base + Cfg::kOffSlot;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (S + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * S + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * S + Cfg::kNumAcc + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * S + 2 * Cfg::kNumAcc);

  const SkinnyArgs& args = p.args;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const long long u_begin = unit_range_start(cta, args.total_units, args.grid);
  const long long u_end = unit_range_start(cta + 1, args.total_units, args.grid);
  const int KB = args.k_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbarrier_init(full_bar(s), 1);
      mbarrier_init(empty_bar(s), 1);
    }
    for (int a = 0; a < Cfg::kNumAcc; ++a) {
      mbarrier_init(tfull_bar(a), 1);
      mbarrier_init(tempty_bar(a), 4);
    }
    mbarrier_init(drain_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&p.map_w);
    tma_prefetch_map(&p.map_x);
  }
  if (warp == 1) {
    tmem_alloc<1>(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish<1>();
  }
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem_base = ld_shared_u32(tmem_slot);
  // Programmatic serialization: no global memory above this line (see the tile kernel).
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (elect_one()) {
      const uint64_t stream_policy = l2_policy_evict_first();
      const uint64_t keep_policy = l2_policy_evict_last();
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      const int pf = args.prefetch;
      auto prefetch_unit = [&](long long v) {
        if (v >= u_end) return;
        const int pt = int(v / KB);
        for (int sub = 0; sub < Cfg::kSub; ++sub)
          tma_prefetch_l2_2d(&p.map_w, int(v - (long long)pt * KB) * Cfg::kBlockK, pt * Cfg::kTileW + sub * 128);
      };
      for (int j = 0; j < pf; ++j) prefetch_unit(u_begin + j);
      for (long long u = u_begin; u < u_end; ++u) {
        const int tile = int(u / KB);
        const int kb = int(u - (long long)tile * KB);
        if (pf > 0) prefetch_unit(u + pf);
        if (!mbarrier_wait(empty_bar(stage), phase ^ 1u, args.timeout_ns)) {
          record_status(args.status, kStatusProducerTimeout);
          ok = false;
          break;
        }
        mbarrier_arrive_expect_tx(full_bar(stage), Cfg::kStageTx);
        const int kx = kb * Cfg::kBlockK;
#pragma unroll
        for (int sub = 0; sub < Cfg::kSub; ++sub)
          tma_load_2d_hint(w_smem + stage * Cfg::kWBytes + sub * Cfg::kWBoxBytes, &p.map_w, full_bar(stage), kx,
                           tile * Cfg::kTileW + sub * 128, stream_policy);
        tma_load_2d_hint(x_smem + stage * Cfg::kXBytes, &p.map_x, full_bar(stage), kx, 0, keep_policy);
        if constexpr (Cfg::kMx) {
          const int sy = kb * Cfg::kSfAtomsK;
#pragma unroll
          for (int sub = 0; sub < Cfg::kSub; ++sub)
            tma_load_3d(sfw_smem + stage * Cfg::kSfwBytes + 512u * Cfg::kSfAtomsK * sub, &p.map_sfw, full_bar(stage), 0,
                        sy, tile * Cfg::kSub + sub);
#pragma unroll
          for (int j = 0; j < Cfg::kXAtoms; ++j)
            tma_load_3d(sfx_smem + stage * Cfg::kSfxBytes + 512u * Cfg::kSfAtomsK * j, &p.map_sfx, full_bar(stage), 0,
                        sy, j);
        }
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok)
        for (int s = 0; s < S; ++s) (void)mbarrier_wait(empty_bar(s), phase ^ 1u, 1000000ull);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      const uint64_t w_desc0 = umma_desc_at<typename Cfg::WTile>(w_smem).desc_;
      const uint64_t x_desc0 = umma_desc_at<typename Cfg::XTile>(x_smem).desc_;
      uint32_t stage = 0, phase = 0, iter = 0;
      bool ok = true;
      long long u = u_begin;
      while (ok && u < u_end) {
        const int tile = int(u / KB);
        const long long seg_end = ((long long)tile + 1) * KB < u_end ? ((long long)tile + 1) * KB : u_end;
        const uint32_t acc = iter & 1u;
        const uint32_t acc_phase = (iter >> 1) & 1u;
        if (!mbarrier_wait(tempty_bar(acc), acc_phase ^ 1u, args.timeout_ns)) {
          record_status(args.status, kStatusMmaTimeout);
          break;
        }
        tcgen05_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kAccCols;
        for (long long v = u; v < seg_end; ++v) {
          if (!mbarrier_wait(full_bar(stage), phase, args.timeout_ns)) {
            record_status(args.status, kStatusMmaTimeout);
            ok = false;
            break;
          }
          tcgen05_fence_after();
          const uint64_t w_desc = w_desc0 + ((stage * Cfg::kWBytes) >> 4);
          const uint64_t x_desc = x_desc0 + ((stage * Cfg::kXBytes) >> 4);
          if constexpr (Cfg::kMx) {
            // Scales to TMEM: weights' atom (sub, q) at kSfwCol + 4 (q * kSub + sub), tokens' (j, q)
            // at kSfxCol + 4 (q * kXAtoms + j).
#pragma unroll
            for (int q = 0; q < Cfg::kSfAtomsK; ++q) {
#pragma unroll
              for (int sub = 0; sub < Cfg::kSub; ++sub)
                tmem_cp_32x128b_warpx4<1>(tmem_base + Cfg::kSfwCol + 4 * (q * Cfg::kSub + sub),
                                          encode_smem_desc(sfw_smem + stage * Cfg::kSfwBytes +
                                                               512u * (sub * Cfg::kSfAtomsK + q),
                                                           0, 128, UmmaLayout::SWIZZLE_NONE));
#pragma unroll
              for (int j = 0; j < Cfg::kXAtoms; ++j)
                tmem_cp_32x128b_warpx4<1>(tmem_base + Cfg::kSfxCol + 4 * (q * Cfg::kXAtoms + j),
                                          encode_smem_desc(sfx_smem + stage * Cfg::kSfxBytes +
                                                               512u * (j * Cfg::kSfAtomsK + q),
                                                           0, 128, UmmaLayout::SWIZZLE_NONE));
            }
          }
#pragma unroll
          for (int k = 0; k < Cfg::kBlockK / Cfg::kUmmaK; ++k) {
            const uint64_t koff = block_offset_16B<typename Cfg::WTile>(k);
            const uint32_t accumulate = (v != u || k != 0) ? 1u : 0u;
#pragma unroll
            for (int sub = 0; sub < Cfg::kSub; ++sub) {
              const uint64_t wd = w_desc + ((sub * Cfg::kWBoxBytes) >> 4) + koff;
              if constexpr (Cfg::kMx) {
                const int q = k / Cfg::kMmasPerSfAtom;
                const uint32_t id = uint32_t(k % Cfg::kMmasPerSfAtom) * Cfg::kSfIdStep;
                const uint32_t idesc = Cfg::kIdesc | (id << 29) | (id << 4);
                const uint32_t sfw_t = tmem_base + Cfg::kSfwCol + 4 * (q * Cfg::kSub + sub);
                const uint32_t sfx_t = tmem_base + Cfg::kSfxCol + 4 * Cfg::kXAtoms * q;
                if constexpr (Cfg::kNv)
                  umma_nvf4_ss<1>(d_tmem + sub * TOK, wd, x_desc + koff, idesc, sfw_t, sfx_t, accumulate);
                else if constexpr (Cfg::kFp4)
                  umma_mxf4_ss<1>(d_tmem + sub * TOK, wd, x_desc + koff, idesc, sfw_t, sfx_t, accumulate);
                else
                  umma_mxf8_ss<1>(d_tmem + sub * TOK, wd, x_desc + koff, idesc, sfw_t, sfx_t, accumulate);
              } else if constexpr (Cfg::kIsF8)
                umma_f8_ss<1>(d_tmem + sub * TOK, wd, x_desc + koff, Cfg::kIdesc, accumulate);
              else
                umma_f16_ss<1>(d_tmem + sub * TOK, wd, x_desc + koff, Cfg::kIdesc, accumulate);
            }
          }
          umma_commit<1>(empty_bar(stage));
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit<1>(tfull_bar(acc));
        u = seg_end;
        ++iter;
      }
      umma_commit<1>(drain_bar);
      if (!mbarrier_wait(drain_bar, 0, args.timeout_ns)) record_status(args.status, kStatusDrainTimeout);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int quarter = warp & 3;
    const uint32_t lane_base = uint32_t(quarter * 32) << 16;
    float alpha = args.alpha;
    if (args.scale_a != nullptr) alpha *= *args.scale_a;
    if (args.scale_b != nullptr) alpha *= *args.scale_b;
    const int lrow = quarter * 32 + lane;  // row inside a 128-row weight box
    uint32_t iter = 0;
    long long u = u_begin;
    while (u < u_end) {
      const int tile = int(u / KB);
      const long long tile_begin = (long long)tile * KB;
      const long long seg_end = tile_begin + KB < u_end ? tile_begin + KB : u_end;
      const uint32_t acc = iter & 1u;
      const uint32_t acc_phase = (iter >> 1) & 1u;
      if (!mbarrier_wait(tfull_bar(acc), acc_phase, args.timeout_ns)) {
        if (lane == 0) record_status(args.status, kStatusEpilogueTimeout);
        break;
      }
      tcgen05_fence_after();
      const int first = cta_of_unit(tile_begin, args.total_units, args.grid);
      const int last = cta_of_unit(tile_begin + KB - 1, args.total_units, args.grid);
      const int contributors = last - first + 1;
      const int me = cta - first;
      const long long slot0 = (long long)tile + first;  // slots of this tile: slot0 .. slot0 + contributors - 1
      float* mine = args.slots + (slot0 + me) * (long long)(TOK * Cfg::kTileW);
      // Drain the accumulator 32 tokens at a time: straight to C when this CTA owns the whole
      // tile, else into this contributor's slot (layout [token][tile rows]: 128-byte warp stores).
#pragma unroll 1
      for (int sub = 0; sub < Cfg::kSub; ++sub) {
        const int row = sub * 128 + lrow;          // weight row inside the tile
        const int col = tile * Cfg::kTileW + row;  // = the C column this thread owns
        const bool col_ok = col < args.n;
#pragma unroll 1
        for (int j0 = 0; j0 < TOK; j0 += 32) {
          uint32_t r[32];
          const uint32_t taddr = tmem_base + lane_base + acc * Cfg::kAccCols + uint32_t(sub * TOK + j0);
          if constexpr (TOK % 32 == 0) {
            tmem_ld_32x32b_x32(taddr, r);
          } else {
            tmem_ld_32x32b_x16(taddr, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
          }
          tmem_wait_ld();
          constexpr int kW = (TOK % 32 == 0) ? 32 : 16;
          if (contributors == 1) {
            if (col_ok) store_c_column<OutT, kW>(args, r, j0, col, alpha);
          } else {
#pragma unroll
            for (int q = 0; q < kW; ++q) mine[(j0 + q) * Cfg::kTileW + row] = __uint_as_float(r[q]);
          }
        }
      }
      tcgen05_fence_before();
      __syncwarp();
      if (lane == 0) mbarrier_arrive(tempty_bar(acc));

      if (contributors > 1) {
        __threadfence();
        __syncwarp();
        int ticket = 0;
        if (lane == 0) ticket = atomicAdd(&args.tickets[tile * 4 + quarter], 1);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket == contributors - 1) {
          // Last to arrive: every partial is visible (writers fence before their ticket). Sum the
          // slots in contributor order, so the result does not depend on who finished last.
          __threadfence();
#pragma unroll 1
          for (int sub = 0; sub < Cfg::kSub; ++sub) {
            const int row = sub * 128 + lrow;
            const int col = tile * Cfg::kTileW + row;
#pragma unroll 1
            for (int j0 = 0; j0 < TOK; j0 += 32) {
              float sum[32];
#pragma unroll
              for (int q = 0; q < 32; ++q) sum[q] = 0.0f;
              for (int s2 = 0; s2 < contributors; ++s2) {
                const float* part = args.slots + (slot0 + s2) * (long long)(TOK * Cfg::kTileW);
#pragma unroll
                for (int q = 0; q < 32; ++q)
                  if (j0 + q < TOK) sum[q] += __ldcg(part + (j0 + q) * Cfg::kTileW + row);
              }
              uint32_t r[32];
#pragma unroll
              for (int q = 0; q < 32; ++q) r[q] = __float_as_uint(sum[q]);
              if (col < args.n) store_c_column<OutT, 32>(args, r, j0, col, alpha);
            }
          }
          if (lane == 0) args.tickets[tile * 4 + quarter] = 0;  // re-arm for the next call
        }
      }
      u = seg_end;
      ++iter;
    }
  }

  __syncwarp();
  tcgen05_fence_before();
  __syncthreads();
  if (warp == 1) {
    tcgen05_fence_after();
    tmem_dealloc<1>(tmem_base, Cfg::kTmemCols);
  }
#endif  // KL_ARCH_SM100
}

#endif  // __CUDACC__

}  // namespace kl::gemm
