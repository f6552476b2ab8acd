#pragma once

// Persistent, warp-specialised dense GEMM for sm_100a:  C[M,N] (+)= alpha * A[M,K] . B[N,K]^T
// (K-major operands by default, MN-major ones as options; C row-major), in bf16 / f16 / fp8 /
// fp6 / fp4, optionally block-scaled (MX, NVFP4), batched or m-grouped. No counterpart in the reference:
// kernel_lib ships the descriptor encoders (tma_desc.hpp, umma_desc.hpp) this kernel is built
// from, but no kernel.
//
// Roles (192 threads, or 320 with eight epilogue warps; one CTA per SM):
//   warp 0      TMA producer: fills a Stages-deep ring of (A, B[, scales]) K-blocks in shared memory.
//   warp 1      MMA issuer: one thread issues tcgen05.mma into a TMEM accumulator and commits
//               each consumed stage back to the producer; warp 1 also owns the TMEM allocation.
//   warps 2..   epilogue: tcgen05.ld -> scale -> convert -> swizzled shared staging -> TMA store.
// Two TMEM accumulators (2 x BlockN fp32 columns) let the epilogue of tile i overlap the main
// loop of tile i + 1 (block-scaled 256-column tiles keep one; see kNumAcc). Tiles are walked
// persistently in groups of `group_m` tile-rows so that the CTAs running at the same time share A
// and B tiles in L2; when that leaves the last wave short, its tiles are cut into K-ranges and
// summed through fp32 slots (the split tail, see TnArgs::sk_tiles and WorkSeq).
//
// CtaGroup = 2 runs a CTA pair (cluster of 2) on a 256-row tile with cta_group::2 MMAs: each CTA
// loads its own 128 rows of A and its own half of B (no multicast), the even CTA issues the MMAs,
// and every byte, stage release and accumulator hand-off is signalled through mbarriers in both
// CTAs.
//
// Every wait is bounded (args.timeout_ns). On a timeout the role records a bit in *args.status,
// stops, and the CTA still drains its MMAs and frees TMEM before it exits.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

#include <kl/arch/cluster.hpp>
#include <kl/arch/griddep.hpp>
#include <kl/arch/mbarrier.hpp>
#include <kl/arch/multimem.hpp>
#include <kl/arch/tcgen05.hpp>
#include <kl/arch/tma.hpp>
#include <kl/kl.hpp>

namespace kl::gemm {

// Status bits a kernel ORs into *status when a bounded wait runs out.
enum : int {
  kStatusProducerTimeout = 1,
  kStatusMmaTimeout = 2,
  kStatusEpilogueTimeout = 4,
  kStatusDrainTimeout = 8,
};

template <typename InT, typename OutT, int CtaGroup, int BlockN, int Stages, bool DirectStore = false,
          bool AMn = false, bool BMn = false, class Sw = Swizzle128B, int SfVec = 0, int NSub = 1>
struct TnConfig {
  using in_type = InT;
  using out_type = OutT;
  static constexpr int kCtaGroup = CtaGroup;
  // true: the epilogue writes C straight from registers (16-byte vector stores per row) and the
  // shared memory that would stage TMA stores goes to the operand ring instead.
  static constexpr bool kDirectStore = DirectStore;
  static constexpr int kCtaM = 128;                    // rows of A (= TMEM lanes) per CTA
  static constexpr int kTileM = kCtaM * CtaGroup;      // rows of C per tile
  // Wide tiles (NSub > 1): NSub MMAs of N = BlockN side by side share every stage of A, so a tile is
  // BlockN * NSub columns of C and each byte of A brought from L2 feeds NSub times the MACs (a 256 x
  // 512 CTA-pair tile moves 3/4 of the operand bytes per MAC of a 256 x 256 one). Its accumulator
  // takes all of TMEM: one buffer, drained by eight epilogue warps before the next tile starts.
  static constexpr int kNSub = NSub;
  static constexpr int kBlockN = BlockN;               // N of one MMA
  static constexpr int kTileN = BlockN * NSub;         // columns of C per tile
  static constexpr int kCtaN = BlockN / CtaGroup;      // rows of B each CTA loads per sub-tile
  static constexpr int kBlockK = 128 / int(sizeof(InT));  // 128 bytes of K per stage
  static constexpr int kUmmaK = 32 / int(sizeof(InT));    // K of one tcgen05.mma
  static constexpr int kStages = Stages;
  // Block scaling (SfVec = K-elements per scale: 0 = none, 32 = MX with UE8M0 scales, 16 = NVFP4
  // with UE4M3 scales): one scale per SfVec K-elements of every row of A and B, given in the
  // 128 x 4 blocked layout (512-byte atoms: 128 rows x 4 scales, byte (r % 32) * 16 + (r / 32) * 4
  // + j for row r and K-group j). Each stage brings, by TMA, the atoms of this CTA's 128 rows of A
  // and of all the tile's rows of B (in both CTAs of a pair); the MMA thread moves them into TMEM
  // (tcgen05.cp 32x128b.warpx4) ahead of the stage's block-scaled MMAs. A stage holds 128 bytes of
  // K: 128 elements for fp8 (one atom along K, one scale byte per MMA), 256 for packed fp4 (two
  // atoms and two scale bytes per MMA with SfVec 32, four atoms and a whole scale word per MMA
  // with SfVec 16).
  static constexpr int kSfVec = SfVec;
  static constexpr bool kMx = SfVec != 0;
  static constexpr bool kNv = SfVec == 16;
  static constexpr bool kFp4 = std::is_same_v<InT, e2m1x2>;
  // Packed fp6 (e3m2 / e2m3): one element per shared-memory byte like fp8 (TMA's 16U6 type unpacks
  // 12 bytes into each 16-byte slot), consumed by kind::mxf8f6f4 like MXFP8; a stage's TMA
  // transactions count the packed bytes, 3/4 of the tile's shared-memory footprint.
  static constexpr bool kFp6 = is_fp6<InT>;
  // A tile of B rows [tn * BlockN, +BlockN) starts r = (tn * BlockN) % 128 rows into a 128-row
  // scale block, r a multiple of gcd(BlockN, 128) >= 32: the tile's scales span kSfbAtoms blocks,
  // copied to TMEM side by side, and the MMAs read them from word r / 32 on (row r + j of the first
  // block sits in lane j % 32, word (r + j) / 32). So BlockN = 192 works with 128-row scale blocks.
  static constexpr int kSfbGcd = (BlockN % 128 == 0) ? 128 : (BlockN % 64 == 0) ? 64 : 32;
  static constexpr int kSfbAtoms = kMx ? (128 - kSfbGcd + BlockN + 127) / 128 : 0;  // 128-row scale blocks of B per tile
  static constexpr int kSfAtomsK = kMx ? (kFp4 ? 256 : 128) / (4 * SfVec) : 0;  // atoms along K per stage
  static constexpr int kMmasPerSfAtom = kMx ? 4 / kSfAtomsK : 1;  // MMAs (32 bytes of K each) per atom
  static constexpr uint32_t kSfIdStep = 4u / uint32_t(kMmasPerSfAtom);  // scale bytes per MMA
  static constexpr uint32_t kSfaBytes = 512u * kSfAtomsK;
  static constexpr uint32_t kSfbBytes = 512u * kSfAtomsK * kSfbAtoms;
  // Two TMEM accumulators (epilogue of tile i overlaps the MMAs of tile i + 1), except for block
  // scaling with 256 columns (2 x 256 accumulator columns would leave none for the scales) and for
  // wide tiles, whose one accumulator of 2 x 256 columns fills TMEM.
  static constexpr int kNumAcc = ((kMx && BlockN == 256) || NSub > 1) ? 1 : 2;
  static constexpr int kAccCols = kTileN;              // fp32 accumulator columns per buffer
  static constexpr int kSfaCol = kAccCols * kNumAcc;   // TMEM columns of A's and B's scales
  static constexpr int kSfbCol = kSfaCol + 4 * kSfAtomsK;
  static constexpr int kTmemUsed = kAccCols * kNumAcc + 4 * kSfAtomsK * (1 + kSfbAtoms);
  static constexpr int kTmemCols = (kTmemUsed <= 32) ? 32 : (kTmemUsed <= 64) ? 64
                                 : (kTmemUsed <= 128) ? 128 : (kTmemUsed <= 256) ? 256 : 512;
  // Epilogue warps. With two accumulators, 4 warps (one per TMEM lane quarter) drain a tile while
  // the MMAs fill the other. With one, the MMAs wait for the drain, so 8 warps (two per quarter,
  // each half of the columns) first load all their columns into registers, hand the accumulator
  // back, and only then convert and store.
  // Wide tiles drain chunk by chunk (their columns do not fit in registers).
  static constexpr int kEpiWarps = kNumAcc == 1 ? 8 : 4;
  static constexpr bool kEarlyRelease = kNumAcc == 1 && NSub == 1;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kWarpCols = kTileN / (kEpiWarps / 4);  // accumulator columns per epilogue warp
  static constexpr int kChunkCols = 128 / int(sizeof(OutT));  // epilogue store box width (128 B)
  static constexpr int kChunks = kWarpCols / kChunkCols;       // chunks per epilogue warp and tile
  static constexpr int kStageBufs = kEpiWarps == 4 ? 2 : 1;    // C staging buffers per epilogue warp

  // Operand majors. K-major (the default): the operand is stored [rows, K] and its smem tile is
  // rows x K. MN-major: stored [K, rows] (A^T / B^T in memory), smem tile K x rows, MN contiguous,
  // read by the MMA through MN-major descriptors (instruction-descriptor major bit 1).
  static constexpr bool kAMn = AMn;
  static constexpr bool kBMn = BMn;
  // Operand swizzle of K-major tiles. 128 B (the default) makes a stage's K one swizzle atom wide;
  // with 64 B or 32 B the same 128 bytes of K are two or four atom columns, each its own TMA box,
  // and the K-slices of the MMAs step across them (block_offset_16B).
  using swizzle = Sw;
  using ATile = std::conditional_t<AMn, SmemTile<InT, kBlockK, kCtaM>, SmemTile<InT, kCtaM, kBlockK, Sw>>;
  using BTile = std::conditional_t<BMn, SmemTile<InT, kBlockK, kCtaN>, SmemTile<InT, kCtaN, kBlockK, Sw>>;
  using CBox = SmemTile<OutT, 32, kChunkCols>;

  static constexpr uint32_t kABytes = ATile::bytes;
  static constexpr uint32_t kBSubBytes = BTile::bytes;  // one sub-tile of B
  static constexpr uint32_t kBBytes = BTile::bytes * NSub;
  static constexpr uint32_t kStageTx = (kFp6 ? (kABytes + kBBytes) / 4 * 3 : kABytes + kBBytes) + kSfaBytes + kSfbBytes;
  static constexpr uint32_t kCBytes = CBox::bytes;     // 4 KB per staging buffer
  static constexpr uint32_t kOffA = 0;
  static constexpr uint32_t kOffB = kOffA + kStages * kABytes;
  static constexpr uint32_t kOffC = kOffB + kStages * kBBytes;
  static constexpr uint32_t kOffSf = kOffC + (DirectStore ? 0u : uint32_t(kEpiWarps * kStageBufs) * kCBytes);
  static constexpr uint32_t kOffSfb = kOffSf + kStages * kSfaBytes;
  static constexpr uint32_t kOffBar = kOffSfb + kStages * kSfbBytes;
  static constexpr uint32_t kNumBars = 2 * kStages + 2 * kNumAcc + 1;
  static constexpr uint32_t kOffSlot = kOffBar + 8 * kNumBars;
  static constexpr uint32_t kSmemBytes = kOffSlot + 16 + 1024;  // + slack to align the base to 1 KB

  static constexpr bool kIsF8 = sizeof(InT) == 1;
  static constexpr uint32_t idesc() {
    if constexpr (kNv)  // scale format bit 23: 0 = UE4M3
      return mma_instr_desc_block_scaled<InT, InT, kTileM, BlockN>() & ~(1u << 23);
    else if constexpr (kMx)
      return mma_instr_desc_block_scaled<InT, InT, kTileM, BlockN>();
    else
      return mma_instr_desc<InT, InT, float, kTileM, BlockN, AMn ? UmmaMajor::MN : UmmaMajor::K,
                            BMn ? UmmaMajor::MN : UmmaMajor::K>();
  }
  static constexpr uint32_t kIdesc = idesc();

  static_assert(kTmemUsed <= 512, "accumulators and scales exceed TMEM");
  static_assert(!kMx || (sizeof(InT) == 1 && !AMn && !BMn && std::is_same_v<Sw, Swizzle128B> && BlockN % 32 == 0),
                "block-scaled: 8-bit or packed fp4 K-major operands, 128-byte swizzle, tile N a multiple of 32");
  static_assert(SfVec == 0 || SfVec == 32 || (SfVec == 16 && kFp4), "scales per 32 elements, or per 16 for fp4");
  static_assert(NSub == 1 || (NSub == 2 && !kMx && !DirectStore), "wide tiles: two sub-tiles, no block scaling");
  static_assert(!kFp4 || kMx, "packed fp4 operands are block-scaled (kind::mxf4 / mxf4nvf4)");
  static_assert(!kFp6 || SfVec == 32, "fp6 operands are MX block-scaled (kind::mxf8f6f4, a scale per 32)");
  static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
  static_assert(BlockN % (16 * CtaGroup) == 0 && BlockN <= 256, "UMMA N");
  static_assert(kCtaN % 8 == 0 && kCtaN <= 256, "B tile rows");
  static_assert(kWarpCols % kChunkCols == 0, "epilogue chunking");
  static_assert(!(kEarlyRelease && DirectStore), "the early-release epilogue stages through shared memory");
  static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "stages must keep 1 KB alignment");
  static_assert(std::is_same_v<Sw, Swizzle128B> || (!AMn && !BMn), "MN-major operands use 128-byte swizzle");
  static_assert(!std::is_same_v<Sw, SwizzleNone>, "operand tiles are swizzled");
};

struct TnArgs {
  int m, n, k;
  int tiles_m, tiles_n, k_blocks;
  int group_m;                  // raster group height, in tiles
  float alpha;                  // C = alpha * (A . B^T) [* *scale_a * *scale_b]
  const float* scale_a;         // optional device scalars (nullptr = 1)
  const float* scale_b;
  int* status;                  // device word; timeout bits are ORed in
  unsigned long long timeout_ns;
  int prefetch;                 // L2 prefetch distance, in K-blocks of the producer's sequence (0 = off)
  void* c;                      // C and its row pitch in elements (direct-store epilogue; read for C += result)
  long long ldc;
  unsigned long long* clock_probe;  // optional: per CTA {clock64, globaltimer} at start and end
  int batch;                    // independent GEMMs (rank-3 tensor maps when > 1)
  long long batch_stride_c;     // elements between the C matrices (direct stores and C reads)
  int c_reduce;                 // 0: C = result; 1: C += result (fp32 C: TMA reducing stores; 16-bit C: read, add, store)
  const int* m_block_group;     // m-grouped GEMM: B matrix of each 128-row block of A / C (-1 = padding)
  int sfb_group_blocks;         // m-grouped block-scaled: 128-row scale blocks of each group's B
  // Split tail: when the tile count leaves the last wave short, its `sk_tiles` tiles (the last in
  // tile order) are each cut into `sk_split` equal K-ranges, dealt round-robin like whole tiles in
  // range-major order, so the workers of one wave read the same K-range of neighbouring tiles and
  // keep the L2 reuse of the data-parallel waves. Each range's fp32 partial sum goes to its own slot;
  // a ticket per (tile, CTA of the pair, epilogue warp) counts them in, and the warp that arrives
  // last adds the slots in range order and stores C. 0 tail tiles = every tile whole.
  int sk_tiles;
  int sk_split;
  int* sk_tickets;              // [sk_tiles * CtaGroup * kEpiWarps], zero between launches
  float* sk_slots;              // [sk_tiles * sk_split * CtaGroup][128 * BlockN]
  // NVLink multicast address of C's element (0, 0) (pitch ldc), or nullptr. When set, every
  // finished chunk of C is read back from its staging buffer and written once with multimem
  // stores, which land in the C of every GPU bound to the multicast object (this one's included):
  // the column-sharded GEMM leaves the whole C everywhere and each GPU sends its shard once.
  void* mc_c;
};

// One piece of work: K-blocks [kb0, kb1) of tile t; q = its K-range (0 for a whole tile).
struct TilePiece {
  int t, kb0, kb1, q;
};

// The pieces one worker processes, in order: first tail pieces p = worker + j W of the sk_tiles *
// sk_split (piece p is K-range p / sk_tiles of tail tile p % sk_tiles, the tail being the last
// sk_tiles tiles), then tiles t = worker + i W of the first num_tiles - sk_tiles, whole. Split tiles
// go first so that their slot traffic and final sums overlap the whole tiles' MMAs instead of
// trailing the last wave. Producer, MMA issuer and epilogue walk the same sequence.
struct WorkSeq {
  int workers, dp_tiles, tail, split, k_blocks, t_dp, p;
  KL_HOST_DEVICE WorkSeq(int worker, int num_workers, int num_tiles, int sk_tiles, int sk_split, int k_blocks_)
      : workers(num_workers), dp_tiles(num_tiles - sk_tiles), tail(sk_tiles), split(sk_split > 0 ? sk_split : 1),
        k_blocks(k_blocks_), t_dp(worker), p(worker) {}
  KL_HOST_DEVICE bool next(TilePiece& w) {
    if (p < tail * split) {
      const int q = p / tail, r = p - q * tail;
      w = {dp_tiles + r, int((long long)q * k_blocks / split), int((long long)(q + 1) * k_blocks / split), q};
      p += workers;
      return true;
    }
    if (t_dp < dp_tiles) {
      w = {t_dp, 0, k_blocks, 0};
      t_dp += workers;
      return true;
    }
    return false;
  }
};

// Most peers an epilogue can push C tiles to (one NVLink/NVSwitch domain of 8 GPUs).
inline constexpr int kMaxPeers = 7;

struct TnParams {
  CUtensorMap map_a;  // A [M, K], box {kBlockK, 128}
  CUtensorMap map_b;  // B [N, K], box {kBlockK, kCtaN} (rank 3 [batch or groups, N, K] when batched / grouped)
  CUtensorMap map_c;  // C [M, N], box {kChunkCols, 32}
  // The same C block in other GPUs' memory (peer-mapped pointers): every finished tile is also
  // TMA-stored there, so a column-sharded GEMM leaves the whole C on every GPU with no separate
  // all-gather. Stores only; nothing in this kernel reads peer memory.
  CUtensorMap map_peer[kMaxPeers];
  int n_peers;
  // Block scales (TnConfig::kMx): the blocked arrays of A and B as [row blocks, K blocks, 128]
  // 32-bit words, box {128, kSfAtomsK, 1} = one stage's atoms of 128 rows.
  CUtensorMap map_sfa;
  CUtensorMap map_sfb;
  TnArgs args;
};

// Grouped raster: tiles [g*group_m, (g+1)*group_m) x [0, tiles_n) are visited column by column.
KL_HOST_DEVICE void tile_coords(int t, int tiles_m, int tiles_n, int group_m, int& tm, int& tn) {
  const int per_group = group_m * tiles_n;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int rows = (tiles_m - first_m) < group_m ? (tiles_m - first_m) : group_m;
  const int r = t - g * per_group;
  tm = first_m + r % rows;
  tn = r / rows;
}

// Batched tiles: all tiles of matrix 0, then matrix 1, ...; each matrix in grouped raster order.
KL_HOST_DEVICE void tile_coords(int t, int tiles_m, int tiles_n, int group_m, int& bz, int& tm, int& tn) {
  const int per_matrix = tiles_m * tiles_n;
  bz = t / per_matrix;
  tile_coords(t - bz * per_matrix, tiles_m, tiles_n, group_m, tm, tn);
}

#if defined(__CUDACC__)

KL_DEVICE void record_status(int* status, int bit) { atomicOr(status, bit); }

KL_DEVICE void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

KL_DEVICE uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
  return v;
}

KL_DEVICE uint32_t ld_shared_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

KL_DEVICE void st_global_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

KL_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Two fp32 results rounded (to nearest even) to a 16-bit output type and packed low-first.
template <typename OutT>
KL_DEVICE uint32_t pack_out2(float lo, float hi) {
  if constexpr (std::is_same_v<OutT, __half>) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    return pack_bf16x2(lo, hi);
  }
}

// Two 16-bit values (low first) widened to fp32.
template <typename OutT>
KL_DEVICE float2 unpack_out2(uint32_t u) {
  if constexpr (std::is_same_v<OutT, __half>)
    return __half22float2(*reinterpret_cast<__half2*>(&u));
  else
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
}

KL_DEVICE uint4 ld_global_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

template <typename OutT>
KL_DEVICE OutT to_out(float x) {
  if constexpr (std::is_same_v<OutT, __half>)
    return __float2half_rn(x);
  else if constexpr (std::is_same_v<OutT, __nv_bfloat16>)
    return __float2bfloat16_rn(x);
  else
    return x;
}

// Issue the TMA boxes of one operand tile. K-major tiles are (rows, K) boxes at (x = k, y = row);
// MN-major tiles are (K, rows) with the MN coordinate innermost: x = row, y = k.
template <class Tile, bool Mn, int CG>
KL_DEVICE void load_operand(uint32_t dst, const void* map, uint32_t bar, int k0, int row0, int bz, bool batched) {
  using Box = TmaBox<Tile>;
#pragma unroll
  for (int i = 0; i < Box::count; ++i) {
    const int x = Mn ? row0 + Box::col(i) : k0 + Box::col(i);
    const int y = Mn ? k0 + Box::row(i) : row0 + Box::row(i);
    const uint32_t d = dst + Box::smem_offset(i);
    if constexpr (CG == 1) {
      if (batched)
        tma_load_3d(d, map, bar, x, y, bz);
      else
        tma_load_2d(d, map, bar, x, y);
    } else {
      if (batched)
        tma_load_3d_pair(d, map, bar, x, y, bz);
      else
        tma_load_2d_pair(d, map, bar, x, y);
    }
  }
}

// Descriptor of K-slice 0 of an operand tile at `addr`, and the 16-byte-unit step to K-slice k.
template <class Tile, bool Mn>
KL_HOST_DEVICE constexpr uint64_t operand_desc0(uint32_t addr) {
  if constexpr (Mn)
    return umma_desc_mn_at<Tile>(addr, 0, 0, Tile::cols).desc_;
  else
    return umma_desc_at<Tile>(addr).desc_;
}
template <class Tile, bool Mn>
KL_HOST_DEVICE constexpr uint32_t operand_kstep_16B(int k) {
  using T = typename Tile::value_type;
  if constexpr (Mn)
    return static_cast<uint32_t>(detail::tile_offset(Tile::rows, Tile::atom_elems, k * mma_k<T>, 0) * bits_of<T> / 128);
  else
    return block_offset_16B<Tile>(k);
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::kThreads, 1) gemm_tn_kernel(const __grid_constant__ TnParams p) {
#if defined(KL_ARCH_SM100)
  using InT = typename Cfg::in_type;
  using OutT = typename Cfg::out_type;
  constexpr int CG = Cfg::kCtaGroup;
  constexpr int S = Cfg::kStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t a_smem = base + Cfg::kOffA;
  const uint32_t b_smem = base + Cfg::kOffB;
  const uint32_t c_smem = base + Cfg::kOffC;
  const uint32_t sfa_smem = base + Cfg::kOffSf;
  const uint32_t sfb_smem = base + Cfg::kOffSfb;
  const uint32_t bar0 = base + Cfg::kOffBar;
  const uint32_t tmem_slot = base + Cfg::kOffSlot;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (S + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * S + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * S + Cfg::kNumAcc + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * S + 2 * Cfg::kNumAcc);

  const TnArgs& args = p.args;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta_rank = (CG == 2) ? cluster_ctarank() : 0u;  // rank inside the pair
  const int worker = blockIdx.x / CG;
  const int num_workers = gridDim.x / CG;
  const int num_tiles = args.tiles_m * args.tiles_n * args.batch;
  const bool batched = args.batch > 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbarrier_init(full_bar(s), 1);
      mbarrier_init(empty_bar(s), 1);
    }
    for (int a = 0; a < Cfg::kNumAcc; ++a) {
      mbarrier_init(tfull_bar(a), 1);
      mbarrier_init(tempty_bar(a), Cfg::kEpiWarps * CG);  // one arrival per epilogue warp of the pair
    }
    mbarrier_init(drain_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&p.map_a);
    tma_prefetch_map(&p.map_b);
    tma_prefetch_map(&p.map_c);
    if constexpr (Cfg::kMx) {
      tma_prefetch_map(&p.map_sfa);
      tma_prefetch_map(&p.map_sfb);
    }
  }
  if (warp == 1) {
    tmem_alloc<CG>(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish<CG>();
  }
  tcgen05_fence_before();
  if constexpr (CG == 2) {
    cluster_sync();  // the peer's barriers must exist before any cross-CTA arrive or TMA
  } else {
    __syncthreads();
  }
  tcgen05_fence_after();
  const uint32_t tmem_base = ld_shared_u32(tmem_slot);
  // Launched with programmatic serialization, this CTA may have started while the previous kernel
  // on the stream still runs: the prologue above touched no global memory, everything below may.
  // Then let the next launch start its own prologue on SMs this grid leaves free.
  griddep_wait();
  griddep_launch_dependents();
  if (args.clock_probe != nullptr && threadIdx.x == 0) {
    args.clock_probe[4 * blockIdx.x + 0] = clock64();
    args.clock_probe[4 * blockIdx.x + 1] = globaltimer_ns();
  }

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (elect_one()) {
      const uint32_t leader_full0 = (CG == 2) ? mapa_shared(full_bar(0), 0) : full_bar(0);
      // L2 prefetch runs `pf` K-blocks ahead of the loads along this CTA's own sequence of
      // (tile, K-block) units, crossing into its next tile where needed.
      const int pf = args.prefetch;
      auto prefetch_unit = [&](int t, int kb) {
        while (kb >= args.k_blocks && t < num_tiles) {
          kb -= args.k_blocks;
          t += num_workers;
        }
        if (t >= num_tiles) return;
        int pbz, ptm, ptn;
        tile_coords(t, args.tiles_m, args.tiles_n, args.group_m, pbz, ptm, ptn);
        if (batched || Cfg::kAMn || Cfg::kBMn || args.m_block_group != nullptr) return;  // 2-D, K-major maps only
        tma_prefetch_l2_2d(&p.map_a, kb * Cfg::kBlockK, ptm * Cfg::kTileM + int(cta_rank) * Cfg::kCtaM);
#pragma unroll
        for (int j = 0; j < Cfg::kNSub; ++j)
          tma_prefetch_l2_2d(&p.map_b, kb * Cfg::kBlockK, ptn * Cfg::kTileN + j * Cfg::kBlockN + int(cta_rank) * Cfg::kCtaN);
      };
      if (pf > 0)
        for (int j = 0; j < pf; ++j) prefetch_unit(worker, j);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      WorkSeq seq(worker, num_workers, num_tiles, args.sk_tiles, args.sk_split, args.k_blocks);
      TilePiece pc;
      while (ok && seq.next(pc)) {
        const int t = pc.t;
        int bz, tm, tn;
        tile_coords(t, args.tiles_m, args.tiles_n, args.group_m, bz, tm, tn);
        const int a_row = tm * Cfg::kTileM + int(cta_rank) * Cfg::kCtaM;
        const int b_row = tn * Cfg::kTileN + int(cta_rank) * Cfg::kCtaN;
        // m-grouped: A and C are one [M, *] matrix, B one of a rank-3 stack, chosen per 128-row block
        // (a block marked -1 loads B as zeros: padding rows come out 0). A CTA pair's 256-row tile
        // uses the group of its first block: both blocks must name the same group.
        const int gz = args.m_block_group != nullptr ? __ldg(args.m_block_group + tm * CG) : 0;
        for (int kb = pc.kb0; kb < pc.kb1; ++kb) {
          if (pf > 0) prefetch_unit(t, kb + pf);  // data-parallel launches only (sk_tiles = 0)
          if (!mbarrier_wait(empty_bar(stage), phase ^ 1u, args.timeout_ns)) {
            record_status(args.status, kStatusProducerTimeout);
            ok = false;
            break;
          }
          const int kx = kb * Cfg::kBlockK;
          if constexpr (CG == 1) {
            mbarrier_arrive_expect_tx(full_bar(stage), Cfg::kStageTx);
            load_operand<typename Cfg::ATile, Cfg::kAMn, 1>(a_smem + stage * Cfg::kABytes, &p.map_a, full_bar(stage),
                                                            kx, a_row, bz, batched);
#pragma unroll
            for (int j = 0; j < Cfg::kNSub; ++j) {  // sub-tile j: B rows [j BlockN, (j + 1) BlockN) of the tile
              const uint32_t bd = b_smem + stage * Cfg::kBBytes + j * Cfg::kBSubBytes;
              if (args.m_block_group != nullptr)
                load_operand<typename Cfg::BTile, Cfg::kBMn, 1>(bd, &p.map_b, full_bar(stage), kx,
                                                                b_row + j * Cfg::kBlockN, gz, true);
              else
                load_operand<typename Cfg::BTile, Cfg::kBMn, 1>(bd, &p.map_b, full_bar(stage), kx,
                                                                b_row + j * Cfg::kBlockN, bz, batched);
            }
            if constexpr (Cfg::kMx) {
              // K-block kb's scale atoms: A's row block (tm) and the tile's row blocks of B (a block
              // past the end of B loads as zeros, for output columns that are never stored).
              const int sy = kb * Cfg::kSfAtomsK;  // first K atom of this stage
              tma_load_3d(sfa_smem + stage * Cfg::kSfaBytes, &p.map_sfa, full_bar(stage), 0, sy, tm);
#pragma unroll
              for (int j = 0; j < Cfg::kSfbAtoms; ++j)
                tma_load_3d(sfb_smem + stage * Cfg::kSfbBytes + 512u * Cfg::kSfAtomsK * j, &p.map_sfb, full_bar(stage),
                            0, sy, gz * args.sfb_group_blocks + (tn * Cfg::kTileN) / 128 + j);
            }
          } else {
            // The leader's barrier counts the bytes of both CTAs; only the leader arrives.
            if (cta_rank == 0)
              mbarrier_arrive_expect_tx(full_bar(stage), 2u * Cfg::kStageTx);
            const uint32_t fb = leader_full0 + 8u * stage;
            load_operand<typename Cfg::ATile, Cfg::kAMn, 2>(a_smem + stage * Cfg::kABytes, &p.map_a, fb, kx, a_row, bz,
                                                            batched);
#pragma unroll
            for (int j = 0; j < Cfg::kNSub; ++j) {  // sub-tile j: this CTA's half of its BlockN rows of B
              const uint32_t bd = b_smem + stage * Cfg::kBBytes + j * Cfg::kBSubBytes;
              if (args.m_block_group != nullptr)
                load_operand<typename Cfg::BTile, Cfg::kBMn, 2>(bd, &p.map_b, fb, kx, b_row + j * Cfg::kBlockN, gz, true);
              else
                load_operand<typename Cfg::BTile, Cfg::kBMn, 2>(bd, &p.map_b, fb, kx, b_row + j * Cfg::kBlockN, bz,
                                                                batched);
            }
            if constexpr (Cfg::kMx) {
              // Each CTA: the scales of its own 128 rows of A, and of all the tile's rows of B.
              const int sy = kb * Cfg::kSfAtomsK;
              tma_load_3d_pair(sfa_smem + stage * Cfg::kSfaBytes, &p.map_sfa, fb, 0, sy, 2 * tm + int(cta_rank));
#pragma unroll
              for (int j = 0; j < Cfg::kSfbAtoms; ++j)
                tma_load_3d_pair(sfb_smem + stage * Cfg::kSfbBytes + 512u * Cfg::kSfAtomsK * j, &p.map_sfb, fb, 0, sy,
                                 gz * args.sfb_group_blocks + (tn * Cfg::kTileN) / 128 + j);
            }
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let copies already in flight land before the CTA can exit (bounded, short).
        for (int s = 0; s < S; ++s) (void)mbarrier_wait(empty_bar(s), phase ^ 1u, 1000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if ((CG == 1 || cta_rank == 0) && elect_one()) {
      const uint64_t a_desc0 = operand_desc0<typename Cfg::ATile, Cfg::kAMn>(a_smem);
      const uint64_t b_desc0 = operand_desc0<typename Cfg::BTile, Cfg::kBMn>(b_smem);
      const uint32_t peer = cta_rank ^ 1u;
      uint32_t stage = 0, phase = 0;
      uint32_t iter = 0;
      bool ok = true;
      WorkSeq seq(worker, num_workers, num_tiles, args.sk_tiles, args.sk_split, args.k_blocks);
      TilePiece pc;
      for (; ok && seq.next(pc); ++iter) {
        const int t = pc.t;
        const uint32_t acc = iter % Cfg::kNumAcc;
        const uint32_t acc_phase = (iter / Cfg::kNumAcc) & 1u;
        if (!mbarrier_wait(tempty_bar(acc), acc_phase ^ 1u, args.timeout_ns)) {
          record_status(args.status, kStatusMmaTimeout);
          ok = false;
          break;
        }
        tcgen05_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kAccCols;
        uint32_t sfb_word = 0;  // first TMEM word of B's scales for this tile's rows
        if constexpr (Cfg::kMx) {
          int tbz, ttm, ttn;
          tile_coords(t, args.tiles_m, args.tiles_n, args.group_m, tbz, ttm, ttn);
          sfb_word = uint32_t(((ttn * Cfg::kTileN) % 128) / 32);
        }
        for (int kb = pc.kb0; kb < pc.kb1; ++kb) {
          if (!mbarrier_wait(full_bar(stage), phase, args.timeout_ns)) {
            record_status(args.status, kStatusMmaTimeout);
            ok = false;
            break;
          }
          tcgen05_fence_after();
          const uint64_t a_desc = a_desc0 + ((stage * Cfg::kABytes) >> 4);
          const uint64_t b_desc = b_desc0 + ((stage * Cfg::kBBytes) >> 4);
          if constexpr (Cfg::kMx) {
            // The stage's scales into TMEM: one 32x128b copy (replicated to the four lane quarters)
            // per 128 rows; the MMAs below are ordered after these copies.
            // TMEM: A's atom q at kSfaCol + 4q; B's K atom q at kSfbCol + 4 * kSfbAtoms * q, its row blocks
            // side by side (rows r of the tile in 32-bit word r / 32).
#pragma unroll
            for (int q = 0; q < Cfg::kSfAtomsK; ++q) {
              tmem_cp_32x128b_warpx4<CG>(
                  tmem_base + Cfg::kSfaCol + 4 * q,
                  encode_smem_desc(sfa_smem + stage * Cfg::kSfaBytes + 512u * q, 0, 128, UmmaLayout::SWIZZLE_NONE));
#pragma unroll
              for (int j = 0; j < Cfg::kSfbAtoms; ++j)
                tmem_cp_32x128b_warpx4<CG>(
                    tmem_base + Cfg::kSfbCol + 4 * (q * Cfg::kSfbAtoms + j),
                    encode_smem_desc(sfb_smem + stage * Cfg::kSfbBytes + 512u * (j * Cfg::kSfAtomsK + q), 0, 128,
                                     UmmaLayout::SWIZZLE_NONE));
            }
          }
#pragma unroll
          for (int k = 0; k < Cfg::kBlockK / Cfg::kUmmaK; ++k) {
            const uint64_t ka = operand_kstep_16B<typename Cfg::ATile, Cfg::kAMn>(k);
            const uint64_t kb16 = operand_kstep_16B<typename Cfg::BTile, Cfg::kBMn>(k);
            const uint32_t accumulate = (kb != pc.kb0) || (k != 0);  // a piece starts a fresh sum
            if constexpr (Cfg::kMx) {
              // K-slice k: scale atom q, starting at byte `id` of every 32-bit scale word.
              const int q = k / Cfg::kMmasPerSfAtom;
              const uint32_t id = uint32_t(k % Cfg::kMmasPerSfAtom) * Cfg::kSfIdStep;
              const uint32_t idesc = Cfg::kIdesc | (id << 29) | (id << 4);
              const uint32_t sfa_t = tmem_base + Cfg::kSfaCol + 4 * q;
              const uint32_t sfb_t = tmem_base + Cfg::kSfbCol + 4 * Cfg::kSfbAtoms * q + sfb_word;
              if constexpr (Cfg::kNv)
                umma_nvf4_ss<CG>(d_tmem, a_desc + ka, b_desc + kb16, idesc, sfa_t, sfb_t, accumulate);
              else if constexpr (Cfg::kFp4)
                umma_mxf4_ss<CG>(d_tmem, a_desc + ka, b_desc + kb16, idesc, sfa_t, sfb_t, accumulate);
              else
                umma_mxf8_ss<CG>(d_tmem, a_desc + ka, b_desc + kb16, idesc, sfa_t, sfb_t, accumulate);
            }
            else {
#pragma unroll
              for (int j = 0; j < Cfg::kNSub; ++j) {  // sub-tile j into accumulator columns [j BlockN, ...)
                const uint64_t bj = b_desc + kb16 + ((j * Cfg::kBSubBytes) >> 4);
                const uint32_t dj = d_tmem + uint32_t(j * Cfg::kBlockN);
                if constexpr (Cfg::kIsF8)
                  umma_f8_ss<CG>(dj, a_desc + ka, bj, Cfg::kIdesc, accumulate);
                else
                  umma_f16_ss<CG>(dj, a_desc + ka, bj, Cfg::kIdesc, accumulate);
              }
            }
          }
          // Stage consumed once these MMAs complete: release it in both CTAs of the pair.
          umma_commit<CG>(empty_bar(stage));
          if constexpr (CG == 2) umma_commit<CG>(mapa_shared(empty_bar(stage), peer));
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit<CG>(tfull_bar(acc));
        if constexpr (CG == 2) umma_commit<CG>(mapa_shared(tfull_bar(acc), peer));
      }
      // Every MMA this thread issued must finish before TMEM is freed.
      umma_commit<CG>(drain_bar);
      if (!mbarrier_wait(drain_bar, 0, args.timeout_ns)) record_status(args.status, kStatusDrainTimeout);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..)
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int ew = warp - 2;       // epilogue warp index -> staging buffers
    const int wcol = (ew / 4) * Cfg::kWarpCols;  // this warp's first accumulator column
    const uint32_t lane_base = uint32_t(quarter * 32) << 16;
    float alpha = args.alpha;
    if (args.scale_a != nullptr) alpha *= *args.scale_a;
    if (args.scale_b != nullptr) alpha *= *args.scale_b;
    const uint32_t tempty_leader0 = (CG == 2) ? mapa_shared(tempty_bar(0), 0) : tempty_bar(0);
    uint32_t nbuf = 0;
    int bz = 0, row0 = 0;

    // Chunk `col` (kChunkCols fp32 accumulator columns of this thread's row, in v) scaled, converted
    // and written to C: through a swizzled staging buffer and a TMA store (or reducing store), or
    // straight from registers (direct-store configs).
    auto emit_chunk = [&](const uint32_t* v, int col) {
      if constexpr (Cfg::kDirectStore) {
        // Each thread owns one row of the chunk (128 bytes of C): eight 16-byte stores, or
        // element by element on the ragged right edge.
        const int row = row0 + lane;
        if (row < args.m && col < args.n) {
          OutT* dst = static_cast<OutT*>(args.c) + (long long)bz * args.batch_stride_c + (long long)row * args.ldc + col;
          if (col + Cfg::kChunkCols <= args.n) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if constexpr (sizeof(OutT) == 2) {
                const float* f = reinterpret_cast<const float*>(&v[8 * j]);
                st_global_v4(dst + 8 * j, pack_out2<OutT>(f[0] * alpha, f[1] * alpha),
                             pack_out2<OutT>(f[2] * alpha, f[3] * alpha), pack_out2<OutT>(f[4] * alpha, f[5] * alpha),
                             pack_out2<OutT>(f[6] * alpha, f[7] * alpha));
              } else {
                const float* f = reinterpret_cast<const float*>(&v[4 * j]);
                st_global_v4(dst + 4 * j, __float_as_uint(f[0] * alpha), __float_as_uint(f[1] * alpha),
                             __float_as_uint(f[2] * alpha), __float_as_uint(f[3] * alpha));
              }
            }
          } else {
#pragma unroll
            for (int e = 0; e < Cfg::kChunkCols; ++e)  // unrolled: v stays in registers
              if (col + e < args.n) dst[e] = to_out<OutT>(__uint_as_float(v[e]) * alpha);
          }
        }
      } else {
        const bool store = row0 < args.m && col < args.n;
        const uint32_t buf = c_smem + uint32_t(ew * Cfg::kStageBufs + (nbuf % Cfg::kStageBufs)) * Cfg::kCBytes;
        // The buffer's previous store must have finished reading it.
        if (lane == 0) tma_store_wait_read<Cfg::kStageBufs - 1>();
        __syncwarp();
        const uint32_t row_addr = buf + uint32_t(lane) * 128u;
        const uint32_t sw = uint32_t(lane & 7);
        if constexpr (sizeof(OutT) == 2) {
          // C += result on a 16-bit C: the TMA unit's reducing store would round twice, so each thread
          // reads its row of the chunk, 16 bytes at a time, adds in fp32 and the sum is stored, rounded
          // once.
          const int row = row0 + lane;
          const bool add = args.c_reduce && row < args.m && col < args.n;
          const OutT* src =
              static_cast<const OutT*>(args.c) + (long long)bz * args.batch_stride_c + (long long)row * args.ldc + col;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 old = make_uint4(0u, 0u, 0u, 0u);
            if (add) {
              if (col + 8 * j + 8 <= args.n) {
                old = ld_global_v4(src + 8 * j);
              } else {
                uint16_t h[8] = {};
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  if (col + 8 * j + e < args.n) h[e] = reinterpret_cast<const uint16_t*>(src)[8 * j + e];
                old = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                                 h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
              }
            }
            const float* f = reinterpret_cast<const float*>(&v[8 * j]);
            const float2 o0 = unpack_out2<OutT>(old.x), o1 = unpack_out2<OutT>(old.y);
            const float2 o2 = unpack_out2<OutT>(old.z), o3 = unpack_out2<OutT>(old.w);
            st_shared_v4(row_addr + ((uint32_t(j) ^ sw) << 4), pack_out2<OutT>(f[0] * alpha + o0.x, f[1] * alpha + o0.y),
                         pack_out2<OutT>(f[2] * alpha + o1.x, f[3] * alpha + o1.y),
                         pack_out2<OutT>(f[4] * alpha + o2.x, f[5] * alpha + o2.y),
                         pack_out2<OutT>(f[6] * alpha + o3.x, f[7] * alpha + o3.y));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float* f = reinterpret_cast<const float*>(&v[4 * j]);
            st_shared_v4(row_addr + ((uint32_t(j) ^ sw) << 4), __float_as_uint(f[0] * alpha),
                         __float_as_uint(f[1] * alpha), __float_as_uint(f[2] * alpha), __float_as_uint(f[3] * alpha));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (args.mc_c != nullptr) {
          // Multicast C: the warp reads its 32 staged rows back, four rows of 128 bytes per pass
          // (lane = 8 x row-in-pass + 16-byte piece), and stores every piece once to the multicast
          // address, coalesced along the rows. The host checks that the base, the pitch and the
          // width of C are multiples of 16 bytes, so a piece is wholly in or out of C.
          if (store) {
            const int piece = lane & 7;
            const int pcol = col + piece * (16 / int(sizeof(OutT)));
#pragma unroll
            for (int it = 0; it < 8; ++it) {
              const int r = it * 4 + (lane >> 3);
              const uint4 x = ld_shared_v4(buf + uint32_t(r) * 128u + ((uint32_t(piece) ^ uint32_t(r & 7)) << 4));
              if (row0 + r < args.m && pcol < args.n)
                multimem_st_v4(static_cast<OutT*>(args.mc_c) + (long long)(row0 + r) * args.ldc + pcol, x.x, x.y, x.z,
                               x.w);
            }
          }
          __syncwarp();  // every lane's reads of this buffer before any lane writes it again
        } else if (lane == 0) {
          if (store) {
            if (args.c_reduce && sizeof(OutT) == 4) {
              // C += tile on an fp32 C: the TMA unit reads C, adds the staged values and writes back.
              if (batched) {
                tma_reduce_add_3d(&p.map_c, buf, col, row0, bz);
                for (int q = 0; q < p.n_peers; ++q) tma_reduce_add_3d(&p.map_peer[q], buf, col, row0, bz);
              } else {
                tma_reduce_add_2d(&p.map_c, buf, col, row0);
                for (int q = 0; q < p.n_peers; ++q) tma_reduce_add_2d(&p.map_peer[q], buf, col, row0);
              }
            } else if (batched) {
              tma_store_3d(&p.map_c, buf, col, row0, bz);
              for (int q = 0; q < p.n_peers; ++q) tma_store_3d(&p.map_peer[q], buf, col, row0, bz);
            } else {
              tma_store_2d(&p.map_c, buf, col, row0);
              for (int q = 0; q < p.n_peers; ++q) tma_store_2d(&p.map_peer[q], buf, col, row0);
            }
          }
          tma_store_commit();  // one group per chunk, empty or not, so wait_read tracks buffers
        }
        ++nbuf;
      }
    };
    // This warp is done reading the accumulator: hand it back to the MMA issuer.
    auto release = [&](uint32_t acc) {
      tcgen05_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2)
          mbarrier_arrive_cluster(tempty_leader0 + 8u * acc);
        else
          mbarrier_arrive(tempty_bar(acc));
      }
    };
    auto load_chunk = [&](uint32_t taddr, uint32_t* v) {
      tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      if constexpr (Cfg::kChunkCols == 64) tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
    };

    // Split tail: each K-range of a tail tile leaves its fp32 partial sum in its own slot (the CTA's
    // 128 x BlockN block), then each epilogue warp counts in on its own ticket; the warp that
    // arrives last adds the slots in K-range order, so the sum does not depend on arrival order, and
    // stores C. Nothing waits on another CTA.
    const int dp_tiles = num_tiles - args.sk_tiles;
    const int erow = quarter * 32 + lane;  // this thread's row of the CTA's 128
    auto slot_of = [&](int q, int r) -> float* {  // K-range q of tail tile r
      const long long piece = (long long)q * args.sk_tiles + r;
      return args.sk_slots + (piece * CG + cta_rank) * (128LL * Cfg::kTileN);
    };
    // Element (r, c) of a slot at ((c / 4) * 128 + r) * 4 + c % 4: one 16-byte store or load per
    // thread covers four columns of its row, and a warp's 32 rows are 512 contiguous bytes.
    auto slot_store = [&](float* slot, int tcol_rel, const uint32_t* v) {
      float4* dst = reinterpret_cast<float4*>(slot) + (long long)(tcol_rel >> 2) * 128 + erow;
#pragma unroll
      for (int j = 0; j < Cfg::kChunkCols / 4; ++j)
        __stcg(dst + 128 * j, make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                          __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3])));
    };
    auto slot_add = [&](const float* slot, int tcol_rel, float* sum) {
      const float4* src = reinterpret_cast<const float4*>(slot) + (long long)(tcol_rel >> 2) * 128 + erow;
#pragma unroll
      for (int j = 0; j < Cfg::kChunkCols / 4; ++j) {
        const float4 x = __ldcg(src + 128 * j);  // L2: written by other SMs during this launch
        sum[4 * j] += x.x;
        sum[4 * j + 1] += x.y;
        sum[4 * j + 2] += x.z;
        sum[4 * j + 3] += x.w;
      }
    };

    uint32_t iter = 0;
    WorkSeq seq(worker, num_workers, num_tiles, args.sk_tiles, args.sk_split, args.k_blocks);
    TilePiece pc;
    for (; seq.next(pc); ++iter) {
      const int t = pc.t;
      int tm, tn;
      tile_coords(t, args.tiles_m, args.tiles_n, args.group_m, bz, tm, tn);
      const uint32_t acc = iter % Cfg::kNumAcc;
      const uint32_t acc_phase = (iter / Cfg::kNumAcc) & 1u;
      if (!mbarrier_wait(tfull_bar(acc), acc_phase, args.timeout_ns)) {
        if (lane == 0) record_status(args.status, kStatusEpilogueTimeout);
        break;
      }
      tcgen05_fence_after();
      row0 = tm * Cfg::kTileM + int(cta_rank) * Cfg::kCtaM + quarter * 32;
      const int col0 = tn * Cfg::kTileN + wcol;
      const uint32_t tcol = tmem_base + lane_base + acc * Cfg::kAccCols + uint32_t(wcol);
      const bool split = Cfg::kNSub == 1 && t >= dp_tiles && args.sk_split > 1;
      if (split) {
        // A K-range of a tail tile: its partial sum into its slot, then the ticket.
        // (Chunk by chunk in every config: split tiles are few, registers are not.)
        const int r = t - dp_tiles;
        float* own = slot_of(pc.q, r);
#pragma unroll 1
        for (int c = 0; c < Cfg::kChunks; ++c) {
          uint32_t v[Cfg::kChunkCols];
          load_chunk(tcol + uint32_t(c * Cfg::kChunkCols), v);
          tmem_wait_ld();
          if (c == Cfg::kChunks - 1) release(acc);
          slot_store(own, wcol + c * Cfg::kChunkCols, v);
        }
        __threadfence();  // this thread's slot writes before the warp's arrival
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          int* ticket = args.sk_tickets + ((long long)r * CG + cta_rank) * Cfg::kEpiWarps + ew;
          last = atomicAdd(ticket, 1) == args.sk_split - 1;
          if (last) {
            atomicExch(ticket, 0);  // ready for the next launch
            __threadfence();        // the other contributors' slots before the reads below
          }
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        __syncwarp();
        if (last) {
#pragma unroll 1
          for (int c = 0; c < Cfg::kChunks; ++c) {
            uint32_t v[Cfg::kChunkCols];  // the sum, as fp32 bits (emit_chunk's accumulator form)
            float* sum = reinterpret_cast<float*>(v);
#pragma unroll
            for (int e = 0; e < Cfg::kChunkCols; ++e) sum[e] = 0.0f;
            // The slots two at a time, both loads in flight before either is added (the L2 round
            // trips, not the adds, bound this sum), still added in K-range order.
            const int trel = wcol + c * Cfg::kChunkCols;
            int q = 0;
#pragma unroll 1
            for (; q + 1 < args.sk_split; q += 2) {
              const float4* s0 = reinterpret_cast<const float4*>(slot_of(q, r)) + (long long)(trel >> 2) * 128 + erow;
              const float4* s1 = reinterpret_cast<const float4*>(slot_of(q + 1, r)) + (long long)(trel >> 2) * 128 + erow;
              float4 x0[Cfg::kChunkCols / 4], x1[Cfg::kChunkCols / 4];
#pragma unroll
              for (int j = 0; j < Cfg::kChunkCols / 4; ++j) {
                x0[j] = __ldcg(s0 + 128 * j);
                x1[j] = __ldcg(s1 + 128 * j);
              }
#pragma unroll
              for (int j = 0; j < Cfg::kChunkCols / 4; ++j) {
                sum[4 * j] += x0[j].x;
                sum[4 * j + 1] += x0[j].y;
                sum[4 * j + 2] += x0[j].z;
                sum[4 * j + 3] += x0[j].w;
              }
#pragma unroll
              for (int j = 0; j < Cfg::kChunkCols / 4; ++j) {
                sum[4 * j] += x1[j].x;
                sum[4 * j + 1] += x1[j].y;
                sum[4 * j + 2] += x1[j].z;
                sum[4 * j + 3] += x1[j].w;
              }
            }
            if (q < args.sk_split) slot_add(slot_of(q, r), trel, sum);
            emit_chunk(v, col0 + c * Cfg::kChunkCols);
          }
        }
      } else if constexpr (Cfg::kEarlyRelease) {
        // All of this warp's columns into registers, accumulator back to the MMAs, then the stores.
        uint32_t v[Cfg::kWarpCols];
#pragma unroll
        for (int c = 0; c < Cfg::kChunks; ++c) load_chunk(tcol + uint32_t(c * Cfg::kChunkCols), &v[c * Cfg::kChunkCols]);
        tmem_wait_ld();
        release(acc);
#pragma unroll
        for (int c = 0; c < Cfg::kChunks; ++c) emit_chunk(&v[c * Cfg::kChunkCols], col0 + c * Cfg::kChunkCols);
      } else {
#pragma unroll 1
        for (int c = 0; c < Cfg::kChunks; ++c) {
          uint32_t v[Cfg::kChunkCols];
          load_chunk(tcol + uint32_t(c * Cfg::kChunkCols), v);
          tmem_wait_ld();
          if (c == Cfg::kChunks - 1) release(acc);
          emit_chunk(v, col0 + c * Cfg::kChunkCols);
        }
      }
    }
    if constexpr (!Cfg::kDirectStore) {
      if (lane == 0) tma_store_wait<0>();
    }
    if (args.mc_c != nullptr) multimem_fence();  // this thread's multicast stores, before the kernel ends
  }

  // ------------------------------------------------------------------ teardown
  __syncwarp();
  tcgen05_fence_before();
  if constexpr (CG == 2) {
    cluster_sync();  // neither CTA frees TMEM or exits while the pair still signals it
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tcgen05_fence_after();
    tmem_dealloc<CG>(tmem_base, Cfg::kTmemCols);
  }
  if (args.clock_probe != nullptr && threadIdx.x == 0) {
    args.clock_probe[4 * blockIdx.x + 2] = clock64();
    args.clock_probe[4 * blockIdx.x + 3] = globaltimer_ns();
  }
#endif  // KL_ARCH_SM100
}

#endif  // __CUDACC__

}  // namespace kl::gemm
