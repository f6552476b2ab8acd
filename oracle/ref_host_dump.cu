// Reference descriptor tables, computed by the reference's OWN headers (kernel_lib/include/kl)
// compiled against CUTLASS/CuTe 4.5.0. TEST INFRASTRUCTURE ONLY: built by oracle/Makefile into
// oracle/_ref/ref_host_dump from the sources under the reference checkout; its JSON output is
// committed as tests/golden/ref_host_tables.json by tests/golden/gen_golden.py.
//
// Host-only parts: smem layouts (kernel_lib/include/kl/layout/smem_tile.hpp:33-76), TmaBox
// (kernel_lib/include/kl/layout/tma_desc.hpp:47-74), block_offset_16B and the UMMA smem descriptor
// body of kl::umma_desc evaluated at shared address 0 (kernel_lib/include/kl/layout/umma_desc.hpp:
// 24-47; CuTe's host path of cast_smem_ptr_to_uint yields 0), and mma_instr_desc
// (kernel_lib/include/kl/layout/umma_desc.hpp:51-58). Instruction descriptors the reference rejects
// (M = 256) come from CuTe's make_instr_desc directly and are tagged "cute".
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include <kl/kl.hpp>

namespace {

FILE* out = nullptr;
bool first_entry = true;

void begin_entry() {
  std::fprintf(out, first_entry ? "\n" : ",\n");
  first_entry = false;
}

template <typename T>
const char* tname();
template <> const char* tname<kl::bf16>() { return "bf16"; }
template <> const char* tname<kl::f16>() { return "f16"; }
template <> const char* tname<float>() { return "f32"; }
template <> const char* tname<int8_t>() { return "i8"; }
template <> const char* tname<kl::e4m3>() { return "e4m3"; }
template <> const char* tname<kl::e5m2>() { return "e5m2"; }

template <typename Tile>
void dump_tile() {
  using T = typename Tile::value_type;
  using Box = kl::TmaBox<Tile>;
  begin_entry();
  std::fprintf(out, "{\"kind\": \"tile\", \"type\": \"%s\", \"rows\": %d, \"cols\": %d, \"swizzle\": %d, ", tname<T>(),
               Tile::rows, Tile::cols, Tile::swizzle::bytes);
  std::fprintf(out, "\"bytes\": %d, \"alignment\": %d, \"atom_elems\": %d, ", Tile::bytes, Tile::alignment,
               Tile::atom_elems);
  // Layout offsets, as layout_type{}(r, c) and as element distance through tile.tensor() on a
  // 1 KB-aligned host tile (where the swizzle of the pointer's address bits applies).
  alignas(1024) static unsigned char storage[1 << 20];
  Tile& tile = *reinterpret_cast<Tile*>(storage);
  auto L = typename Tile::layout_type{};
  auto inner = L.layout_b();
  std::fprintf(out, "\"layout\": [");
  for (int r = 0; r < Tile::rows; ++r)
    for (int c = 0; c < Tile::cols; ++c) std::fprintf(out, "%s%lld", (r | c) ? "," : "", (long long)L(r, c));
  std::fprintf(out, "], \"layout_b\": [");
  for (int r = 0; r < Tile::rows; ++r)
    for (int c = 0; c < Tile::cols; ++c) std::fprintf(out, "%s%lld", (r | c) ? "," : "", (long long)inner(r, c));
  std::fprintf(out, "], \"tensor\": [");
  auto t = tile.tensor();
  for (int r = 0; r < Tile::rows; ++r)
    for (int c = 0; c < Tile::cols; ++c)
      std::fprintf(out, "%s%lld", (r | c) ? "," : "", (long long)(&t(r, c) - tile.data()));
  std::fprintf(out, "], ");
  std::fprintf(out, "\"box\": {\"inner\": %d, \"outer\": %d, \"col_boxes\": %d, \"row_boxes\": %d, \"count\": %d, \"bytes\": %d, \"pos\": [",
               Box::inner, Box::outer, Box::col_boxes, Box::row_boxes, Box::count, Box::bytes);
  for (int i = 0; i < Box::count; ++i)
    std::fprintf(out, "%s[%d, %d, %u]", i ? "," : "", Box::row(i), Box::col(i), Box::smem_offset(i));
  std::fprintf(out, "]}");
  if constexpr (Tile::cols % kl::mma_k<T> == 0) {
    constexpr int nk = kl::num_k_blocks<Tile>;
    std::fprintf(out, ", \"num_k_blocks\": %d, \"block_offset_16B\": [", nk);
    bool f = true;
    for (int row = 0; row < Tile::rows; row += 8)
      for (int k = 0; k < nk; ++k) {
        std::fprintf(out, "%s[%d, %d, %u]", f ? "" : ",", row, k, kl::block_offset_16B<Tile>(k, row));
        f = false;
      }
    std::fprintf(out, "], \"umma_desc_base0\": [");
    // kl::umma_desc's body (umma_desc.hpp:40-45) on the host: CuTe's descriptor of the first
    // (Rows x mma_k) slice, then the 32-bit add of block_offset_16B.
    f = true;
    for (int row = 0; row < Tile::rows; row += 8)
      for (int k = 0; k < nk; ++k) {
        auto first = cute::local_tile(tile.tensor(), cute::Shape<cute::Int<Tile::rows>, cute::Int<kl::mma_k<T>>>{},
                                      cute::make_coord(0, 0));
        kl::SmemDesc desc = cute::UMMA::make_umma_desc<cute::UMMA::Major::K>(first);
        desc.lo += kl::block_offset_16B<Tile>(k, row);
        std::fprintf(out, "%s[%d, %d, \"0x%016llx\"]", f ? "" : ",", row, k, (unsigned long long)desc.desc_);
        f = false;
      }
    std::fprintf(out, "]");
  }
  std::fprintf(out, "}");
}

// MN-major operand tiles (no counterpart in the reference, which is K-major only): CuTe's own
// canonical MN-major atom tiled K-groups first (Step<_2,_1>), the arrangement a TMA box of
// one swizzle span of MN by all K rows produces. Records CuTe's physical offsets and
// make_umma_desc<Major::MN> for every K-slice at shared address 0.
template <typename T, int MN, int K, typename Atom, int SwBytes>
void dump_mn_tile(const char* sw_name) {
  begin_entry();
  auto L = cute::tile_to_shape(Atom{}, cute::Shape<cute::Int<MN>, cute::Int<K>>{}, cute::Step<cute::_2, cute::_1>{});
  alignas(1024) static unsigned char storage[1 << 20];
  T* base = reinterpret_cast<T*>(storage);
  auto t = cute::make_tensor(cute::make_smem_ptr(base), L);
  std::fprintf(out, "{\"kind\": \"mn_tile\", \"type\": \"%s\", \"mn\": %d, \"k\": %d, \"swizzle\": %d, \"tensor\": [", tname<T>(),
               MN, K, SwBytes);
  bool f = true;
  for (int k = 0; k < K; ++k)
    for (int mn = 0; mn < MN; ++mn) {
      std::fprintf(out, "%s%lld", f ? "" : ",", (long long)(&t(mn, k) - base));
      f = false;
    }
  std::fprintf(out, "], \"umma_desc_mn_base0\": [");
  constexpr int mk = kl::mma_k<T>;
  for (int kb = 0; kb < K / mk; ++kb) {
    auto slice = cute::local_tile(t, cute::Shape<cute::Int<MN>, cute::Int<mk>>{}, cute::make_coord(0, kb));
    kl::SmemDesc d = cute::UMMA::make_umma_desc<cute::UMMA::Major::MN>(slice);
    // make_umma_desc reads the slice's address through the host path (0): add the slice offset.
    d.desc_ += uint64_t((&slice(0, 0) - base) * sizeof(T) >> 4);
    std::fprintf(out, "%s\"0x%016llx\"", kb ? "," : "", (unsigned long long)d.desc_);
  }
  std::fprintf(out, "]}");
  (void)sw_name;
}

template <typename A, typename B, typename Acc, int M, int N>
void dump_idesc_ref() {
  begin_entry();
  std::fprintf(out, "{\"kind\": \"idesc\", \"a\": \"%s\", \"b\": \"%s\", \"acc\": \"%s\", \"m\": %d, \"n\": %d, \"source\": \"kl\", \"value\": \"0x%08x\"}",
               tname<A>(), tname<B>(), tname<Acc>(), M, N, (unsigned)kl::mma_instr_desc<A, B, Acc, M, N>());
}

template <typename A, typename B, typename Acc, int M, int N>
void dump_idesc_cute() {
  begin_entry();
  auto d = cute::UMMA::make_instr_desc<A, B, Acc, M, N, cute::UMMA::Major::K, cute::UMMA::Major::K>();
  std::fprintf(out, "{\"kind\": \"idesc\", \"a\": \"%s\", \"b\": \"%s\", \"acc\": \"%s\", \"m\": %d, \"n\": %d, \"source\": \"cute\", \"value\": \"0x%08x\"}",
               tname<A>(), tname<B>(), tname<Acc>(), M, N, (unsigned)d.desc_);
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: %s out.json\n", argv[0]);
    return 2;
  }
  out = std::fopen(argv[1], "w");
  if (!out) return 1;
  std::fprintf(out, "[");
  using kl::SmemTile;
  dump_tile<SmemTile<kl::bf16, 128, 64>>();
  dump_tile<SmemTile<kl::bf16, 256, 64>>();
  dump_tile<SmemTile<kl::bf16, 128, 128>>();
  dump_tile<SmemTile<kl::bf16, 512, 64>>();
  dump_tile<SmemTile<kl::bf16, 512, 128>>();
  dump_tile<SmemTile<kl::bf16, 128, 64, kl::Swizzle64B>>();
  dump_tile<SmemTile<kl::bf16, 256, 64, kl::Swizzle64B>>();
  dump_tile<SmemTile<kl::bf16, 128, 32, kl::Swizzle64B>>();
  dump_tile<SmemTile<kl::bf16, 128, 32, kl::Swizzle32B>>();
  dump_tile<SmemTile<kl::bf16, 128, 16, kl::Swizzle32B>>();
  dump_tile<SmemTile<kl::bf16, 128, 64, kl::Swizzle64B>>();  // 128 B of K as 2 or 4 atom columns
  dump_tile<SmemTile<kl::bf16, 128, 64, kl::Swizzle32B>>();
  dump_tile<SmemTile<kl::bf16, 128, 8, kl::SwizzleNone>>();
  dump_tile<SmemTile<kl::bf16, 128, 16, kl::SwizzleNone>>();
  dump_tile<SmemTile<kl::bf16, 32, 64>>();
  dump_tile<SmemTile<kl::f16, 128, 64>>();
  dump_tile<SmemTile<int8_t, 128, 128>>();
  dump_tile<SmemTile<int8_t, 256, 128>>();
  dump_tile<SmemTile<kl::e4m3, 128, 128>>();
  dump_tile<SmemTile<kl::e4m3, 256, 128>>();
  dump_tile<SmemTile<float, 128, 32>>();
  dump_tile<SmemTile<float, 32, 32>>();
  dump_tile<SmemTile<float, 64, 32, kl::Swizzle64B>>();

  namespace GM = cute::SM90::GMMA;
  dump_mn_tile<kl::bf16, 128, 64, GM::Layout_MN_SW128_Atom<kl::bf16>, 128>("sw128");
  dump_mn_tile<kl::bf16, 256, 64, GM::Layout_MN_SW128_Atom<kl::bf16>, 128>("sw128");
  dump_mn_tile<kl::bf16, 128, 32, GM::Layout_MN_SW64_Atom<kl::bf16>, 64>("sw64");
  dump_mn_tile<kl::bf16, 64, 32, GM::Layout_MN_SW32_Atom<kl::bf16>, 32>("sw32");
  dump_mn_tile<kl::e4m3, 128, 128, GM::Layout_MN_SW128_Atom<kl::e4m3>, 128>("sw128");

  dump_idesc_ref<kl::bf16, kl::bf16, float, 128, 256>();
  dump_idesc_ref<kl::bf16, kl::bf16, float, 128, 128>();
  dump_idesc_ref<kl::bf16, kl::bf16, float, 128, 16>();
  dump_idesc_ref<kl::bf16, kl::bf16, float, 128, 64>();
  dump_idesc_ref<kl::bf16, kl::bf16, float, 64, 8>();
  dump_idesc_ref<kl::bf16, kl::bf16, float, 64, 256>();
  dump_idesc_ref<kl::f16, kl::f16, float, 128, 256>();
  dump_idesc_ref<kl::f16, kl::f16, kl::f16, 128, 128>();
  dump_idesc_ref<kl::e4m3, kl::e4m3, float, 128, 256>();
  dump_idesc_ref<kl::e4m3, kl::e4m3, float, 128, 128>();
  dump_idesc_ref<kl::e4m3, kl::e4m3, float, 64, 64>();
  dump_idesc_ref<kl::e5m2, kl::e5m2, float, 128, 256>();
  dump_idesc_ref<kl::e5m2, kl::e5m2, float, 128, 128>();
  dump_idesc_ref<kl::e4m3, kl::e5m2, float, 128, 256>();
  dump_idesc_cute<kl::bf16, kl::bf16, float, 256, 256>();
  dump_idesc_cute<kl::bf16, kl::bf16, float, 256, 128>();
  dump_idesc_cute<kl::e4m3, kl::e4m3, float, 256, 256>();
  dump_idesc_cute<kl::f16, kl::f16, float, 256, 64>();
  dump_idesc_cute<kl::f16, kl::f16, float, 256, 256>();
  dump_idesc_cute<kl::e5m2, kl::e5m2, float, 256, 256>();
  {  // MN-major operand bits (a_major / b_major = 1), CuTe's encoder.
    auto mn = [](auto d, const char* what) {
      begin_entry();
      std::fprintf(out, "{\"kind\": \"idesc_major\", \"what\": \"%s\", \"value\": \"0x%08x\"}", what, (unsigned)d.desc_);
    };
    using cute::UMMA::Major;
    mn(cute::UMMA::make_instr_desc<kl::bf16, kl::bf16, float, 128, 256, Major::MN, Major::K>(), "bf16 M128 N256 A=MN B=K");
    mn(cute::UMMA::make_instr_desc<kl::bf16, kl::bf16, float, 128, 256, Major::K, Major::MN>(), "bf16 M128 N256 A=K B=MN");
    mn(cute::UMMA::make_instr_desc<kl::bf16, kl::bf16, float, 256, 256, Major::MN, Major::MN>(), "bf16 M256 N256 A=MN B=MN");
  }
  {  // Block-scaled (MXFP8) instruction descriptors, CuTe's encoder: UE8M0 scales, K-major operands;
     // the runtime form carries the scale-factor ids (TMEM byte of the scale word) in bits 29-30 / 4-5.
    auto bs = [](uint32_t d, const char* a, const char* b, int m, int n, int a_sf, int b_sf) {
      begin_entry();
      std::fprintf(out, "{\"kind\": \"idesc_block_scaled\", \"a\": \"%s\", \"b\": \"%s\", \"m\": %d, \"n\": %d, "
                   "\"a_sf_id\": %d, \"b_sf_id\": %d, \"value\": \"0x%08x\"}", a, b, m, n, a_sf, b_sf, (unsigned)d);
    };
    using cute::UMMA::Major;
    using UE8 = cutlass::float_ue8m0_t;
    using E4 = cutlass::float_e4m3_t;
    using E5 = cutlass::float_e5m2_t;
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<E4, E4, float, UE8, 128, 256, Major::K, Major::K>()), "e4m3", "e4m3", 128, 256, 0, 0);
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<E4, E4, float, UE8, 128, 128, Major::K, Major::K>()), "e4m3", "e4m3", 128, 128, 0, 0);
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<E5, E4, float, UE8, 128, 256, Major::K, Major::K>()), "e5m2", "e4m3", 128, 256, 0, 0);
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<E5, E5, float, UE8, 256, 256, Major::K, Major::K>()), "e5m2", "e5m2", 256, 256, 0, 0);
    using E2 = cutlass::float_e2m1_t;  // packed e2m1 (kind::mxf4 / mxf4nvf4)
    using UE4 = cutlass::float_ue4m3_t;
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<E2, E2, float, UE8, 128, 256, Major::K, Major::K>()), "e2m1", "e2m1", 128, 256, 0, 0);
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<E2, E2, float, UE8, 256, 256, Major::K, Major::K>()), "e2m1", "e2m1", 256, 256, 0, 0);
    {
      const uint64_t r = cute::UMMA::make_runtime_instr_desc_block_scaled<E2, E2, float, UE8, 256, 256, Major::K, Major::K>(
          2u << 30, 2u << 30);
      bs(uint32_t(r >> 32), "e2m1", "e2m1", 256, 256, 2, 2);
    }
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<E2, E2, float, UE4, 128, 256, Major::K, Major::K>()), "e2m1/ue4m3", "e2m1/ue4m3", 128, 256, 0, 0);
    // fp6 through kind::mxf8f6f4 (CuTe's shared-memory element types for TMA-unpacked fp6).
    using F6a = cutlass::detail::float_e3m2_unpacksmem_t;
    using F6b = cutlass::detail::float_e2m3_unpacksmem_t;
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<F6a, F6a, float, UE8, 128, 256, Major::K, Major::K>()), "e3m2", "e3m2", 128, 256, 0, 0);
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<F6b, F6b, float, UE8, 256, 256, Major::K, Major::K>()), "e2m3", "e2m3", 256, 256, 0, 0);
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<F6b, F6a, float, UE8, 256, 192, Major::K, Major::K>()), "e2m3", "e3m2", 256, 192, 0, 0);
    bs(uint32_t(cute::UMMA::make_instr_desc_block_scaled<E4, F6a, float, UE8, 128, 128, Major::K, Major::K>()), "e4m3", "e3m2", 128, 128, 0, 0);
    {
      const uint64_t r = cute::UMMA::make_runtime_instr_desc_block_scaled<F6a, F6a, float, UE8, 256, 256, Major::K, Major::K>(
          3u << 30, 1u << 30);
      bs(uint32_t(r >> 32), "e3m2", "e3m2", 256, 256, 3, 1);
    }
    for (int a_sf = 0; a_sf < 4; ++a_sf)
      for (int b_sf = 0; b_sf < 4; ++b_sf) {
        const uint64_t r = cute::UMMA::make_runtime_instr_desc_block_scaled<E4, E4, float, UE8, 128, 256, Major::K, Major::K>(
            uint32_t(a_sf) << 30 | 0x100u, uint32_t(b_sf) << 30 | 0x108u);
        bs(uint32_t(r >> 32), "e4m3", "e4m3", 128, 256, a_sf, b_sf);
      }
  }
  std::fprintf(out, "\n]\n");
  std::fclose(out);
  return 0;
}
