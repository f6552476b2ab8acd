// Compile-time and host checks of the header-only kl API (<kl/kl.hpp>), restating the reference's
// kernel_lib/tests/unit/test_smem_tile.cu and the host parts of test_umma_desc.cu. Built and run
// by tests/test_headers.py; every static_assert is a test, and main() returns the failure count.
#include <cstddef>
#include <cstdio>
#include <vector>

#include <kl/kl.hpp>

// test_smem_tile.cu:28-45 (SizesAndAlignment)
using A = kl::SmemTile<kl::bf16, 128, 64>;
static_assert(A::bytes == 128 * 64 * 2);
static_assert(A::alignment == 1024);
static_assert(sizeof(A) == A::bytes);
static_assert(alignof(A) == 1024);
static_assert(A::atom_elems == 64);
static_assert(A::layout_type::size() == 128 * 64 && A::layout_type::cosize() == 128 * 64);
using W = kl::SmemTile<int8_t, 128, 128>;
static_assert(W::atom_elems == 128 && W::bytes == 128 * 128);
using C = kl::SmemTile<kl::bf16, 128, 32, kl::Swizzle64B>;
static_assert(C::alignment == 512 && C::atom_elems == 32);

// test_smem_tile.cu:60-67 (StructOfTilesKeepsAlignment)
struct Stage {
  kl::SmemTile<kl::bf16, 128, 64> a;
  kl::SmemTile<kl::bf16, 256, 64> b;
};
static_assert(offsetof(Stage, b) % 1024 == 0);
static_assert(sizeof(Stage) == 128 * 64 * 2 + 256 * 64 * 2);

// test_smem_tile.cu:69-90 (TmaBox)
static_assert(kl::TmaBox<A>::inner == 64 && kl::TmaBox<A>::outer == 128 && kl::TmaBox<A>::count == 1);
static_assert(kl::TmaBox<A>::bytes == A::bytes);
using X = kl::SmemTile<kl::bf16, 128, 128>;
static_assert(kl::TmaBox<X>::inner == 64 && kl::TmaBox<X>::count == 2);
static_assert(kl::TmaBox<X>::smem_offset(0) == 0u && kl::TmaBox<X>::smem_offset(1) == 128u * 64 * 2);
using T512 = kl::TmaBox<kl::SmemTile<kl::bf16, 512, 128>>;
static_assert(T512::outer == 256 && T512::row_boxes == 2 && T512::col_boxes == 2 && T512::count == 4);
static_assert(T512::row(1) == 256 && T512::col(2) == 64 && T512::smem_offset(3) == 98304u);

// test_umma_desc.cu:78-94 (InstrDesc known answer), built by hand from the field layout.
constexpr uint32_t expected = (1u << 4) | (1u << 7) | (1u << 10) | (32u << 17) | (8u << 24);
static_assert(expected == 0x08400490u);
static_assert(kl::mma_instr_desc<kl::bf16, kl::bf16, float, 128, 256>() == expected);
// The CTA-pair shape (M = 256) the reference's encoder rejects.
static_assert(kl::mma_instr_desc<kl::bf16, kl::bf16, float, 256, 256>() == 0x10400490u);
static_assert(kl::mma_instr_desc<kl::e4m3, kl::e4m3, float, 128, 256>() == 0x08400010u);

// test_umma_desc.cu:96-114 (known fields, bf16 128x64 SW128) at a base of 0x400.
constexpr kl::SmemDesc d0 = kl::umma_desc_at<A>(0x400, 0);
static_assert(kl::mma_k<kl::bf16> == 16 && kl::num_k_blocks<A> == 4);
static_assert(kl::block_offset_16B<A>(1) == 2 && kl::block_offset_16B<A>(3) == 6);
static_assert(kl::block_offset_16B<X>(4) == 1024);

// Swizzle: the 16-byte chunk index XOR the row within the 8-row pattern.
static_assert(kl::swizzle_bytes<kl::Swizzle128B>(1 * 128 + 0 * 16) == 1 * 128 + 1 * 16);
static_assert(kl::swizzle_bytes<kl::Swizzle128B>(7 * 128 + 5 * 16) == 7 * 128 + 2 * 16);

static_assert(kl::SmemTileType<A> && !kl::SmemTileType<int>);

int main() {
  int failures = 0;
  auto expect = [&](bool ok, const char* what) {
    if (!ok) {
      std::printf("FAIL %s\n", what);
      ++failures;
    }
  };
  // test_smem_tile.cu:51-58 (LayoutIsBijectionOntoStorage), swizzled and plain.
  {
    using B = kl::SmemTile<kl::bf16, 128, 128>;
    auto L = B::layout_type{};
    std::vector<int> hits(B::size, 0), hits_b(B::size, 0);
    for (int r = 0; r < B::rows; ++r)
      for (int c = 0; c < B::cols; ++c) {
        ++hits[L(r, c)];
        ++hits_b[L.layout_b()(r, c)];
      }
    bool ok = true;
    for (int i = 0; i < B::size; ++i) ok = ok && hits[i] == 1 && hits_b[i] == 1;
    expect(ok, "layout is a bijection onto storage");
  }
  // Descriptor fields through the union.
  {
    kl::SmemDesc d = d0;
    expect(d.layout_type_ == 2, "layout SWIZZLE_128B");
    expect(d.version_ == 1, "version 1");
    expect(d.stride_byte_offset_ == 64, "SBO 1024 B");
    expect(d.leading_byte_offset_ == 1, "LBO 1");
    expect(d.base_offset_ == 0, "base offset 0");
    expect(d.start_address_ == (0x400 >> 4), "start address");
    for (int k = 0; k < 4; ++k) {
      kl::SmemDesc dk = kl::umma_desc_at<A>(0x400, k);
      expect(dk.start_address_ == (0x400 >> 4) + 2 * k, "start advances 32 B per k-block");
    }
    using B512 = kl::SmemTile<kl::bf16, 512, 64>;
    kl::SmemDesc second = kl::umma_desc_at<B512>(0x400, 0, 256);
    expect(second.start_address_ == ((0x400 + 32 * 1024) >> 4) && second.base_offset_ == 0, "row block 256 at +32 KB");
  }
  // Row-major views.
  {
    static float buf[2 * 3 * 4];
    auto g = kl::row_major(buf, 2, 3, 4);
    expect(g.rank == 3 && g.shape[0] == 2 && g.stride[0] == 12 && g.stride[1] == 4 && g.stride[2] == 1, "row_major");
    auto s = kl::row_major_strided(buf, 3, 2, 8);
    expect(s.shape[0] == 3 && s.shape[1] == 2 && s.stride[0] == 8 && s.stride[1] == 1, "row_major_strided");
  }
  // Tensor-map validation (no driver needed: every case fails before the driver call).
  {
    alignas(16) static kl::bf16 mem[64];
    auto throws = [](auto fn) {
      try {
        fn();
      } catch (std::invalid_argument const&) {
        return true;
      }
      return false;
    };
    expect(throws([&] { kl::make_tma_load<A>(kl::row_major(mem + 1, 4096, 4096)); }), "misaligned");
    expect(throws([&] { kl::make_tma_load<A>(kl::row_major_strided(mem, 4096, 4096, 1024)); }), "row_stride < cols");
    expect(throws([&] { kl::make_tma_load<A>(kl::row_major(mem, 4096, 4100)); }), "pitch % 16");
    expect(throws([&] { kl::make_tma_load<A>(kl::row_major(mem, 0, 4096)); }), "empty");
  }
  std::printf("%d failures\n", failures);
  return failures;
}
