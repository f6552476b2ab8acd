// Host checks of the tile kernels' work schedule (kl::gemm::WorkSeq and tn_schedule's split tail),
// over many (tiles, workers, K-blocks, K-ranges per tail tile).
// Prints "N failures"; exit status 0 when there are none.

#include <algorithm>
#include <cstdio>
#include <map>
#include <set>
#include <vector>

#include <kl/gemm/gemm.hpp>

using namespace kl::gemm;

static int failures = 0;
#define CHECK(c, ...)                      \
  do {                                     \
    if (!(c)) {                            \
      ++failures;                          \
      if (failures < 20) {                 \
        std::printf("FAIL %s: ", #c);      \
        std::printf(__VA_ARGS__);          \
        std::printf("\n");                \
      }                                    \
    }                                      \
  } while (0)

// The pieces every worker walks, against what the kernel relies on.
static void check_case(int tiles, int sk_tiles, int split, int W, int KB) {
  const int dp = tiles - sk_tiles;
  std::vector<std::vector<int>> cover(tiles, std::vector<int>(KB, 0));
  std::map<int, std::set<int>> ranges;  // tail tile -> its K-ranges seen
  for (int w = 0; w < W; ++w) {
    WorkSeq seq(w, W, tiles, sk_tiles, split, KB);
    TilePiece pc;
    bool in_whole = false;
    while (seq.next(pc)) {
      CHECK(pc.t >= 0 && pc.t < tiles && pc.kb0 >= 0 && pc.kb0 < pc.kb1 && pc.kb1 <= KB, "t %d [%d,%d)", pc.t, pc.kb0, pc.kb1);
      if (!(pc.t >= 0 && pc.t < tiles)) return;
      if (pc.t < dp) {
        in_whole = true;
        CHECK(pc.t % W == w && pc.kb0 == 0 && pc.kb1 == KB && pc.q == 0, "whole tile %d of w %d", pc.t, w);
      } else {
        CHECK(!in_whole, "tail piece of tile %d after a whole tile (w %d)", pc.t, w);
        CHECK(pc.q >= 0 && pc.q < split, "range %d of %d", pc.q, split);
        CHECK(ranges[pc.t].insert(pc.q).second, "tile %d range %d twice", pc.t, pc.q);
        if (split == 1) CHECK(pc.kb0 == 0 && pc.kb1 == KB, "unsplit tail tile %d", pc.t);
      }
      for (int kb = pc.kb0; kb < pc.kb1; ++kb) ++cover[pc.t][kb];
    }
  }
  for (int t = 0; t < tiles; ++t)
    for (int kb = 0; kb < KB; ++kb) CHECK(cover[t][kb] == 1, "unit (%d, %d) covered %d times", t, kb, cover[t][kb]);
  for (int t = dp; t < tiles; ++t) CHECK(int(ranges[t].size()) == split, "tail tile %d has %d ranges", t, int(ranges[t].size()));
}

template <int CG>
using Pair = TnConfig<kl::bf16, kl::bf16, CG, 256, CG == 2 ? 6 : 4>;
// 256 x 512 CTA-pair tiles (two N = 256 sub-tiles per stage of A).
using Wide = TnConfig<kl::bf16, kl::bf16, 2, 256, 4, false, false, false, kl::Swizzle128B, 0, 2>;
static_assert(Wide::kTileN == 512 && Wide::kCtaN == 128 && Wide::kAccCols == 512 && Wide::kNumAcc == 1 &&
                  Wide::kEpiWarps == 8 && !Wide::kEarlyRelease && Wide::kBBytes == 2 * Wide::kBSubBytes,
              "wide tile geometry");

int main() {
  int cases = 0;
  for (int W : {1, 2, 3, 7, 74, 148})
    for (int tiles : {1, 2, 5, 73, 74, 75, 128, 147, 148, 149, 256, 300})
      for (int KB : {1, 2, 3, 16, 128})
        for (int split : {1, 2, 3, 4}) {
          if (split > KB) continue;
          const int R = tiles % W == 0 ? W : tiles % W;
          const int workers = tiles > W ? W : std::min(W, R * split);
          check_case(tiles, 0, 1, W, KB);
          check_case(tiles, R, split, workers, KB);
          ++cases;
        }
  // Decisions on the N-sharded 8192^3 bf16 GEMM (CTA pair, 256 x 256 tiles, 74 pairs).
  Problem pr;
  pr.k = 8192;
  pr.m = 8192;
  struct Want { int n, tail, split; };
  for (Want c : {Want{8192, 0, 1}, Want{4096, 0, 1}, Want{2048, 34, 2}, Want{1024, 0, 1}}) {
    pr.n = c.n;
    const TnSchedule s = tn_schedule<Pair<2>>(pr, 74);
    CHECK(s.sk_tiles == c.tail && s.sk_split == c.split, "n %d: tail %d x %d, want %d x %d", c.n, s.sk_tiles, s.sk_split,
          c.tail, c.split);
    CHECK(s.sk_tiles == 0 || (s.workers == 74 && s.ticket_bytes <= kTnStreamKTicketBytes &&
                              kTnStreamKTicketBytes + s.slot_bytes <= kTnStreamKWorkspaceBytes),
          "n %d: workspace", c.n);
  }
  pr.n = 2048;
  pr.stream_k = -1;
  CHECK(tn_schedule<Pair<2>>(pr, 74).sk_tiles == 0, "stream_k = -1 turns the tail off");
  pr.n = 1024;
  pr.stream_k = 1;
  CHECK(tn_schedule<Pair<2>>(pr, 74).sk_tiles == 54 && tn_schedule<Pair<2>>(pr, 74).sk_split == 2,
        "forced: the 54-tile tail in two ranges (no s pays, so the smallest)");
  pr.stream_k = 1;
  pr.n = 8192;
  CHECK(tn_schedule<Pair<2>>(pr, 74).sk_tiles == 1024 % 74 && tn_schedule<Pair<2>>(pr, 74).sk_split >= 2,
        "stream_k = 1 splits the tail");
  pr.m = 256;
  pr.n = 512;
  CHECK(tn_schedule<Pair<2>>(pr, 74).sk_tiles == 2 && tn_schedule<Pair<2>>(pr, 74).sk_split == 4 &&
            tn_schedule<Pair<2>>(pr, 74).workers == 8,
        "two tiles on many workers: four ranges each, eight workers");
  pr.max_ctas = 6;
  CHECK(tn_schedule<Pair<2>>(pr, 74).workers == 3, "max_ctas caps the workers");
  pr.max_ctas = 0;
  pr.k = 128;  // two K-blocks of 64: at most two ranges
  CHECK(tn_schedule<Pair<2>>(pr, 74).sk_split == 2, "no more ranges than K-blocks: %d", tn_schedule<Pair<2>>(pr, 74).sk_split);
  pr.k = 64;
  CHECK(tn_schedule<Pair<2>>(pr, 74).sk_tiles == 0, "one K-block: nothing to split");
  pr.k = 8192;
  pr.stream_k = 0;
  pr.m = 8192;
  pr.n = 1024;
  CHECK(tn_schedule<Pair<1>>(pr, 148).sk_tiles == 0, "one-CTA tiles: 256 on 148 workers, the four ranges cost more");
  pr.n = 2048;
  CHECK(tn_schedule<Pair<1>>(pr, 148).sk_tiles == 68 && tn_schedule<Pair<1>>(pr, 148).sk_split == 2,
        "one-CTA tiles: 512 on 148 workers, the 68 of the last wave in two ranges");
  // Wide tiles: whole tiles only, and the tile counts behind the default choice.
  pr.stream_k = 0;
  pr.m = 8192;
  for (int n : {8192, 4096, 2048, 1024}) {
    pr.n = n;
    const TnSchedule w = tn_schedule<Wide>(pr, 74);
    CHECK(w.tiles == 32 * (n / 512) && w.sk_tiles == 0 && w.workers == std::min(74, w.tiles), "wide n %d: %d tiles",
          n, w.tiles);
  }
  pr.stream_k = 1;
  CHECK(tn_schedule<Wide>(pr, 74).sk_tiles == 0, "wide tiles never split, even when asked");
  std::printf("%d cases, %d failures\n", cases, failures);
  return failures == 0 ? 0 : 1;
}
