// Host checks of the tile kernels' work schedule (kl::gemm::WorkSeq, tn_schedule, the stream-K
// contributor and slot bookkeeping the epilogue uses), over many (tiles, workers, K-blocks).
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

// What the epilogue computes for (worker w, tile t) in the stream-K region: the contributors and
// w's slot.
static void check_case(int tiles, int sk_tiles, int W, int KB) {
  const int dp = tiles - sk_tiles;
  const long long U = (long long)sk_tiles * KB;
  std::vector<std::vector<int>> cover(tiles, std::vector<int>(KB, 0));
  std::map<int, std::set<int>> contributors;  // tile -> workers with a piece of it
  std::set<long long> slots_used;
  for (int w = 0; w < W; ++w) {
    WorkSeq seq(w, W, tiles, sk_tiles, KB);
    TilePiece pc;
    int prev_t = -1;
    bool in_sk = false;
    std::set<long long> my_slots;
    while (seq.next(pc)) {
      CHECK(pc.t >= 0 && pc.t < tiles && pc.kb0 >= 0 && pc.kb0 < pc.kb1 && pc.kb1 <= KB, "t %d [%d,%d)", pc.t, pc.kb0, pc.kb1);
      if (!(pc.t >= 0 && pc.t < tiles)) return;
      CHECK(pc.t > prev_t, "pieces in tile order (w %d t %d after %d)", w, pc.t, prev_t);
      if (pc.t < dp) {
        CHECK(!in_sk && pc.t % W == w && pc.kb0 == 0 && pc.kb1 == KB, "data-parallel tile %d of w %d", pc.t, w);
      } else {
        in_sk = true;
        contributors[pc.t].insert(w);
      }
      for (int kb = pc.kb0; kb < pc.kb1; ++kb) ++cover[pc.t][kb];
      prev_t = pc.t;
    }
  }
  for (int t = 0; t < tiles; ++t)
    for (int kb = 0; kb < KB; ++kb) CHECK(cover[t][kb] == 1, "unit (%d, %d) covered %d times", t, kb, cover[t][kb]);
  for (auto& [t, ws] : contributors) {
    const long long tu0 = (long long)(t - dp) * KB;
    const int wf = sk_worker_of_unit(tu0, U, W), wl = sk_worker_of_unit(tu0 + KB - 1, U, W);
    CHECK(wf == *ws.begin() && wl == *ws.rbegin() && int(ws.size()) == wl - wf + 1,
          "tile %d: contributors [%d, %d] vs %d..%d", t, wf, wl, *ws.begin(), *ws.rbegin());
    if (wf == wl) continue;
    for (int w : ws) {  // the slot the epilogue's slot_of picks
      const int first_t = dp + int(sk_unit_start(w, U, W) / KB);
      const long long s = 2LL * w + (t == first_t ? 0 : 1);
      CHECK(slots_used.insert(s).second, "slot %lld used twice (tile %d, worker %d)", s, t, w);
    }
  }
}

template <int CG>
using Pair = TnConfig<kl::bf16, kl::bf16, CG, 256, CG == 2 ? 6 : 4>;

int main() {
  int cases = 0;
  for (int W : {1, 2, 3, 7, 74, 148})
    for (int tiles : {1, 2, 5, 73, 74, 75, 128, 147, 148, 149, 256, 300})
      for (int KB : {1, 2, 3, 16, 128}) {
        const int tail = tiles < 2 * W ? tiles : W + tiles % W;
        // tn_schedule's worker count for the split region: at least one unit per worker.
        const int wk = tail == tiles ? std::min(W, tail * KB) : W;
        check_case(tiles, 0, W, KB);
        check_case(tiles, tail, wk, KB);
        ++cases;
      }
  // Decisions on the N-sharded 8192^3 bf16 GEMM (CTA pair, 256 x 256 tiles, 74 pairs).
  Problem pr;
  pr.k = 8192;
  pr.m = 8192;
  for (auto [n, want] : std::vector<std::pair<int, int>>{{8192, 0}, {4096, 0}, {2048, 108}, {1024, 128}}) {
    pr.n = n;
    const TnSchedule s = tn_schedule<Pair<2>>(pr, 74);
    CHECK(s.sk_tiles == want, "n %d: sk_tiles %d, want %d", n, s.sk_tiles, want);
    CHECK(s.sk_tiles == 0 || (s.workers == 74 && s.ticket_bytes <= kTnStreamKTicketBytes &&
                              kTnStreamKTicketBytes + s.slot_bytes <= kTnStreamKWorkspaceBytes),
          "n %d: workspace", n);
  }
  pr.n = 1024;
  pr.stream_k = -1;
  CHECK(tn_schedule<Pair<2>>(pr, 74).sk_tiles == 0, "stream_k = -1 turns the tail off");
  pr.stream_k = 1;
  pr.n = 8192;
  CHECK(tn_schedule<Pair<2>>(pr, 74).sk_tiles == 74 + 1024 % 74, "stream_k = 1 splits the tail");
  pr.m = 256;
  pr.n = 512;
  CHECK(tn_schedule<Pair<2>>(pr, 74).sk_tiles == 2 && tn_schedule<Pair<2>>(pr, 74).workers == 74,
        "small problems split over every worker");
  pr.max_ctas = 6;
  CHECK(tn_schedule<Pair<2>>(pr, 74).workers == 3, "max_ctas caps the workers");
  pr.max_ctas = 0;
  pr.k = 128;  // 2 tiles x 2 K-blocks of 64: four units, so four workers
  CHECK(tn_schedule<Pair<2>>(pr, 74).workers == 4, "no more workers than units: %d", tn_schedule<Pair<2>>(pr, 74).workers);
  pr.k = 8192;
  pr.stream_k = 0;
  pr.max_ctas = 0;
  pr.m = 8192;
  pr.n = 1024;
  CHECK(tn_schedule<Pair<1>>(pr, 148).sk_tiles == 256, "one-CTA tiles: 256 on 148 workers (86 %%) all split");
  std::printf("%d cases, %d failures\n", cases, failures);
  return failures == 0 ? 0 : 1;
}
