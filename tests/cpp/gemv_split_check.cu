// Host check of the config-1 GEMV's split geometry (q4_gemv_tma.cuh: shape_ok, range_of,
// segs_of, tile_ctas, slots_bound; the functions the kernel and qora_q4_gemv use), for
// every shape the kernel takes among config 1's, SmolLM3-3B's other projections, their
// tensor-parallel shards and edge shapes, on several SM counts: every (tile, row) owned by
// exactly one CTA, ranges of whole boxes (at least one, at most kMaxBoxes, so they fit
// the shared memory), at most two segments per CTA, the CTAs of a tile consecutive with
// slots 0..n-1 as tile_ctas gives them, n within the host's slot allocation, and exactly
// one finisher (the last slot) per tile. Prints "ok" or the first failure.
#include <cstdio>
#include <vector>

#include "../../qora-llm_b200/csrc/q4_gemv_tma.cuh"

using namespace qora::g1;
using qora::kTileCols;

int main() {
  const long long ks[] = {64, 128, 1024, 1536, 2048, 2752, 4096, 5504, 11008, 16384};
  const long long ns[] = {256, 512, 1024, 1536, 2048, 3072, 4096, 5504, 11008, 22016, 128256};
  const int gs[] = {148, 132, 144, 16};
  int checked = 0;
  for (int G : gs)
    for (long long k : ks)
      for (long long n : ns) {
        if (!shape_ok(k, n, G)) continue;
        const int K = (int)k, tiles = (int)(n / kTileCols);
        const unsigned boxes = (unsigned)(tiles * (K / kBoxRows));
        const int slots = slots_bound(K, boxes, G);
        std::vector<int> cover((size_t)tiles * K, 0), next_slot(tiles, 0), finishers(tiles, 0);
        for (int c = 0; c < G; ++c) {
          int l0, l1;
          range_of(c, G, boxes, &l0, &l1);
          const Segs sg = segs_of(l0, l1, K);
          bool bad = l1 <= l0 || l0 % kBoxRows || l1 % kBoxRows || (l1 - l0) / kBoxRows > kMaxBoxes ||
                     l1 - l0 > kMaxRows || sg.n < 1 || sg.n > 2;
          int covered = 0;
          for (int s = 0; s < sg.n && !bad; ++s) {
            const int t = sg.t[s];
            int first, last;
            tile_ctas(t, K, G, boxes, &first, &last);
            const int slot = c - first, nsl = last - first + 1;
            bad |= slot != next_slot[t] || nsl > slots || c > last;
            ++next_slot[t];
            if (slot == nsl - 1) ++finishers[t];
            for (int r = sg.r0[s]; r < sg.r1[s]; ++r) ++cover[(size_t)t * K + r];
            covered += sg.r1[s] - sg.r0[s];
          }
          bad |= covered != l1 - l0;
          if (bad) {
            std::printf("FAIL G=%d k=%lld n=%lld cta %d range [%d, %d)\n", G, k, n, c, l0, l1);
            return 1;
          }
        }
        for (int t = 0; t < tiles; ++t) {
          int first, last;
          tile_ctas(t, K, G, boxes, &first, &last);
          if (next_slot[t] != last - first + 1 || finishers[t] != 1) {
            std::printf("FAIL G=%d k=%lld n=%lld tile %d: %d slots, %d finishers\n", G, k, n, t, next_slot[t],
                        finishers[t]);
            return 1;
          }
        }
        for (size_t p = 0; p < cover.size(); ++p)
          if (cover[p] != 1) {
            std::printf("FAIL G=%d k=%lld n=%lld row %zu covered %d times\n", G, k, n, p, cover[p]);
            return 1;
          }
        ++checked;
      }
  // config 1 must be among the shapes the kernel takes on a B200
  if (!shape_ok(2048, 11008, 148) || checked < 20) {
    std::printf("FAIL: config 1 not taken or too few shapes checked (%d)\n", checked);
    return 1;
  }
  std::printf("ok\n");
  return 0;
}
