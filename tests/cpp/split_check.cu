// Host check of the persistent step's tile-aligned down_proj split (al_first / al_tile /
// al_span in megakernel.cuh, the same functions the kernel and the engine's buffer sizing
// use): every (tile, row) is owned by exactly one CTA, no CTA's span crosses a tile, the
// CTAs of a tile are consecutive with slots 0..n-1, n never exceeds ceil(g / tiles), and
// no CTA holds more rows than the shared input buffer. Prints "ok" or the first failure.
#include <cstdio>
#include <vector>

#include "../../qora-llm_b200/csrc/megakernel.cuh"

using namespace qora::mk;

int main() {
  struct Case {
    int g, T, K;
  };
  // SmolLM3-3B down_proj (8 tiles of 256 columns, 11,008 rows) on 148 SMs, its
  // tensor-parallel row splits, the test models' shapes, other SM counts and edge shapes
  const Case cases[] = {{148, 8, 11008}, {148, 8, 5504}, {148, 8, 2752}, {148, 8, 1376}, {148, 4, 1536},
                        {148, 8, 1536},  {132, 8, 11008}, {144, 8, 11008}, {16, 8, 100},  {148, 148, 64},
                        {17, 16, 33},    {148, 1, 11008}, {8, 8, 8}};
  for (const Case& cs : cases) {
    Args a{};
    a.subn[DOWN] = cs.g;
    a.tiles[DOWN] = cs.T;
    a.K[DOWN] = cs.K;
    std::vector<int> cover((size_t)cs.T * cs.K, 0), next_slot(cs.T, 0);
    const int nmax = (cs.g + cs.T - 1) / cs.T;
    for (int lc = 0; lc < cs.g; ++lc) {
      int out[3];
      al_span(a, DOWN, lc, out);
      const int l0 = out[0], n = out[1], f0 = out[2], t = l0 / cs.K;
      bool bad = n <= 0 || (l0 + n - 1) / cs.K != t || f0 != al_first(t, cs.g, cs.T) || lc - f0 != next_slot[t] ||
                 al_tile(lc, cs.g, cs.T) != t || n > kXsCap;
      const int nt = al_first(t + 1, cs.g, cs.T) - al_first(t, cs.g, cs.T);
      bad |= nt < 1 || nt > nmax;
      if (bad) {
        std::printf("FAIL g=%d T=%d K=%d lc=%d span=(%d,%d) first=%d\n", cs.g, cs.T, cs.K, lc, l0, n, f0);
        return 1;
      }
      ++next_slot[t];
      for (int p = l0; p < l0 + n; ++p) ++cover[p];
    }
    for (int t = 0; t < cs.T; ++t)
      if (next_slot[t] != al_first(t + 1, cs.g, cs.T) - al_first(t, cs.g, cs.T)) {
        std::printf("FAIL g=%d T=%d K=%d tile %d slots %d\n", cs.g, cs.T, cs.K, t, next_slot[t]);
        return 1;
      }
    for (size_t p = 0; p < cover.size(); ++p)
      if (cover[p] != 1) {
        std::printf("FAIL g=%d T=%d K=%d row %zu covered %d times\n", cs.g, cs.T, cs.K, p, cover[p]);
        return 1;
      }
  }
  std::printf("ok\n");
  return 0;
}
