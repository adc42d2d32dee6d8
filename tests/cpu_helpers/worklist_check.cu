// Test helper (host program, runs on the CPU): the GEMM kernels' work distribution, taken from the package's own
// header (reax::WorkList, reax::split_rr_tiles), checked over a sweep of problem sizes and two very long K.  Built and run by
// tests/test_gemm_schedule_cpu.py.
//
// For G work units (CTAs, or clusters of two for the pair kernels), `tiles` tiles of `nk` k-blocks each:
//   unsplit: every tile is run by exactly one unit, whole, units taking tiles c, c + G, ..;
//   split:   the raster tiles first, then a head piece, whole tiles, a tail piece; every (tile, k-block) is run
//            exactly once; a tile is cut at most once, the head piece [0, ke) by unit c and the tail [ke, nk) by unit
//            c + 1 (so a unit's tail always waits on its predecessor's head, which waits for nothing); every unit's
//            share holds at least one tile; and when two or more waves are split, a whole tile sits between a unit's
//            head and its tail (the restore of the partial overlaps that tile's MMAs).
// Prints "ok <cases>" and exits 0, or prints the first violation and exits 1.
#include <cstdio>
#include <vector>

#include "gemm_sm100.cuh"

static int fail(const char* what, int tiles, int nk, int G, int c) {
  std::printf("FAIL %s: tiles=%d nk=%d G=%d unit=%d\n", what, tiles, nk, G, c);
  return 1;
}

static int check(int tiles, int nk, int G, bool split) {
  using reax::WorkList;
  const int rr = split ? reax::split_rr_tiles(tiles, G) : tiles;
  if (split && (rr % G != 0 || tiles - rr < G || tiles - rr > 3 * G)) return fail("raster share", tiles, nk, G, -1);
  std::vector<unsigned char> cover((size_t)tiles * nk, 0);
  std::vector<int> head_tile(G, -1), head_end(G, -1), tail_tile(G, -1), tail_begin(G, -1);
  for (int c = 0; c < G; ++c) {
    WorkList w;
    if (split) w.init<true>(tiles, rr, nk, c, G);
    else w.init<false>(tiles, rr, nk, c, G);
    long long share = 0;
    int last_kind = -1, seen_head = -1, seen_tail = -1;
    for (int i = 0; i < w.count; ++i) {
      int t, kb0, kb1, kind;
      w.item(i, t, kb0, kb1, kind);
      if (t < 0 || t >= tiles || kb0 < 0 || kb1 > nk || kb0 >= kb1) return fail("item range", tiles, nk, G, c);
      if (i < w.n_rr && (kind != reax::WK_FULL || t != c + i * G)) return fail("raster item", tiles, nk, G, c);
      if (kind == reax::WK_HEAD) {
        if (kb0 != 0 || kb1 == nk || seen_tail >= 0 || seen_head >= 0) return fail("head piece", tiles, nk, G, c);
        seen_head = i;
        head_tile[c] = t;
        head_end[c] = kb1;
      } else if (kind == reax::WK_TAIL) {
        if (kb0 == 0 || kb1 != nk || i != w.count - 1) return fail("tail piece", tiles, nk, G, c);
        seen_tail = i;
        tail_tile[c] = t;
        tail_begin[c] = kb0;
      } else if (kb0 != 0 || kb1 != nk) {
        return fail("whole tile", tiles, nk, G, c);
      }
      if (last_kind == reax::WK_TAIL) return fail("item after the tail", tiles, nk, G, c);
      last_kind = kind;
      if (i >= w.n_rr) share += kb1 - kb0;
      for (int k = kb0; k < kb1; ++k) cover[(size_t)t * nk + k] += 1;
    }
    if (split) {
      if (share < nk) return fail("share below one tile", tiles, nk, G, c);
      if (seen_head >= 0 && seen_tail >= 0 && tiles - rr >= 2 * G && seen_tail - seen_head < 2)
        return fail("no whole tile between head and tail", tiles, nk, G, c);
    } else if (w.count != (tiles - c + G - 1) / G) {
      return fail("raster count", tiles, nk, G, c);
    }
  }
  for (size_t e = 0; e < cover.size(); ++e)
    if (cover[e] != 1) return fail("k-block covered not exactly once", tiles, nk, G, (int)(e / nk));
  if (split) {
    if (tail_tile[0] >= 0) return fail("first unit has a tail", tiles, nk, G, 0);
    if (head_tile[G - 1] >= 0) return fail("last unit has a head", tiles, nk, G, G - 1);
    for (int c = 0; c + 1 < G; ++c) {
      const bool h = head_tile[c] >= 0, t = tail_tile[c + 1] >= 0;
      if (h != t) return fail("head without the next unit's tail", tiles, nk, G, c);
      if (h && (head_tile[c] != tail_tile[c + 1] || head_end[c] != tail_begin[c + 1]))
        return fail("head and tail disagree", tiles, nk, G, c);
    }
  }
  return 0;
}

int main() {
  long long cases = 0;
  // work-unit counts: 148 and 132 SMs, their pairs (74, 66), a few others; k-blocks per tile as the bench and the
  // tests use them (1, 3, 16, 32, 63, 64) and a few more; tile counts up to four waves past the unit count
  const int units[] = {148, 74, 132, 66, 2, 3, 7, 64};
  const int nks[] = {1, 2, 3, 16, 32, 63, 64, 65, 128};
  for (int G : units)
    for (int nk : nks)
      for (int tiles = 1; tiles <= 4 * G + 3; ++tiles) {
        if (check(tiles, nk, G, false)) return 1;
        ++cases;
        if (tiles > G && tiles % G != 0) {  // the split kernels run only when the last wave is partial
          if (check(tiles, nk, G, true)) return 1;
          ++cases;
        }
      }
  // the shapes of BASELINE config 2 and its shards (128 x 256 tiles on 148 SMs, 256 x 256 pair tiles on 74 pairs)
  const int cfg2[][2] = {{1792, 148}, {896, 148}, {448, 148}, {224, 148}, {896, 74}, {448, 74}, {224, 74}, {112, 74}};
  for (auto& tg : cfg2) {
    if (check(tg[0], 64, tg[1], false)) return 1;
    if (tg[0] % tg[1] != 0 && check(tg[0], 64, tg[1], true)) return 1;
    cases += 2;
  }
  // long K: k-blocks of the split tiles x work units past 2^32 (the schedule's products must not wrap)
  const int big[][3] = {{3 * 148 - 1, 65536, 148}, {220, 300000, 74}};
  for (auto& b : big) {
    if (check(b[0], b[1], b[2], true)) return 1;
    ++cases;
  }
  std::printf("ok %lld\n", cases);
  return 0;
}
