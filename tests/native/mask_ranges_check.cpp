// Host-side check of the mask arithmetic in attn_common.cuh against the element-wise
// definition (causal kpos <= qpos, qpos - kpos <= wl, kpos - qpos <= wr, key < Skv) on random
// masks: kv_tile_range, tile_is_full, full_tile_range and row_col_interval.
// Built and run by tests/test_mask_arith_cpu.py; exit status 0 = no mismatch.
#include <cstdio>
#include <random>

#include "attn_common.cuh"

using namespace mlxp;

static bool admissible(const MaskSpec& m, long long i, long long j) {
  if (j < 0 || j >= m.Skv) return false;
  const long long qp = i + m.q_off, kp = j + m.kv_off;
  if (m.causal && kp > qp) return false;
  if (m.wl >= 0 && qp - kp > m.wl) return false;
  if (m.wr >= 0 && kp - qp > m.wr) return false;
  return true;
}

int main(int argc, char** argv) {
  const int trials = argc > 1 ? atoi(argv[1]) : 3000;
  std::mt19937_64 g(12345);
  long long bad = 0;
  auto report = [&](const char* what, int trial) {
    if (bad++ < 10) printf("mismatch in %s (trial %d)\n", what, trial);
  };
  for (int trial = 0; trial < trials; ++trial) {
    MaskSpec m;
    m.causal = (int)(g() % 2);
    m.wl = (g() % 3 == 0) ? -1 : (long long)(g() % 400);
    m.wr = (g() % 3 == 0) ? -1 : (long long)(g() % 400);
    m.Skv = 1 + (long long)(g() % 700);
    m.q_off = (long long)(g() % 1200) - 600;
    m.kv_off = (long long)(g() % 1200) - 600;
    const int BN = (g() % 2) ? 128 : 64;
    const long long r0 = (long long)(g() % 600), r1 = r0 + 1 + (long long)(g() % 128);
    // per-row admissible interval and the tile-level summaries
    bool any = false, tile_any[64] = {false}, tile_all[64];
    const int ntile = (int)((m.Skv + BN - 1) / BN);
    for (int t = 0; t < 64; ++t) tile_all[t] = true;
    for (long long i = r0; i < r1; ++i) {
      for (int t = 0; t < ntile; ++t) {
        const long long c0 = (long long)t * BN;
        int c_lo, c_hi;
        row_col_interval(m, i, c0, BN, c_lo, c_hi);
        for (int c = 0; c < BN; ++c) {
          const bool a = admissible(m, i, c0 + c);
          if (a != (c >= c_lo && c <= c_hi)) report("row_col_interval", trial);
          any |= a;
          tile_any[t] |= a;
          tile_all[t] &= a;
        }
      }
    }
    int tlo, thi;
    kv_tile_range(m, r0, r1, BN, tlo, thi);
    for (int t = 0; t < ntile; ++t) {
      if (tile_any[t] && (t < tlo || t >= thi)) report("kv_tile_range (admissible tile left out)", trial);
      if (tile_is_full(m, r0, r1, (long long)t * BN, (long long)t * BN + BN) != tile_all[t])
        report("tile_is_full", trial);
    }
    if (!any && thi > tlo) {
      // an empty range is allowed to be reported as a (fully masked) range only if it is empty
      report("kv_tile_range (non-empty for a fully masked block)", trial);
    }
    int flo, fhi;
    full_tile_range(m, r0, r1, BN, flo, fhi);
    for (int t = -2; t < ntile + 2; ++t) {
      const bool want = t >= 0 && t < ntile && tile_all[t];
      if (want != (t >= flo && t < fhi)) report("full_tile_range", trial);
    }
  }
  printf("%d random masks checked, %lld mismatches\n", trials, bad);
  return bad != 0;
}
