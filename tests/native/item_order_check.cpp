// Host-side check of item_coords (attn_common.cuh), the work-item order of the persistent
// tensor-core kernel, on random shapes: every (unit, key split, query block) is produced by
// exactly one item index; in heavy-first order the units form n_groups consecutive groups whose
// sizes differ by at most one, and inside a group the query blocks never get heavier (later
// query blocks of a causal mask first).  Built and run by tests/test_mask_arith_cpu.py; exit
// status 0 = no violation.
#include <cstdio>
#include <random>
#include <vector>

#include "attn_common.cuh"

using namespace mlxp;

int main(int argc, char** argv) {
  const int trials = argc > 1 ? atoi(argv[1]) : 2000;
  std::mt19937_64 g(777);
  long long bad = 0;
  auto report = [&](const char* what, int trial) {
    if (bad++ < 10) printf("violation: %s (trial %d)\n", what, trial);
  };
  for (int trial = 0; trial < trials; ++trial) {
    FwdParams p{};
    p.B = 1 + (int)(g() % 6);
    p.H = 1 + (int)(g() % 40);
    p.n_qblk = 1 + (int)(g() % 20);
    p.splits = (g() % 3 == 0) ? 1 + (int)(g() % 4) : 1;
    p.heavy_first = (int)(g() % 2);
    const int BH = p.B * p.H;
    p.n_groups = 1 + (int)(g() % BH);
    const int n = p.n_qblk * BH * p.splits;
    std::vector<int> seen((size_t)n, 0);
    int prev_qb = 1 << 30, cur_group = -1;
    for (int idx = 0; idx < n; ++idx) {
      int bh, split, qb;
      item_coords(p, idx, bh, split, qb);
      if (bh < 0 || bh >= BH || split < 0 || split >= p.splits || qb < 0 || qb >= p.n_qblk) {
        report("coordinates out of range", trial);
        continue;
      }
      seen[((size_t)bh * p.splits + split) * p.n_qblk + qb]++;
      if (p.heavy_first) {
        // units of one group are a contiguous range; items of a group are contiguous
        const int base = BH / p.n_groups, n_big = BH % p.n_groups;
        const int grp = bh < n_big * (base + 1) ? bh / (base + 1)
                                                : n_big + (bh - n_big * (base + 1)) / base;
        if (grp != cur_group) {
          if (grp != cur_group + 1) report("groups out of order", trial);
          cur_group = grp;
          prev_qb = 1 << 30;
        }
        if (qb > prev_qb) report("a lighter query block before a heavier one", trial);
        prev_qb = qb;
      }
    }
    for (int c : seen)
      if (c != 1) {
        report("an item produced other than once", trial);
        break;
      }
  }
  printf("%lld violations\n", bad);
  return bad ? 1 : 0;
}
