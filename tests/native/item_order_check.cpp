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
  // With RoPE rotation items: every rotation item (group, chunk) and attention item (unit,
  // split, query block) exactly once, each in its unit's group, and every attention item after
  // the last rotation item of its group.
  for (int trial = 0; trial < trials; ++trial) {
    FwdParams p{};
    p.B = 1 + (int)(g() % 5);
    p.H = 1 + (int)(g() % 40);
    p.n_qblk = 1 + (int)(g() % 12);
    p.splits = (g() % 3 == 0) ? 1 + (int)(g() % 3) : 1;
    p.heavy_first = (int)(g() % 2);
    p.rope_items = 1 + (int)(g() % 20);
    const int BH = p.B * p.H;
    p.n_groups = 1 + (int)(g() % BH);
    const int base = BH / p.n_groups, n_big = BH % p.n_groups;
    auto group_of = [&](int bh) {
      return bh < n_big * (base + 1) ? bh / (base + 1) : n_big + (bh - n_big * (base + 1)) / base;
    };
    const int n_att = p.n_qblk * BH * p.splits, n_rot = p.n_groups * p.rope_items;
    std::vector<int> seen_a((size_t)n_att, 0), seen_r((size_t)n_rot, 0);
    std::vector<int> last_rot(p.n_groups, -1), first_att(p.n_groups, 1 << 30);
    for (int idx = 0; idx < n_att + n_rot; ++idx) {
      int bh, split, qb, rot, grp;
      item_coords_rope(p, idx, bh, split, qb, rot, grp);
      if (bh < 0 || bh >= BH || grp != group_of(bh)) {
        report("rope: unit out of range or in the wrong group", trial);
        continue;
      }
      if (rot >= 0) {
        if (rot >= p.rope_items) { report("rope: chunk out of range", trial); continue; }
        if (bh != (grp < n_big ? grp * (base + 1) : n_big * (base + 1) + (grp - n_big) * base))
          report("rope: rotation item not at its group's first unit", trial);
        seen_r[(size_t)grp * p.rope_items + rot]++;
        last_rot[grp] = idx > last_rot[grp] ? idx : last_rot[grp];
      } else {
        if (split < 0 || split >= p.splits || qb < 0 || qb >= p.n_qblk) {
          report("rope: attention coordinates out of range", trial);
          continue;
        }
        seen_a[((size_t)bh * p.splits + split) * p.n_qblk + qb]++;
        first_att[grp] = idx < first_att[grp] ? idx : first_att[grp];
      }
    }
    for (int c : seen_a) if (c != 1) { report("rope: attention item not produced once", trial); break; }
    for (int c : seen_r) if (c != 1) { report("rope: rotation item not produced once", trial); break; }
    for (int gi = 0; gi < p.n_groups; ++gi)
      if (first_att[gi] < last_rot[gi]) report("rope: attention before its group's rotation", trial);
  }
  printf("%lld violations\n", bad);
  return bad ? 1 : 0;
}
