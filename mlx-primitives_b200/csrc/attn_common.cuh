// attn_common.cuh — parameters and mask arithmetic shared by the attention kernels.
//
// Masking semantics (positions are absolute: qpos = i + q_off, kpos = j + kv_off):
//   causal        kpos <= qpos                       (flash.py:286 kv_limit = q_end;
//                                                     _online_softmax.py:149-161)
//   window_left   qpos - kpos <= wl  (wl >= 0)       (sliding_window.py:154-160, |i-j| <= W)
//   window_right  kpos - qpos <= wr  (wr >= 0)
//   key index j < Skv (rows past the end of K/V are zero-filled by TMA and must be masked).
// For one query row the admissible keys of a tile form one contiguous interval, so masking a
// boundary tile costs two compares per score and no tile is ever masked element-wise unless it
// straddles a boundary.
#pragma once

#include <cstdint>

#ifndef __CUDACC__  // plain C++ (host-side checks of the mask arithmetic)
#define __host__
#define __device__
#endif

namespace mlxp {

struct MaskSpec {
  int causal;
  long long wl, wr;     // -1 = unbounded
  long long q_off, kv_off;
  long long Skv;
};

// Admissible key-index range [lo, hi) for the query rows [r0, r1) (local indices, r1 > r0).
__host__ __device__ inline void kv_index_range(const MaskSpec& m, long long r0, long long r1,
                                               long long& lo, long long& hi) {
  const long long qmin = r0 + m.q_off, qmax = r1 - 1 + m.q_off;
  lo = 0;
  hi = m.Skv;
  if (m.wl >= 0) {
    const long long l = qmin - m.wl - m.kv_off;
    if (l > lo) lo = l;
  }
  bool bounded = false;
  long long up = 0;
  if (m.causal) {
    up = qmax;
    bounded = true;
  }
  if (m.wr >= 0) {
    const long long u = qmax + m.wr;
    up = bounded ? (u < up ? u : up) : u;
    bounded = true;
  }
  if (bounded) {
    const long long h = up - m.kv_off + 1;
    if (h < hi) hi = h;
  }
  if (hi < lo) hi = lo;
}

// Key-tile range [tlo, thi) of width BN for the query rows [r0, r1); empty when r1 <= r0.
__host__ __device__ inline void kv_tile_range(const MaskSpec& m, long long r0, long long r1,
                                              int BN, int& tlo, int& thi) {
  if (r1 <= r0) {
    tlo = thi = 0;
    return;
  }
  long long lo, hi;
  kv_index_range(m, r0, r1, lo, hi);
  if (hi <= lo) {
    tlo = thi = 0;
    return;
  }
  tlo = (int)(lo / BN);
  thi = (int)((hi + BN - 1) / BN);
}

// True when every (query row in [r0, r1), key in [c0, c1)) is admissible and c1 <= Skv.
__host__ __device__ inline bool tile_is_full(const MaskSpec& m, long long r0, long long r1,
                                             long long c0, long long c1) {
  if (c1 > m.Skv) return false;
  const long long qmin = r0 + m.q_off, qmax = r1 - 1 + m.q_off;
  const long long kmin = c0 + m.kv_off, kmax = c1 - 1 + m.kv_off;
  if (m.causal && kmax > qmin) return false;
  if (m.wl >= 0 && qmax - kmin > m.wl) return false;
  if (m.wr >= 0 && kmax - qmin > m.wr) return false;
  return true;
}

// floor(a / b) and ceil(a / b) for b > 0 and any sign of a.
__host__ __device__ inline long long floor_div(long long a, long long b) {
  return a >= 0 ? a / b : -((-a + b - 1) / b);
}
__host__ __device__ inline long long ceil_div(long long a, long long b) { return -floor_div(-a, b); }

// The key tiles j (width BN) with tile_is_full(m, r0, r1, j*BN, j*BN + BN) form one contiguous
// range [flo, fhi) (empty: flo == fhi): the interior of the causal/window band, cut at Skv.
// Computed once per query tile so the per-key-tile test is two integer compares.
__host__ __device__ inline void full_tile_range(const MaskSpec& m, long long r0, long long r1,
                                                int BN, int& flo, int& fhi) {
  const long long qmin = r0 + m.q_off, qmax = r1 - 1 + m.q_off;
  long long lo = 0, hi = m.Skv / BN;
  if (m.causal) {  // (j+1)*BN - 1 + kv_off <= qmin
    const long long h = floor_div(qmin - m.kv_off + 1, BN);
    if (h < hi) hi = h;
  }
  if (m.wr >= 0) {  // (j+1)*BN - 1 + kv_off - qmin <= wr
    const long long h = floor_div(qmin + m.wr - m.kv_off + 1, BN);
    if (h < hi) hi = h;
  }
  if (m.wl >= 0) {  // qmax - (j*BN + kv_off) <= wl
    const long long l = ceil_div(qmax - m.wl - m.kv_off, BN);
    if (l > lo) lo = l;
  }
  if (hi < lo) hi = lo;
  flo = (int)lo;
  fhi = (int)hi;
}

// Admissible columns [c_lo, c_hi] (inclusive, tile-local, clamped to [-1, BN]) of the tile
// starting at key index c0 for the query at local row `row`.
__host__ __device__ inline void row_col_interval(const MaskSpec& m, long long row, long long c0,
                                                 int BN, int& c_lo, int& c_hi) {
  const long long base = row + m.q_off - (c0 + m.kv_off);  // qpos - kpos of column 0
  long long lo = 0, hi = BN - 1;
  if (m.Skv - 1 - c0 < hi) hi = m.Skv - 1 - c0;
  if (m.causal && base < hi) hi = base;
  if (m.wr >= 0 && base + m.wr < hi) hi = base + m.wr;
  if (m.wl >= 0 && base - m.wl > lo) lo = base - m.wl;
  if (lo > BN) lo = BN;
  if (hi < -1) hi = -1;
  c_lo = (int)lo;
  c_hi = (int)hi;
}

// Parameters of the tensor-core (bf16/fp16) kernel.  Q/K/V are described by TMA tensor maps;
// the slot fields give, for each of q, k and v, the tensor-map dimension (1..3) that holds
// seq, head and batch, and whether head/batch are broadcast (stride 0 -> coordinate 0).
struct TmaCoordMap {
  int8_t slot_s, slot_h, slot_b;  // tensor-map dims 1..3
  int8_t bcast_h, bcast_b;        // 1 = that dim was size-1/broadcast: always coordinate 0
};

struct FwdParams {
  int B, H, Sq, Skv;
  int n_qblk;           // query blocks of 256 rows
  int splits;           // >= 1 key-range splits
  int tiles_per_split;  // key tiles per split (splits > 1)
  int heavy_first;      // order query blocks by descending work (causal)
  int n_groups;         // scheduling groups of (batch, head) units, sizes differing by at
                        // most one unit (see decode_item)
  int kv_group;         // query heads per K/V head (grouped / multi-query attention; 1 = MHA)
  // Output, written through the O tensor map: normal (dtype, normalised) or fp32 (normalised,
  // for callers that merge partial results themselves; no key splits then).
  int out_f32;
  float* lse;                           // [B][H][Sq] contiguous, nullable unless out_f32
  // Accumulate (with out_f32): O and lse hold a running fp32 result (normalised O, natural-log
  // LSE) of earlier key ranges; the kernel merges its own into them (LSE weights) and writes
  // them back.  acc_o is the same fp32 tensor the O tensor map writes, read with these element
  // strides.  A row whose accumulated LSE is -inf takes the new result alone (its O is not
  // read; if the new result is empty too, the row is written as O = 0, LSE = -inf).
  int accumulate;
  const float* acc_o;
  long long acc_sb, acc_sh, acc_ss;
  // RoPE in the same launch (rope_items > 0): besides its attention items every scheduling
  // group has rope_items rotation items — chunks of kRopeRows positions of Q (the first
  // rope_q_items) and of K, each over every (batch, head) unit of the group, so that a thread
  // loads the cos/sin of its positions once for all the group's heads — which rotate the rows
  // (the half-split rotation of the RoPE kernel, rounded once to the element type) into
  // contiguous BHSD copies that the Q and K tensor maps read.  They run as a first phase of
  // the kernel, by all threads of every CTA, before the warp roles split; the TMA producer
  // waits for rot_done[g] == rope_items before loading a group-g item's Q and K.
  int rope_items, rope_q_items;
  const void* rq_src;
  const void* rk_src;
  long long rq_s[3], rk_s[3];   // element strides (batch, head, seq) of the unrotated q and k
  void* rq_dst;
  void* rk_dst;                 // rotated copies: [B][H][Sq][D], [B][H][Skv][D]
  const float* rope_cos;
  const float* rope_sin;        // fp32 [n_pos][D/2]
  long long rope_q_pos, rope_k_pos;  // position of row 0 of q and of k
  unsigned* rot_done;           // per scheduling group, zero at launch
  unsigned* rot_counter;        // next rotation item of the RoPE phase, zero at launch
  // Additive score bias (the custom mask of gqa_attention / mqa_attention), fp32, element
  // strides (batch, head, query row) — 0 for broadcast dims — and unit stride along keys:
  // scores become scale * q.k + bias[b][h][i][j] before the softmax.  Only the kernel
  // instantiation built for it reads this.
  const float* bias;
  long long bias_sb, bias_sh, bias_sq;
  float inv_scale;              // 1 / scale: the bias is added in units of the raw q.k
  // Key splits (splits > 1) are merged inside the kernel.  The query tiles (128 rows) that
  // more than one split touches get a partial per split: the normalised fp32 O of the split
  // at part_o + slot * 128 * D, laid out [D/4][128 rows][4] so that the 32 rows of a warp
  // store and load 512 contiguous bytes, and its natural-log LSE at part_lse + slot * 128,
  // slot = ((unit * n_qtile) + query tile) * splits + split.  Each split adds one to the query
  // tile's counter (tile_cnt[unit * n_qtile + query tile], zero at launch) after its partial is
  // visible, and the split that completes the count merges every partial and writes O.
  float* part_o;
  float* part_lse;
  unsigned* tile_cnt;
  long long part_tiles; // query tiles the workspace has room for (checked before every use)
  int n_qtile;          // query tiles of 128 rows per unit
  float scale_log2;     // softmax scale * log2(e)
  MaskSpec mask;
  TmaCoordMap cq, ck, cv, co;
  int* status;
  unsigned long long timeout_ns;
  // Persistent scheduling: [next item, CTAs finished].  Zero at launch; the last CTA to finish
  // resets both, so consecutive launches on one stream can reuse the pair.
  unsigned* work_counter;
};

// Parameters of the CUDA-core fp32 kernel (plain pointers and strides).
struct FwdParamsF32 {
  int B, H, Sq, Skv;
  int kv_group;  // query heads per K/V head (1 = MHA)
  const float* q;
  const float* k;
  const float* v;
  long long q_sb, q_sh, q_ss, k_sb, k_sh, k_ss, v_sb, v_sh, v_ss;
  float* o;
  long long o_sb, o_sh, o_ss;
  float* lse;  // [B][H][Sq] contiguous, nullable
  float scale_log2;
  MaskSpec mask;
  // Key splits: CTA (query block, split) covers its share of the block's key tiles and writes
  // a normalised partial at o + split * o_split, lse + split * lse_split, then adds one to its
  // query block's counter (blk_cnt[query block], zero at launch); the split that completes the
  // count merges the block's partials (LSE weights) into o_final / lse_final (nullable) and
  // resets the counter.
  int splits;
  long long o_split, lse_split;
  unsigned* blk_cnt;
  float* o_final;
  long long of_sb, of_sh, of_ss;
  float* lse_final;
  // additive score bias (nullable), as FwdParams::bias
  const float* bias;
  long long bias_sb, bias_sh, bias_sq;
};

// Work-item order of the persistent tensor-core kernel: item index idx in [0, n_qblk * B * H *
// splits) -> (batch, head) unit bh, key split and query block qb.
//   heavy_first (causal): the units are cut into n_groups consecutive groups whose sizes differ
//   by at most one unit (the first BH % n_groups groups take one more); inside a group the
//   query blocks go heaviest first across the whole group (longest-processing-time order),
//   then the next group — a group's K/V stays L2-resident while its items run, and the last
//   items of the launch are the lightest ones, which keeps the tail short.  Equal groups
//   matter: a small last group would start its heaviest items only once the previous group had
//   been handed out, and they would run on alone at the end.
//   otherwise: every query block costs the same and the query block is the innermost index,
//   so the items that read the same (unit, key split) K/V run side by side and share it
//   through L2.
__host__ __device__ inline void item_coords(const FwdParams& p, int idx, int& bh, int& split,
                                            int& qb) {
  const int per_unit = p.n_qblk * p.splits;
  if (p.heavy_first) {
    const int BH = p.B * p.H;
    const int base = BH / p.n_groups, n_big = BH % p.n_groups;
    const int big_items = (base + 1) * per_unit;  // items of each of the first n_big groups
    int g0, gsize, local;
    if (idx < n_big * big_items) {
      const int grp = idx / big_items;
      g0 = grp * (base + 1);
      gsize = base + 1;
      local = idx - grp * big_items;
    } else {
      const int r = idx - n_big * big_items;
      const int k = r / (base * per_unit);
      g0 = n_big * (base + 1) + k * base;
      gsize = base;
      local = r - k * base * per_unit;
    }
    const int qrank = local / (gsize * p.splits);
    const int rem = local - qrank * gsize * p.splits;
    bh = g0 + rem / p.splits;
    split = rem % p.splits;
    qb = p.n_qblk - 1 - qrank;
  } else {
    bh = idx / per_unit;
    const int rem = idx - bh * per_unit;
    split = rem / p.n_qblk;
    qb = rem % p.n_qblk;
  }
}

// Positions per RoPE rotation item (FwdParams::rope_items counts chunks of this many rows).
constexpr int kRopeRows = 128;

}  // namespace mlxp
