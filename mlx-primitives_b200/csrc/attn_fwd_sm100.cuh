// attn_fwd_sm100.cuh — bf16/fp16 attention forward on the 5th-generation tensor cores (sm_100a).
//
// Persistent kernel: one CTA per SM pulls work items from a device-wide counter.  A work item
// is 256 query rows (two 128-row Q tiles, "tile 0" and "tile 1") of one (batch, head), against
// a range of 128-key K/V tiles (optionally one of several key splits).  Items are numbered in
// groups of (batch, head) units so that the CTAs running at the same time share K/V through
// L2, heaviest query blocks of a group first when the mask is causal (see decode_item).
//
//   warp 9        TMA producer: fetches items and decodes each into a shared-memory slot for the
//                 other roles, then loads Q once per item and K, V tiles into two shared-memory
//                 rings (128-byte swizzle), K and V released separately.  The rings, barriers and
//                 TMEM persist across items, so the next item's loads overlap the current one.
//   warp 8        MMA issuer (one thread): S_t = Q_t K^T (SS form, fp32 accumulate in TMEM),
//                 then O_t += P_t V (TS form: P_t read from TMEM, V from smem).
//   warps 0-3     softmax for tile 0, warps 4-7 softmax for tile 1: one thread owns one query
//                 row (TMEM lane), reads its 128 scores with tcgen05.ld, masks boundary tiles,
//                 updates the running max/sum, writes P (bf16/fp16, packed two per 32-bit
//                 column) back over the S columns with tcgen05.st, and rescales O in TMEM only
//                 when the running max grew by more than 2^8 (exact: the final 1/l uses the
//                 same stale max as the exponentials).  The same warps run the epilogue, which
//                 overlaps the tensor core's first QK of the next item.
//   warps 10-11   spare (the control warpgroup is register-starved by design).
//
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D); P_t aliases
// the first 64 columns of S_t.  The two tiles ping-pong: while softmax works on S_0 the tensor
// core runs PV_1 / QK_1 and vice versa.  The MMA issue order per tile is PV_t(j), QK_t(j+1):
// tcgen05.mma instructions from one thread execute in order, so QK_t(j+1) may overwrite the
// S/P columns right after PV_t(j) is issued, and the commit after QK_t(j+1) also certifies that
// PV_t(j) finished — which is what lets the softmax warps rescale O without another barrier.
// Across items the same order holds (PV_t(last of i) before QK_t(first of i+1)), and the first
// PV_t of item i+1 (which overwrites O_t) waits for P_t, which the softmax warps publish only
// after their epilogue of item i has read O_t.
//
// Every wait is bounded (mbar_wait); when one gives up the CTA drains its in-flight TMA
// loads and MMAs (bounded again), frees TMEM and returns, leaving the error in the device
// status word.
#pragma once

#include <type_traits>

#include "attn_common.cuh"
#include "rope.cuh"
#include "sm100_ptx.cuh"

namespace mlxp {

// Cycle-counter trace of CTA 0 for pipeline analysis: compiled in only with -DMLXP_TRACE=1
// (roles 0/1 softmax tiles, 2 MMA issuer, 3 TMA producer; 64 iterations x 8 stamps each).
#ifndef MLXP_TRACE
#define MLXP_TRACE 0
#endif
#if MLXP_TRACE
__device__ long long g_mlxp_trace[4 * 64 * 8];
__device__ long long g_mlxp_cta_trace[8192 * 4];  // per item: start ns, end ns, SM id, key tiles
__device__ long long g_mlxp_cta_life[1024 * 3];   // per CTA: entry ns, prologue done ns, exit ns
__device__ long long g_mlxp_rot_trace[2048 * 3];  // per rotation item: start ns, end ns, SM id
#define MLXP_TR(cond, role, it, k)                                                    \
  do {                                                                                \
    if ((cond) && blockIdx.x == 0 && (it) < 64)                                       \
      g_mlxp_trace[((role) * 64 + (it)) * 8 + (k)] = clock64();                       \
  } while (0)
#else
#define MLXP_TR(cond, role, it, k) \
  do {                             \
  } while (0)
#endif

template <int D, int NS>
struct Sm100Cfg {
  static constexpr int BM = 128;  // rows per Q tile (= TMEM lanes)
  static constexpr int BN = 128;  // keys per K/V tile
  static constexpr int KB = D / 64;  // 128-byte (64-element) column blocks
  static constexpr int Q_TILE = BM * D * 2;
  static constexpr int KV_TILE = BN * D * 2;
  static constexpr int BOX_Q = BM * 128;   // bytes of one 64-column box of a Q tile
  static constexpr int BOX_KV = BN * 128;  // bytes of one 64-column box of a K/V tile
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * Q_TILE;
  static constexpr int OFF_V = OFF_K + NS * KV_TILE;
  // Epilogue staging: one 128-row x 128-byte box (16 KB, 128-byte swizzle) per Q tile, from
  // which O leaves through TMA stores (64 bf16/fp16 or 32 fp32 columns per box).
  static constexpr int STAGE_BYTES = BM * 128;
  static constexpr int OFF_STAGE = OFF_V + NS * KV_TILE;
  static constexpr int OFF_BAR = OFF_STAGE + 2 * STAGE_BYTES;
  // barrier indices
  static constexpr int B_QF = 0;           // Q loaded
  static constexpr int B_QE = 1;           // Q buffer free (last QK of the item done)
  // K and V have rings of NS stages each, with a "loaded" and a "free" barrier per stage.  K of
  // key tile j is last read by the QKs issued one step before V of tile j is read, so K's stage
  // is released as soon as those QKs complete: the load of K(j + NS) then has about a whole step
  // more lead than when K and V of a tile were released together (measured: QK waited 0.5-1.4 K
  // cycles per key tile for its K with the shared release).
  static constexpr int B_KF = 2;
  static constexpr int B_VF = B_KF + NS;
  static constexpr int B_KE = B_VF + NS;
  static constexpr int B_VE = B_KE + NS;
  static constexpr int B_SF = B_VE + NS;   // 2: S_t ready
  static constexpr int B_PF = B_SF + 2;    // 2: P_t ready (128 arrivals)
  static constexpr int B_OF = B_PF + 2;    // 2: last PV_t of an item complete
  static constexpr int B_WF = B_OF + 2;    // 2: work-item slot filled
  static constexpr int B_WE = B_WF + 2;    // 2: work-item slot read by every consumer
  static constexpr int B_DR = B_WE + 2;    // 1: MMA drain
  static constexpr int NBAR = B_DR + 1;
  // tmem slot, abort flag, 2 item slots, 2 per-tile "merge the key splits" flags, 2 slots of
  // the RoPE phase's item counter; then the two work-item slots' decoded items (ITEM_INTS ints
  // each, written by the producer so that the other roles need not decode)
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int ITEM_INTS = 16;
  static constexpr int OFF_ITEM = OFF_MISC + 32;
  static constexpr int SMEM_BYTES = OFF_ITEM + 2 * ITEM_INTS * 4;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to align the base to 1024 B
  // Three warpgroups: WG0/WG1 softmax (tiles 0/1), WG2 = MMA warp, TMA warp, two spare warps.
  // Registers are split per SM sub-partition, so the launch gets 65536/384 -> 168 per thread
  // and setmaxnreg moves them to the softmax warpgroups: 2*128*208 + 128*80 = 63488 <= 384*168.
  static constexpr int THREADS = 384;
  static constexpr int REGS_SOFTMAX = 208;
  static constexpr int REGS_CONTROL = 80;
  static_assert(2 * 128 * REGS_SOFTMAX + 128 * REGS_CONTROL <= THREADS * 168, "register split");
  // consumers of a work-item slot: the MMA thread and the 256 softmax threads
  static constexpr int WORK_READERS = 1 + 256;
  static constexpr uint32_t TM_S0 = 0, TM_S1 = 128, TM_O0 = 256, TM_O1 = 256 + D;
  static constexpr uint32_t TM_COLS = 512;
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

// wait-site codes recorded in the device status word
enum : int {
  kSiteProducer = 1,
  kSiteMmaLoad = 2,
  kSiteMmaP = 3,
  kSiteSoftmaxS = 4,
  kSiteSoftmaxO = 5,
  kSiteDrain = 6,
  kSiteSelfTest = 7,
  kSiteWork = 8,
  kSiteEpilogue = 10,
  kSiteRope = 11
};

// Of every 8 column pairs of a score row, this many are exponentiated with exp2_poly2 (FMA pipe)
// and the rest with ex2.approx (MUFU): splits the per-row exp2 work between the two units.
// head_dim 64 has half the MMA work per score, so some of its exponentials go to the FMA pipe;
// for head_dim 128 the measured optimum is MUFU only (the polynomial's extra instructions cost
// more than the MUFU time they save).
#ifndef MLXP_POLY_D64
#define MLXP_POLY_D64 2
#endif
#ifndef MLXP_POLY_D128
#define MLXP_POLY_D128 0
#endif
template <int D>
constexpr int kPolyPerOct = (D == 64) ? MLXP_POLY_D64 : MLXP_POLY_D128;

// Wait without looking at the abort flag (used when draining after an abort).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, int* status,
                                                uint64_t timeout_ns) {
  int dummy_flag = 0;
  WaitCtx w{&dummy_flag, status, timeout_ns};
  if (mbar_try_wait(bar, parity)) return true;
  // mbar_wait_slow reads the flag through a volatile pointer; a private flag is never set.
  return mbar_wait_slow(bar, parity, w, kSiteDrain);
}

__device__ __forceinline__ void tma_coords(const TmaCoordMap& cm, int s, int h, int b, int& c1,
                                           int& c2, int& c3) {
  const int hh = cm.bcast_h ? 0 : h;
  const int bb = cm.bcast_b ? 0 : b;
  c1 = (cm.slot_s == 1) ? s : (cm.slot_h == 1) ? hh : bb;
  c2 = (cm.slot_s == 2) ? s : (cm.slot_h == 2) ? hh : bb;
  c3 = (cm.slot_s == 3) ? s : (cm.slot_h == 3) ? hh : bb;
}

// One work item.  The producer decodes it from its index and publishes it in shared memory
// with the index (put_item / get_item), so that the MMA thread and the softmax warps, which
// start an item on the critical path, read 16 ints instead of redoing the integer divisions
// of the item order (measured: ~1.7 K cycles per item start in the softmax warps).
struct WorkItem {
  int rot, grp;            // rotation chunk (-1: an attention item) and scheduling group
  int b, h, split, q0;
  int lo0, hi0, lo1, hi1;  // key-tile ranges of Q tiles 0 and 1 (empty: lo == hi)
  int lo, hi;              // union range
  int flo0, fhi0, flo1, fhi1;  // key tiles that need no mask, per Q tile (full_tile_range)
};
static_assert(sizeof(WorkItem) == 16 * sizeof(int), "WorkItem is 16 ints");

__device__ __forceinline__ void put_item(volatile int* d, const WorkItem& w) {
  const int* s = reinterpret_cast<const int*>(&w);
#pragma unroll
  for (int i = 0; i < 16; ++i) d[i] = s[i];
}
__device__ __forceinline__ WorkItem get_item(const volatile int* d) {
  WorkItem w;
  int* s = reinterpret_cast<int*>(&w);
#pragma unroll
  for (int i = 0; i < 16; ++i) s[i] = d[i];
  return w;
}

// Decodes work item idx (item_coords in attn_common.cuh gives its unit, key split and query
// block); run by the producer, which publishes the result for the other roles.
template <bool kRope>
__device__ __forceinline__ WorkItem decode_item(const FwdParams& p, int idx, int BN) {
  WorkItem w;
  int bh, qb;
  item_coords(p, idx, bh, w.split, qb);
  w.rot = -1;
  w.grp = 0;
  if constexpr (kRope) {  // the scheduling group, whose rotation the item waits for
    const int base = p.B * p.H / p.n_groups, n_big = p.B * p.H % p.n_groups;
    w.grp = bh < n_big * (base + 1) ? bh / (base + 1) : n_big + (bh - n_big * (base + 1)) / base;
  }
  w.h = bh % p.H;
  w.b = bh / p.H;
  w.q0 = qb * 256;
  int lo_t[2], hi_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const long long r0 = w.q0 + t * 128;
    const long long r1 = (r0 + 128 < p.Sq) ? r0 + 128 : p.Sq;
    kv_tile_range(p.mask, r0, r1, BN, lo_t[t], hi_t[t]);
    if (p.splits > 1) {
      const int s_lo = w.split * p.tiles_per_split, s_hi = s_lo + p.tiles_per_split;
      if (lo_t[t] < s_lo) lo_t[t] = s_lo;
      if (hi_t[t] > s_hi) hi_t[t] = s_hi;
      if (hi_t[t] < lo_t[t]) hi_t[t] = lo_t[t];
    }
  }
  w.lo0 = lo_t[0];
  w.hi0 = hi_t[0];
  w.lo1 = lo_t[1];
  w.hi1 = hi_t[1];
  const bool a0 = w.hi0 > w.lo0, a1 = w.hi1 > w.lo1;
  w.lo = (a0 && a1) ? min(w.lo0, w.lo1) : a0 ? w.lo0 : a1 ? w.lo1 : 0;
  w.hi = (a0 && a1) ? max(w.hi0, w.hi1) : a0 ? w.hi0 : a1 ? w.hi1 : 0;
  int fl[2] = {0, 0}, fh[2] = {0, 0};
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const long long r0 = w.q0 + t * 128;
    const long long r1 = (r0 + 128 < p.Sq) ? r0 + 128 : p.Sq;
    if (r1 > r0) full_tile_range(p.mask, r0, r1, BN, fl[t], fh[t]);
  }
  w.flo0 = fl[0];
  w.fhi0 = fh[0];
  w.flo1 = fl[1];
  w.fhi1 = fh[1];
  return w;
}

// A rotation item, run by all NT threads of the CTA: positions [chunk * kRopeRows, +kRopeRows)
// of Q or K for every (batch, head) unit of one scheduling group, rotated with the half-split
// RoPE (rope_pair: the RoPE kernel's exact arithmetic) into the contiguous copies that the
// tensor maps read.  A thread owns (row, 8-element chunk pair) slots: it loads the slot's cos
// and sin once and applies them to the group's units, whose loads it issues in batches of UB
// before any store (the stores could alias the loads as far as the compiler knows, which would
// otherwise serialise every unit on a full memory latency).
template <int D, bool kBF16, int NT>
__device__ __forceinline__ void rope_rotate_group(const FwdParams& p, const WorkItem& w, int tid) {
  using T = std::conditional_t<kBF16, __nv_bfloat16, __half>;
  constexpr int CP = D / 16;  // chunk pairs (8 elements of each half) per row
  constexpr int UB = 8;       // units whose loads are in flight together
  const bool isq = w.rot < p.rope_q_items;
  const int chunk = isq ? w.rot : w.rot - p.rope_q_items;
  const long long S = isq ? p.Sq : p.Skv;
  const long long r0 = (long long)chunk * kRopeRows;
  const int nrows = (int)(S - r0 < kRopeRows ? S - r0 : kRopeRows);
  const int BH = p.B * p.H, base = BH / p.n_groups, n_big = BH % p.n_groups;
  const int u0 = w.b * p.H + w.h;  // the group's first unit
  const int u1 = u0 + base + (w.grp < n_big ? 1 : 0);
  const long long* st = isq ? p.rq_s : p.rk_s;
  const T* __restrict__ srcb = static_cast<const T*>(isq ? p.rq_src : p.rk_src);
  T* __restrict__ dstb = static_cast<T*>(isq ? p.rq_dst : p.rk_dst);
  const long long pos0 = (isq ? p.rope_q_pos : p.rope_k_pos) + r0;
  for (int i = tid; i < nrows * CP; i += NT) {
    const int r = i / CP, j = i - r * CP;
    const float4* cr = reinterpret_cast<const float4*>(p.rope_cos + (pos0 + r) * (D / 2) + 8 * j);
    const float4* sr = reinterpret_cast<const float4*>(p.rope_sin + (pos0 + r) * (D / 2) + 8 * j);
    const float4 c0 = __ldg(cr), c1 = __ldg(cr + 1), s0 = __ldg(sr), s1 = __ldg(sr + 1);
    const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const long long row = r0 + r;
    for (int u = u0; u < u1; u += UB) {
      uint4 v1[UB], v2[UB];
#pragma unroll
      for (int k = 0; k < UB; ++k) {
        if (u + k < u1) {
          const int b = (u + k) / p.H, h = (u + k) - b * p.H;
          const T* x = srcb + (long long)b * st[0] + (long long)h * st[1] + row * st[2] + 8 * j;
          v1[k] = *reinterpret_cast<const uint4*>(x);
          v2[k] = *reinterpret_cast<const uint4*>(x + D / 2);
        }
      }
#pragma unroll
      for (int k = 0; k < UB; ++k) {
        if (u + k >= u1) continue;
        const T* x1 = reinterpret_cast<const T*>(&v1[k]);
        const T* x2 = reinterpret_cast<const T*>(&v2[k]);
        uint4 o1, o2;
        T* y1 = reinterpret_cast<T*>(&o1);
        T* y2 = reinterpret_cast<T*>(&o2);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float a, bb;
          rope_pair(to_f<T>(x1[e]), to_f<T>(x2[e]), cc[e], ss[e], a, bb);
          y1[e] = from_f<T>(a);
          y2[e] = from_f<T>(bb);
        }
        T* y = dstb + ((long long)(u + k) * S + row) * D + 8 * j;
        *reinterpret_cast<uint4*>(y) = o1;
        *reinterpret_cast<uint4*>(y + D / 2) = o2;
      }
    }
  }
}

template <int D, bool kBF16, int NS, bool kBias, bool kRope>
__global__ void __launch_bounds__(384, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_o, const FwdParams p) {
  using C = Sm100Cfg<D, NS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + C::OFF_MISC + 4);
  volatile int* work_slot = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8);
  volatile int* merge_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 16);
  volatile int* item_slot = reinterpret_cast<volatile int*>(smem + C::OFF_ITEM);  // [2][ITEM_INTS]
  // (RoPE phase: two more slots after merge_flag, work_slot + 4 and + 5)
  auto BAR = [&](int i) -> uint32_t { return sbase + C::OFF_BAR + 8 * i; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = p.n_qblk * p.B * p.H * p.splits;
#if MLXP_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_mlxp_cta_life[blockIdx.x * 3] = (long long)global_timer_ns();
#endif

  if (threadIdx.x == 0) {
    mbar_init(BAR(C::B_QF), 1);
    mbar_init(BAR(C::B_QE), 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(BAR(C::B_KF + i), 1);
      mbar_init(BAR(C::B_VF + i), 1);
      mbar_init(BAR(C::B_KE + i), 1);
      mbar_init(BAR(C::B_VE + i), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(BAR(C::B_SF + t), 1);
      mbar_init(BAR(C::B_PF + t), 128);
      mbar_init(BAR(C::B_OF + t), 1);
      mbar_init(BAR(C::B_WF + t), 1);
      mbar_init(BAR(C::B_WE + t), C::WORK_READERS);
    }
    mbar_init(BAR(C::B_DR), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(smem_u32(tmem_slot), C::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx wctx{abort_flag, p.status, p.timeout_ns};
#if MLXP_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 1024) g_mlxp_cta_life[blockIdx.x * 3 + 1] = (long long)global_timer_ns();
#endif
  if constexpr (kRope) {
    // RoPE phase, before the warp roles split (and rebalance their registers): all threads
    // claim rotation items from their own counter until none is left, then count each one
    // done for its group.  Rotation never waits for anything, so the attention items that
    // wait for it (producer, below) always see it finish.
    volatile int* rot_slot = work_slot + 4;  // merge_flag[2] sits at work_slot + 2
    const int n_rot = p.n_groups * p.rope_items;
    for (int round = 0;; ++round) {
      if (threadIdx.x == 0) rot_slot[round & 1] = (int)atomicAdd(p.rot_counter, 1u);
      __syncthreads();
      const int r = rot_slot[round & 1];
      if (r >= n_rot) break;
      WorkItem w;
      w.grp = r / p.rope_items;
      w.rot = r - w.grp * p.rope_items;
      {
        const int base = p.B * p.H / p.n_groups, n_big = p.B * p.H % p.n_groups;
        const int u0 = w.grp * base + (w.grp < n_big ? w.grp : n_big);
        w.b = u0 / p.H;
        w.h = u0 - w.b * p.H;
      }
#if MLXP_TRACE
      const long long tr0 = (long long)global_timer_ns();
#endif
      rope_rotate_group<D, kBF16, C::THREADS>(p, w, (int)threadIdx.x);
      fence_proxy_async_global();
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) {
        atomicAdd(p.rot_done + w.grp, 1u);
#if MLXP_TRACE
        if (r < 2048) {
          uint32_t smid;
          asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
          g_mlxp_rot_trace[r * 3 + 0] = tr0;
          g_mlxp_rot_trace[r * 3 + 1] = (long long)global_timer_ns();
          g_mlxp_rot_trace[r * 3 + 2] = smid;
        }
#endif
      }
    }
  }

  if (warp >= 8) {
    // ================================ control warpgroup ================================
    setmaxnreg_dec<C::REGS_CONTROL>();
    if (warp == 9) {
      // =================================== TMA producer ===================================
      if (lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        tma_prefetch_desc(&tm_o);
        const uint32_t sQ = sbase + C::OFF_Q, sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
        int fk = 0, n_q = 0;  // key-tile fills (K) and Q loads issued so far
        int fv = 0;           // V fills issued (fk, or fk - 1 after an abort between K and V)
        int rot_ready = -1;   // scheduling groups up to this one have their Q and K rotated
        bool ok = true;
        for (int item = 0; ok; ++item) {
          const int slot = item & 1;
          MLXP_TR(true, 3, item, 0);
          if (item >= 2) {
            ok = mbar_wait(BAR(C::B_WE + slot), ((item >> 1) - 1) & 1, wctx, kSiteWork);
            if (!ok) break;
          }
          // the first item of every CTA is its block index (no atomic on the launch's
          // critical path); later ones come from the counter, past the first gridDim.x.
          const int idx = item == 0 ? (int)blockIdx.x
                                    : (int)(gridDim.x + atomicAdd(p.work_counter, 1u));
          WorkItem w{};
          if (idx < n_items) w = decode_item<kRope>(p, idx, C::BN);
          work_slot[slot] = idx;
          put_item(item_slot + slot * C::ITEM_INTS, w);
          MLXP_TR(true, 3, item, 1);
          mbar_arrive(BAR(C::B_WF + slot));  // release: the slot writes are visible to waiters
          if (idx >= n_items) break;
          if (w.hi <= w.lo) continue;  // empty items load nothing
          if (kRope && w.grp > rot_ready) {
            // Q and K of this group are rotated by the RoPE phase of this and other CTAs: wait
            // until all of the group's rotation items are done
            const unsigned need = (unsigned)p.rope_items;
            ok = wait_count_geq(p.rot_done + w.grp, need, wctx, kSiteRope);
            if (!ok) break;
            fence_proxy_async_global();  // the rotated rows, written by generic stores, for TMA
            rot_ready = w.grp;
          }
#if MLXP_TRACE
          if (idx < 8192) {
            uint32_t smid;
            asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
            g_mlxp_cta_trace[idx * 4 + 0] = (long long)global_timer_ns();
            g_mlxp_cta_trace[idx * 4 + 2] = smid;
            g_mlxp_cta_trace[idx * 4 + 3] = w.hi - w.lo;
          }
#endif
          int c1, c2, c3;
          const bool a0 = w.hi0 > w.lo0, a1 = w.hi1 > w.lo1;
          if (n_q > 0) {
            ok = mbar_wait(BAR(C::B_QE), (n_q - 1) & 1, wctx, kSiteProducer);
            if (!ok) break;
          }
          MLXP_TR(true, 3, item, 2);
          mbar_arrive_expect_tx(BAR(C::B_QF), (a0 + a1) * C::Q_TILE);
          for (int t = 0; t < 2; ++t) {
            if (!(t ? a1 : a0)) continue;
            tma_coords(p.cq, w.q0 + t * 128, w.h, w.b, c1, c2, c3);
#pragma unroll
            for (int kb = 0; kb < C::KB; ++kb)
              tma_load_4d(sQ + t * C::Q_TILE + kb * C::BOX_Q, &tm_q, BAR(C::B_QF), kb * 64, c1,
                          c2, c3);
          }
          ++n_q;
          for (int j = w.lo; j < w.hi && ok; ++j) {
            const int ks = fk % NS;
            if (fk >= NS) ok = mbar_wait(BAR(C::B_KE + ks), ((fk / NS) - 1) & 1, wctx, kSiteProducer);
            if (!ok) break;
            mbar_arrive_expect_tx(BAR(C::B_KF + ks), C::KV_TILE);
            tma_coords(p.ck, j * C::BN, w.h / p.kv_group, w.b, c1, c2, c3);
#pragma unroll
            for (int kb = 0; kb < C::KB; ++kb)
              tma_load_4d(sK + ks * C::KV_TILE + kb * C::BOX_KV, &tm_k, BAR(C::B_KF + ks),
                          kb * 64, c1, c2, c3);
            if (fk >= NS) ok = mbar_wait(BAR(C::B_VE + ks), ((fk / NS) - 1) & 1, wctx, kSiteProducer);
            if (!ok) {
              ++fk;  // K of this fill is in flight (its V is not): the abort path waits for it
              break;
            }
            mbar_arrive_expect_tx(BAR(C::B_VF + ks), C::KV_TILE);
            tma_coords(p.cv, j * C::BN, w.h / p.kv_group, w.b, c1, c2, c3);
#pragma unroll
            for (int kb = 0; kb < C::KB; ++kb)
              tma_load_4d(sV + ks * C::KV_TILE + kb * C::BOX_KV, &tm_v, BAR(C::B_VF + ks),
                          kb * 64, c1, c2, c3);
            MLXP_TR(j == w.lo, 3, item, 3);
            MLXP_TR(j == w.hi - 1, 3, item, 4);
            ++fk;
            ++fv;
          }
        }
        if (!ok) {
          // Abort: let every load already issued land before the CTA releases its smem.
          if (n_q > 0) mbar_wait_drain(BAR(C::B_QF), (n_q - 1) & 1, p.status, p.timeout_ns);
          // the last NS fills of each ring are the latest of their stages (older ones landed
          // before their stage was waited free)
          for (int f = (fk > NS ? fk - NS : 0); f < fk; ++f)
            mbar_wait_drain(BAR(C::B_KF + f % NS), (f / NS) & 1, p.status, p.timeout_ns);
          for (int f = (fv > NS ? fv - NS : 0); f < fv; ++f)
            mbar_wait_drain(BAR(C::B_VF + f % NS), (f / NS) & 1, p.status, p.timeout_ns);
        }
      }
    } else if (warp == 8) {
      // ==================================== MMA issuer ====================================
      if (lane == 0) {
        constexpr uint32_t idesc_qk = make_idesc_f16(128, C::BN, kBF16, false);
        constexpr uint32_t idesc_pv = make_idesc_f16(128, D, kBF16, true);
        // Shared-memory descriptors are kept as (lo, hi) 32-bit words; between MMAs only the
        // start-address field (lo bits 0-13, 16-byte units) moves, so issuing one MMA costs
        // one 32-bit add.  K-major Q/K: LBO unused (16 B).  MN-major V: LBO = next 64 columns.
        const uint32_t q_lo = ((sbase + C::OFF_Q) >> 4) | (1u << 16);
        const uint32_t k_lo = ((sbase + C::OFF_K) >> 4) | (1u << 16);
        const uint32_t v_lo = ((sbase + C::OFF_V) >> 4) | ((uint32_t)(C::BOX_KV >> 4) << 16);

        auto issue_qk = [&](auto tile, int ks) {
          constexpr int T = decltype(tile)::value;
          const uint32_t d = tmem + (T ? C::TM_S1 : C::TM_S0);
          const uint32_t a0 = q_lo + (uint32_t)(T * C::Q_TILE >> 4);
          const uint32_t b0 = k_lo + (uint32_t)ks * (uint32_t)(C::KV_TILE >> 4);
#pragma unroll
          for (int kb = 0; kb < C::KB; ++kb) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              mma_ss(d, sdesc(a0 + (uint32_t)((kb * C::BOX_Q + kk * 32) >> 4)),
                     sdesc(b0 + (uint32_t)((kb * C::BOX_KV + kk * 32) >> 4)), idesc_qk,
                     (kb | kk) ? 1u : 0u);
            }
          }
        };
        auto issue_pv = [&](auto tile, int vs, bool acc) {
          constexpr int T = decltype(tile)::value;
          const uint32_t d = tmem + (T ? C::TM_O1 : C::TM_O0);
          const uint32_t a = tmem + (T ? C::TM_S1 : C::TM_S0);
          const uint32_t b0 = v_lo + (uint32_t)vs * (uint32_t)(C::KV_TILE >> 4);
#pragma unroll
          for (int kk = 0; kk < C::BN / 16; ++kk)
            mma_ts(d, a + kk * 8, sdesc(b0 + (uint32_t)(kk * 16 * 128 >> 4)), idesc_pv,
                   (acc || kk > 0) ? 1u : 0u);
        };
        using T0 = std::integral_constant<int, 0>;
        using T1 = std::integral_constant<int, 1>;
        int c = 0, n_q = 0, pc0 = 0, pc1 = 0;  // consumed key-tile fills, Q loads, P waits
        int ke_pending = -1;  // K ring stage whose release commit is still to be issued
        int trace_f = 0;
        bool ok = true;
        for (int item = 0; ok; ++item) {
          const int slot = item & 1;
          ok = mbar_wait(BAR(C::B_WF + slot), (item >> 1) & 1, wctx, kSiteWork);
          if (!ok) break;
          const int idx = work_slot[slot];
          const WorkItem w = get_item(item_slot + slot * C::ITEM_INTS);
          mbar_arrive(BAR(C::B_WE + slot));
          if (idx >= n_items) break;
          if (w.hi <= w.lo) continue;
          // One tile's share of key tile j: PV_t(j) once P_t(j) is ready (tile_pv), then QK_t(j+1)
          // (tile_qk).  The K of key tile j+1 is fill c+1 (ring stage ksn).
          auto tile_pv = [&](auto tile, int j, int vs) -> bool {
            constexpr int T = decltype(tile)::value;
            const int tlo = T ? w.lo1 : w.lo0, thi = T ? w.hi1 : w.hi0;
            int& pc = T ? pc1 : pc0;
            if (j >= tlo && j < thi) {
              if (!mbar_wait(BAR(C::B_PF + T), pc & 1, wctx, kSiteMmaP)) return false;
              MLXP_TR(true, 2, trace_f, 2 + 2 * T);
              ++pc;
              tc_fence_after();
              issue_pv(tile, vs, j > tlo);
              if (j == thi - 1) tc_commit(BAR(C::B_OF + T));
            }
            return true;
          };
          auto tile_qk = [&](auto tile, int j, bool has_next, int ksn, bool& k_ready) -> bool {
            constexpr int T = decltype(tile)::value;
            const int tlo = T ? w.lo1 : w.lo0, thi = T ? w.hi1 : w.hi0;
            if (has_next && j + 1 >= tlo && j + 1 < thi) {
              if (!k_ready) {
                if (!mbar_wait(BAR(C::B_KF + ksn), ((c + 1) / NS) & 1, wctx, kSiteMmaLoad))
                  return false;
                tc_fence_after();
                k_ready = true;
              }
              issue_qk(tile, ksn);
              tc_commit(BAR(C::B_SF + T));
            }
            MLXP_TR(true, 2, trace_f, 3 + 2 * T);
            return true;
          };

          ok = mbar_wait(BAR(C::B_QF), n_q & 1, wctx, kSiteMmaLoad);
          MLXP_TR(true, 2, trace_f, 6);
          if (ok) ok = mbar_wait(BAR(C::B_KF + c % NS), (c / NS) & 1, wctx, kSiteMmaLoad);
          MLXP_TR(true, 2, trace_f, 7);
          if (!ok) break;
          ++n_q;
          tc_fence_after();
          if (w.lo >= w.lo0 && w.lo < w.hi0) {
            issue_qk(T0{}, c % NS);
            tc_commit(BAR(C::B_SF + 0));
          }
          if (w.lo >= w.lo1 && w.lo < w.hi1) {
            issue_qk(T1{}, c % NS);
            tc_commit(BAR(C::B_SF + 1));
          }
          ke_pending = c % NS;  // K(lo) is consumed once these QKs complete
          if (w.hi - w.lo == 1) tc_commit(BAR(C::B_QE));  // every QK of this item is issued
          for (int j = w.lo; j < w.hi && ok; ++j, ++trace_f, ++c) {
            const int vs = c % NS;
            const bool has_next = j + 1 < w.hi;
            const int ksn = (c + 1) % NS;
            bool k_ready = false;
            MLXP_TR(true, 2, trace_f, 0);
            ok = mbar_wait(BAR(C::B_VF + vs), (c / NS) & 1, wctx, kSiteMmaLoad);
            // K(j+1) too, here rather than between PV_0(j) and QK_0(j+1): a wait in the MMA
            // thread leaves the tensor pipe idle for its duration when few MMAs are queued
            if (ok && has_next) {
              ok = mbar_wait(BAR(C::B_KF + ksn), ((c + 1) / NS) & 1, wctx, kSiteMmaLoad);
              k_ready = true;
            }
            MLXP_TR(true, 2, trace_f, 1);
            if (!ok) break;
            tc_fence_after();
            ok = tile_pv(T0{}, j, vs);
            if (ke_pending >= 0) {
              // the previous step's K release, issued behind PV_0(j) where the MMA queue is full
              tc_commit(BAR(C::B_KE + ke_pending));
              ke_pending = -1;
            }
            if (ok) ok = tile_qk(T0{}, j, has_next, ksn, k_ready);
            if (ok) ok = tile_pv(T1{}, j, vs);
            if (!ok) break;
            tc_commit(BAR(C::B_VE + vs));  // V(j) is consumed
            ok = tile_qk(T1{}, j, has_next, ksn, k_ready);
            if (!ok) break;
            if (has_next) ke_pending = ksn;  // K(j+1) is consumed: every QK(j+1) is issued
            if (j + 2 == w.hi) tc_commit(BAR(C::B_QE));  // the item's last QKs are issued
          }
        }
        if (ke_pending >= 0) tc_commit(BAR(C::B_KE + ke_pending));
        // Every MMA issued by this thread must finish before TMEM/smem are released.
        tc_commit(BAR(C::B_DR));
        mbar_wait_drain(BAR(C::B_DR), 0, p.status, p.timeout_ns);
      }
    }  // warps 10-11: spare
    // ---- teardown: every role is done with TMEM and smem after this barrier
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
      tc_fence_after();
      tmem_dealloc(tmem, C::TM_COLS);
    }
  } else {
    // ============================== softmax + epilogue (tile t) ==============================
    setmaxnreg_inc<C::REGS_SOFTMAX>();
    const int t = warp >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + (t ? C::TM_S1 : C::TM_S0);
    const uint32_t tO = tmem + lane_off + (t ? C::TM_O1 : C::TM_O0);
    const float sl2 = p.scale_log2;
    int n_s = 0, n_o = 0;  // S tiles and item epilogues consumed by this tile so far
    bool ok = true;
    for (int item = 0; ok; ++item) {
      const int slot = item & 1;
      ok = mbar_wait(BAR(C::B_WF + slot), (item >> 1) & 1, wctx, kSiteWork);
      ok = named_bar_and(1 + t, 128, ok);  // the tile's warps leave the item loop together
      if (!ok) break;
      const int idx = work_slot[slot];
      const WorkItem w = get_item(item_slot + slot * C::ITEM_INTS);
      mbar_arrive(BAR(C::B_WE + slot));
      if (idx >= n_items) break;
      const int tlo = t ? w.lo1 : w.lo0, thi = t ? w.hi1 : w.hi0;
      const int qrow = w.q0 + t * 128 + row;
      const long long r0 = w.q0 + t * 128;
      const long long r1 = (r0 + 128 < p.Sq) ? r0 + 128 : p.Sq;
      const int flo = t ? w.flo1 : w.flo0, fhi = t ? w.fhi1 : w.fhi0;  // key tiles that need no mask
      float m = -INFINITY, l = 0.f;

      for (int it = 0; it < thi - tlo; ++it, ++n_s) {
        const int j = tlo + it;
        MLXP_TR(wq == 0 && lane == 0, t, it, 0);
        ok = mbar_wait(BAR(C::B_SF + t), n_s & 1, wctx, kSiteSoftmaxS);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        MLXP_TR(wq == 0 && lane == 0, t, it, 1);
        tc_fence_after();
        // Boundary tiles (rare) are masked in TMEM first, by a small rolled loop over 32-column
        // chunks, so that the unrolled register path below carries no masking code.  Per warp,
        // a chunk that is admissible for all 32 rows is left alone, one that is masked for all
        // of them is overwritten with -inf without being read, and only a straddling chunk is
        // read, masked element-wise and written back.
        {
          if (j < flo || j >= fhi) {
            const long long c0 = (long long)j * C::BN;
            int c_lo, c_hi;
            row_col_interval(p.mask, qrow, c0, C::BN, c_lo, c_hi);
            // the warp's extreme bounds decide each chunk's case once for all 32 rows
            const int lo_min = __reduce_min_sync(0xffffffffu, c_lo);
            const int lo_max = __reduce_max_sync(0xffffffffu, c_lo);
            const int hi_min = __reduce_min_sync(0xffffffffu, c_hi);
            const int hi_max = __reduce_max_sync(0xffffffffu, c_hi);
            const int width = (c_hi >= c_lo) ? c_hi - c_lo + 1 : 0;  // admissible columns
            bool stored = false;
#pragma unroll 1
            for (int k = 0; k < C::BN / 32; ++k) {
              const int k0 = 32 * k, k1 = 32 * k + 31;
              if (lo_max <= k0 && hi_min >= k1) continue;  // admissible for every row
              if (hi_max < k0 || lo_min > k1) {            // masked for every row
                tmem_fill_x32(tS + k0, 0xff800000u);
              } else {
                uint32_t r[32];
                tmem_ld_x32(tS + k0, r);
                tmem_wait_ld();
                reg_fence(r);
                const int lo = c_lo - k0;
#pragma unroll
                for (int i = 0; i < 32; ++i)  // i in [lo, lo + width) <=> (unsigned)(i - lo) < width
                  r[i] = ((unsigned)(i - lo) < (unsigned)width) ? r[i] : 0xff800000u;
                tmem_st_x32(tS + k0, r);
              }
              stored = true;
            }
            if (stored) tmem_wait_st();
          }
        }
        MLXP_TR(wq == 0 && lane == 0, t, it, 5);
        float s[128];
        {
          uint32_t ra[32], rb[32];
          tmem_ld_x32(tS + 0, ra);
          tmem_ld_x32(tS + 32, rb);
          tmem_wait_ld();
          reg_fence(ra);
          reg_fence(rb);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            s[c] = __uint_as_float(ra[c]);
            s[32 + c] = __uint_as_float(rb[c]);
          }
          tmem_ld_x32(tS + 64, ra);
          tmem_ld_x32(tS + 96, rb);
          tmem_wait_ld();
          reg_fence(ra);
          reg_fence(rb);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            s[64 + c] = __uint_as_float(ra[c]);
            s[96 + c] = __uint_as_float(rb[c]);
          }
        }
        if constexpr (kBias) {
          // additive bias (the custom mask of gqa/mqa attention), in units of the raw q.k so
          // that everything below is unchanged; columns past Skv stay -inf
          if (qrow < p.Sq) {
            const float* br = p.bias + (long long)w.b * p.bias_sb + (long long)w.h * p.bias_sh +
                              (long long)qrow * p.bias_sq + (long long)j * C::BN;
            const float isc = p.inv_scale;
            if ((long long)(j + 1) * C::BN <= p.Skv) {
#pragma unroll
              for (int c = 0; c < C::BN / 4; ++c) {
                const float4 b4 = __ldg(reinterpret_cast<const float4*>(br) + c);
                s[4 * c] += b4.x * isc;
                s[4 * c + 1] += b4.y * isc;
                s[4 * c + 2] += b4.z * isc;
                s[4 * c + 3] += b4.w * isc;
              }
            } else {
              const int nvalid = p.Skv - j * C::BN;
#pragma unroll
              for (int c = 0; c < C::BN; ++c)
                if (c < nvalid) s[c] += __ldg(br + c) * isc;
            }
          }
        }
        // row max: 3-input max, four independent chains
        float mx0 = max3(s[0], s[1], s[2]), mx1 = max3(s[3], s[4], s[5]);
        float mx2 = max3(s[6], s[7], s[8]), mx3 = max3(s[9], s[10], s[11]);
#pragma unroll
        for (int c = 12; c < 124; c += 8) {
          mx0 = max3(mx0, s[c], s[c + 1]);
          mx1 = max3(mx1, s[c + 2], s[c + 3]);
          mx2 = max3(mx2, s[c + 4], s[c + 5]);
          mx3 = max3(mx3, s[c + 6], s[c + 7]);
        }
        mx0 = max3(mx0, s[124], s[125]);
        mx1 = max3(mx1, s[126], s[127]);
        const float mloc = max3(mx0, mx1, fmaxf(mx2, mx3)) * sl2;
        MLXP_TR(wq == 0 && lane == 0, t, it, 2);
        const float m_new = fmaxf(m, mloc);
        const bool resc = m_new > m + 8.0f;
        float alpha = 1.f;
        if (resc) {
          alpha = ex2_approx(m - m_new);
          m = m_new;
        }
        const float neg_mu = (m == -INFINITY) ? 0.f : -m;
        // p = 2^(s * scale * log2(e) - m): kPolyPerOct of every 8 column pairs on the FMA
        // pipe (exp2_poly2), the rest on the MUFU unit, so neither unit limits the row.
        const float2 sl2v = make_float2(sl2, sl2), negm = make_float2(neg_mu, neg_mu);
        float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t pk[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float2 x =
                fma2(make_float2(s[64 * hf + 2 * c], s[64 * hf + 2 * c + 1]), sl2v, negm);
            float2 e;
            if ((c & 7) < kPolyPerOct<D>) {
              e = exp2_poly2(x);
            } else {
              e.x = ex2_approx(x.x);
              e.y = ex2_approx(x.y);
            }
            if (c & 1)
              acc1 = add2(acc1, e);
            else
              acc0 = add2(acc0, e);
            pk[c] = pack2<kBF16>(e.x, e.y);
          }
          tmem_st_x32(tS + 32 * hf, pk);
        }
        MLXP_TR(wq == 0 && lane == 0, t, it, 3);
        if (it > 0 && __any_sync(0xffffffffu, resc)) {
          // O_t holds PV_t(j-1) (complete: it was issued before QK_t(j), whose commit we
          // saw); PV_t(j) is not issued before the arrive below, so it sees the rescaled O.
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t ov[32];
            tmem_ld_x32(tO + c * 32, ov);
            tmem_wait_ld();
            reg_fence(ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tmem_st_x32(tO + c * 32, ov);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(BAR(C::B_PF + t));
        MLXP_TR(wq == 0 && lane == 0, t, it, 4);
        l = l * alpha + ((acc0.x + acc1.x) + (acc0.y + acc1.y));
      }
      // The 128 threads of the tile go on together or not at all: a wait that gave up in one
      // warp must not leave the others at the epilogue's barriers.  (A warp that left the loop
      // early raised the abort flag, so the others' waits return at once.)
      ok = named_bar_and(1 + t, 128, ok);
      if (!ok) break;

      // ------------------------------------ epilogue ------------------------------------
      const bool has_rows = qrow < p.Sq;
      const int n_it = thi - tlo;
      // Key splits: the splits whose key tiles reach this query tile are [s_first, s_first +
      // nparts).  With one of them (or none: split 0 then writes the empty rows) the item
      // writes O directly; with more, each writes its partial and the one that completes the
      // tile's count merges them all.  A split that does not reach the tile writes nothing.
      // (Every quantity here is the same for the 128 threads of the tile.)
      int nparts = 1, s_first = 0;
      if (p.splits > 1) {
        int ulo = 0, uhi = 0;
        if (r1 > r0) kv_tile_range(p.mask, r0, r1, C::BN, ulo, uhi);
        s_first = ulo / p.tiles_per_split;
        nparts = (uhi > ulo) ? (uhi - 1) / p.tiles_per_split - s_first + 1 : 0;
        if (nparts == 0 ? w.split != 0 : n_it == 0) continue;
      }
      if (p.accumulate && n_it == 0) continue;  // no key of this range reaches the tile
      // The row's constants, computed while the last PV_t runs.  A row that never saw an
      // admissible key keeps m = -inf: it is empty (O = 0, LSE = -inf) even though the
      // polynomial exp2 leaves ~2^-125 per masked element in l.
      const bool valid = n_it > 0 && l > 0.f && m != -INFINITY;
      const float inv_l = valid ? 1.0f / l : 0.f;
      const float lse_v = valid ? (m + log2f(l)) * 0.69314718055994531f : -INFINITY;
      const bool elected = (wq == 0 && lane == 0);
      const long long tile_id = (long long)(w.b * p.H + w.h) * p.n_qtile + (w.q0 >> 7) + t;
      if (n_it > 0) {
        ok = mbar_wait(BAR(C::B_OF + t), n_o & 1, wctx, kSiteSoftmaxO);
        ok = named_bar_and(1 + t, 128, ok);
        if (!ok) break;
        ++n_o;
        tc_fence_after();
      }
      MLXP_TR(wq == 0 && lane == 0 && n_it > 0, t, n_it - 1, 6);
      bool merge = false;
      if (nparts >= 2 && tile_id >= p.part_tiles) {
        // the workspace does not cover this tile (a host-side sizing error): report, write nothing
        if (elected) atomicCAS(p.status, 0, kDevWorkspace | (kSiteEpilogue << 8));
        continue;
      }
      if (nparts >= 2) {
        // this split's partial: normalised O and LSE, rows interleaved by 16-byte chunks
        float* po = p.part_o + (tile_id * p.splits + w.split) * (128LL * D) + row * 4;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ov[32];
          tmem_ld_x32(tO + c * 32, ov);
          tmem_wait_ld();
          reg_fence(ov);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4*>(po + (c * 8 + i) * 128 * 4) = make_float4(
                __uint_as_float(ov[4 * i]) * inv_l, __uint_as_float(ov[4 * i + 1]) * inv_l,
                __uint_as_float(ov[4 * i + 2]) * inv_l, __uint_as_float(ov[4 * i + 3]) * inv_l);
        }
        p.part_lse[(tile_id * p.splits + w.split) * 128 + row] = lse_v;
        // publish: every thread's stores reach the device scope before the count moves
        __threadfence();
        named_bar_sync(1 + t, 128);
        if (elected) {
          const unsigned prev = atomicAdd(p.tile_cnt + tile_id, 1u);
          const int last = prev == (unsigned)(nparts - 1);
          if (last) {
            p.tile_cnt[tile_id] = 0u;  // every split of the tile has counted: ready for reuse
            __threadfence();
          }
          merge_flag[t] = last;
        }
        named_bar_sync(1 + t, 128);
        merge = merge_flag[t] != 0;
        if (!merge) continue;
      }
      // The merge: w_s = exp(lse_s - max lse) / sum of them; O = sum_s w_s O_s; LSE = max +
      // log(sum).  Partials are read through L2 (ld.global.cg): other SMs wrote them.
      const float* pl = p.part_lse + (tile_id * p.splits + s_first) * 128 + row;
      const float* pb = p.part_o + (tile_id * p.splits + s_first) * (128LL * D) + row * 4;
      float m_tot = -INFINITY, inv_w = 0.f, lse_out = lse_v;
      if (merge) {
        for (int s = 0; s < nparts; ++s) m_tot = fmaxf(m_tot, __ldcg(pl + s * 128));
        float wsum = 0.f;
        if (m_tot != -INFINITY)
          for (int s = 0; s < nparts; ++s) wsum += expf(__ldcg(pl + s * 128) - m_tot);
        inv_w = wsum > 0.f ? 1.0f / wsum : 0.f;
        lse_out = wsum > 0.f ? m_tot + logf(wsum) : -INFINITY;
      }
      // accumulate: weights of the running result and of this one (LSE form of the merge)
      float a_old = 0.f, a_new = 1.f;
      const float* acc_row = nullptr;
      if (p.accumulate && has_rows) {
        const float lse_old = p.lse[((long long)w.b * p.H + w.h) * p.Sq + qrow];
        const float mm = fmaxf(lse_old, lse_v);
        if (mm == -INFINITY) {  // neither has an admissible key: an empty row (O = 0)
          a_old = 0.f;
          a_new = 0.f;
          lse_out = -INFINITY;
        } else {
          const float w_old = lse_old == -INFINITY ? 0.f : expf(lse_old - mm);
          const float w_new = lse_v == -INFINITY ? 0.f : expf(lse_v - mm);
          const float wsum = w_old + w_new;
          a_old = w_old / wsum;
          a_new = w_new / wsum;
          lse_out = mm + logf(wsum);
        }
        if (a_old != 0.f)
          acc_row = p.acc_o + (long long)w.b * p.acc_sb + (long long)w.h * p.acc_sh +
                    (long long)qrow * p.acc_ss;
      }
      if (has_rows && p.lse != nullptr)
        p.lse[((long long)w.b * p.H + w.h) * p.Sq + qrow] = lse_out;
      // O leaves through the tile's staging box: each thread writes its row (128-byte swizzle:
      // 16-byte chunk k of row r at chunk k ^ (r % 8), which spreads a warp's writes over all
      // banks), then one thread stores the box with TMA, which writes whole lines of O (rows
      // past Sq are clipped by the tensor map).  A box is 64 bf16/fp16 or 32 fp32 columns, so
      // one 32-column chunk of O fills half a box (bf16/fp16) or a whole one (fp32).
      {
        const uint32_t stage = sbase + C::OFF_STAGE + t * C::STAGE_BYTES;
        const uint32_t row_base = stage + (uint32_t)row * 128u;
        const uint32_t sw = (uint32_t)(row & 7);
        const bool f32 = p.out_f32 != 0;
        int c1, c2, c3;
        tma_coords(p.co, w.q0 + t * 128, w.h, w.b, c1, c2, c3);
        // The common case (this item's O alone, bf16/fp16 out): one 64-column box at a time,
        // both of its TMEM loads under one wait (a load + wait measured 250-550 cycles here,
        // while the next item's MMAs run).
        const bool fast = !merge && n_it > 0 && !f32 && acc_row == nullptr;
        if (fast) {
          const float f = inv_l * a_new;
#pragma unroll 1
          for (int hb = 0; hb < D / 64; ++hb) {
            uint32_t ua[32], ub[32];
            tmem_ld_x32(tO + hb * 64, ua);
            tmem_ld_x32(tO + hb * 64 + 32, ub);
            tmem_wait_ld();
            reg_fence(ua);
            reg_fence(ub);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              ua[i] = pack2<kBF16>(__uint_as_float(ua[2 * i]) * f, __uint_as_float(ua[2 * i + 1]) * f);
              ub[i] = pack2<kBF16>(__uint_as_float(ub[2 * i]) * f, __uint_as_float(ub[2 * i + 1]) * f);
            }
            if (elected) bulk_wait_group_read0();  // the box's previous store has read it
            named_bar_sync(1 + t, 128);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              st_shared_v4(row_base + ((((uint32_t)k) ^ sw) << 4), ua[4 * k], ua[4 * k + 1],
                           ua[4 * k + 2], ua[4 * k + 3]);
              st_shared_v4(row_base + ((((uint32_t)(k + 4)) ^ sw) << 4), ub[4 * k], ub[4 * k + 1],
                           ub[4 * k + 2], ub[4 * k + 3]);
            }
            fence_proxy_async_smem();
            named_bar_sync(1 + t, 128);
            if (elected) {
              tma_store_4d(&tm_o, stage, hb * 64, c1, c2, c3);
              bulk_commit_group();
            }
          }
        }
#pragma unroll 1
        for (int c = 0; c < (fast ? 0 : D / 32); ++c) {
          float ov[32];
          if (merge) {
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = 0.f;
#pragma unroll 1
            for (int s = 0; s < nparts; ++s) {
              const float ls = __ldcg(pl + s * 128);
              const float ws = (ls == -INFINITY) ? 0.f : expf(ls - m_tot) * inv_w;
              const float* ps = pb + s * (128LL * D) + c * 8 * 128 * 4;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float4 v4 = __ldcg(reinterpret_cast<const float4*>(ps + i * 128 * 4));
                ov[4 * i] += ws * v4.x;
                ov[4 * i + 1] += ws * v4.y;
                ov[4 * i + 2] += ws * v4.z;
                ov[4 * i + 3] += ws * v4.w;
              }
            }
          } else if (n_it > 0) {
            uint32_t ou[32];
            tmem_ld_x32(tO + c * 32, ou);
            tmem_wait_ld();
            reg_fence(ou);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = __uint_as_float(ou[i]) * (inv_l * a_new);
            if (acc_row != nullptr) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float4 o4 = *reinterpret_cast<const float4*>(acc_row + c * 32 + 4 * i);
                ov[4 * i] += a_old * o4.x;
                ov[4 * i + 1] += a_old * o4.y;
                ov[4 * i + 2] += a_old * o4.z;
                ov[4 * i + 3] += a_old * o4.w;
              }
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = 0.f;
          }
          if (f32 || !(c & 1)) {
            // the previous store from this box has finished reading it
            if (elected) bulk_wait_group_read0();
            named_bar_sync(1 + t, 128);
          }
          if (f32) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              st_shared_v4(row_base + ((((uint32_t)i) ^ sw) << 4), __float_as_uint(ov[4 * i]),
                           __float_as_uint(ov[4 * i + 1]), __float_as_uint(ov[4 * i + 2]),
                           __float_as_uint(ov[4 * i + 3]));
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t k = (uint32_t)((c & 1) * 4 + i);
              st_shared_v4(row_base + ((k ^ sw) << 4), pack2<kBF16>(ov[8 * i + 0], ov[8 * i + 1]),
                           pack2<kBF16>(ov[8 * i + 2], ov[8 * i + 3]),
                           pack2<kBF16>(ov[8 * i + 4], ov[8 * i + 5]),
                           pack2<kBF16>(ov[8 * i + 6], ov[8 * i + 7]));
            }
          }
          if (f32 || (c & 1)) {
            fence_proxy_async_smem();
            named_bar_sync(1 + t, 128);
            if (elected) {
              tma_store_4d(&tm_o, stage, f32 ? c * 32 : (c >> 1) * 64, c1, c2, c3);
              bulk_commit_group();
            }
          }
        }
      }
      MLXP_TR(wq == 0 && lane == 0 && n_it > 0, t, n_it - 1, 7);
#if MLXP_TRACE
      if (t == 1 && wq == 0 && lane == 0 && idx < 8192)
        g_mlxp_cta_trace[idx * 4 + 1] = (long long)global_timer_ns();
#endif
    }
    // every TMA store of O has completed before the CTA (and its staging smem) goes away
    if (wq == 0 && lane == 0) bulk_wait_group0();
    tc_fence_before();
    __syncthreads();  // teardown barrier (pairs with the control warpgroup's)
#if MLXP_TRACE
    if (threadIdx.x == 0 && blockIdx.x < 1024) g_mlxp_cta_life[blockIdx.x * 3 + 2] = (long long)global_timer_ns();
#endif
    // The last CTA to finish resets the launch's work counter for the next launch.
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(p.work_counter + 1, 1u) == gridDim.x - 1) {
        atomicExch(p.work_counter, 0u);
        atomicExch(p.work_counter + 1, 0u);
        __threadfence();
      }
    }
  }
}

}  // namespace mlxp
