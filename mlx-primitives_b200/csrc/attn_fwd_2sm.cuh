// attn_fwd_2sm.cuh — bf16/fp16 attention forward, head_dim 128, on CTA pairs with the 2-SM
// tensor-core MMA (tcgen05.mma.cta_group::2).
//
// A cluster of two CTAs (two SMs) takes one work item: 256 query rows of one (batch, head,
// key split) — CTA r of the pair owns rows 128 r .. 128 r + 127 — against a range of 128-key
// tiles.  The even CTA's MMA thread issues M=256 MMAs that span both SMs: each CTA keeps its
// own Q tile, S and O in its own shared memory / TMEM, and only HALF of every K and V tile
// (keys 64 r .. 64 r + 63 of K, head-dim columns 64 r .. 64 r + 63 of V), so per SM a key tile
// costs 32 KB of L2 -> shared-memory traffic instead of 64 KB.
//
// Per CTA, TMEM holds three S buffers and O: S0 [0,128) S1 [128,256) S2 [256,384) O [384,512).
// Key tile x of the item goes to S buffer (x mod 3) (counted across items); its P is written
// back over the first 32 columns of each 64-column half of that buffer.  With three buffers the
// MMA stream is a sequence of blocks, one per key tile x:
//     block x = PV(x) [O += P_x V_x, TS]  interleaved MMA by MMA with  QK(x+2) [S = Q K_{x+2}^T]
// (two independent accumulator chains: measured 64 cycles per M=256 K=16 MMA back to back, 72
// with one tcgen05.commit per block, against 107 for the ping-pong order of two 128-row tiles
// sharing two S buffers).  Blocks x = lo-2 and lo-1 issue only QK(lo), QK(lo+1); the last two
// blocks only PV.  One commit per block arrives on E[block mod 3] in BOTH CTAs; that single
// event means: S(x+2) is ready, PV(x) is done (O may be rescaled before PV(x+1)), and the
// block's K/V ring slot is free.
//
//   warps 0-7   softmax of this CTA's 128 rows: warps w and w+4 share TMEM lanes 32(w%4)..+31
//               (one thread per row) and take columns 0-63 / 64-127 of S; the two halves of a
//               row exchange their partial maxima through shared memory (a 64-thread named
//               barrier per step), so both use the same running max.  Lazy O rescale (only when
//               the max grows by more than 2^8), P packed to bf16/fp16 pairs, epilogue.
//   warp 8      even CTA: MMA issuer (one thread); both CTAs: TMEM allocation for the pair
//   warp 9      TMA producer of this CTA's Q tile and K/V halves; the even CTA's producer also
//               takes work items from the device counter and hands them to the odd CTA
//   warps 10-11 spare
//
// Barriers live in both CTAs; those the MMA thread waits on (QF, F, PF, WE) count arrivals and
// TMA bytes of both CTAs in the even CTA's copy.  Every wait is bounded.
//
// Status: opt-in (mlxp_set_forward_kernel(1)); the single-SM kernel is faster on every shape
// measured (config 2: 836 against ~1000 TFLOPS; config 3: 908 against ~1100; non-causal 16K:
// 856 against 1005).  With three S buffers the softmax of tile x+1 must finish within one MMA
// block (16 MMAs, ~1150 cycles), but a 128 x 128 softmax step takes ~2000 cycles here (two
// warps per row with a per-step max exchange; 1024 MUFU cycles per SM at best), and a pair
// finishes a 256-row item twice as fast as one SM, so item boundaries (O read-out, Q reload)
// come twice as often.  With the softmax arithmetic removed the kernel reaches ~1050 / ~1150
// TFLOPS on configs 2 / 3, so both limits would have to move for it to pay.
#pragma once

#include "attn_fwd_sm100.cuh"

namespace mlxp {

template <bool kBF16>
struct Fwd2SmCfg {
  static constexpr int D = 128, BM = 128, BN = 128;
  static constexpr int Q_TILE = BM * D * 2;        // 32 KB, two 64-column boxes
  static constexpr int BOX_Q = BM * 128;           // 16 KB
  static constexpr int K_HALF = (BN / 2) * D * 2;  // 16 KB: 64 keys, two boxes of 64 rows
  static constexpr int BOX_KH = (BN / 2) * 128;    // 8 KB
  static constexpr int V_HALF = BN * 64 * 2;       // 16 KB: 128 keys x 64 columns
  static constexpr int SLOT = K_HALF + V_HALF;     // one K/V ring slot
  // K/V ring depth: the loads of block x are issued when block x - NSLOT completes, and the
  // MMA thread wants them about NSLOT - 2 blocks plus one softmax step later
  static constexpr int NSLOT = 4;
  // One Q buffer: it is released by the commit of the item's last QK, two blocks before the
  // item ends, which leaves the next item's Q load two blocks to land
  static constexpr int NQ = 1;
  static constexpr int STAGE_BYTES = BM * 128;     // epilogue staging box, one per column half
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = OFF_Q + NQ * Q_TILE;
  static constexpr int OFF_STAGE = OFF_KV + NSLOT * SLOT;
  static constexpr int OFF_XM = OFF_STAGE + 2 * STAGE_BYTES;  // float [2 parity][2 half][128]
  static constexpr int OFF_XL = OFF_XM + 2 * 2 * 128 * 4;     // float [2 half][128]
  static constexpr int OFF_BAR = OFF_XL + 2 * 128 * 4;
  enum {
    B_QF = 0,               // NQ: Q buffer loaded (both CTAs' bytes, even CTA)
    B_QE = B_QF + NQ,       // NQ: Q buffer free (commit)
    B_F = B_QE + NQ,        // NSLOT: ring slot loaded (both CTAs' bytes, even CTA)
    B_E = B_F + NSLOT,      // NSLOT: block done (commit)
    B_PF = B_E + NSLOT,     // 2: P ready (16 warp arrivals, even CTA)
    B_OF = B_PF + 2,        // 1: the item's last PV done (commit)
    B_WF = B_OF + 1,        // 2: work slot filled
    B_WE = B_WF + 2,        // 2: work slot read (18 arrivals, even CTA)
    B_DR = B_WE + 2,        // 1: MMA drain
    NBAR = B_DR + 1
  };
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // tmem slot, abort flag, 2 item slots
  static constexpr int SMEM_BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
  static constexpr int THREADS = 384;
  static constexpr int REGS_SOFTMAX = 208;
  static constexpr int REGS_CONTROL = 80;
  static_assert(2 * 128 * REGS_SOFTMAX + 128 * REGS_CONTROL <= THREADS * 168, "register split");
  static constexpr int PF_ARRIVALS = 16;  // 8 softmax warps per CTA
  static constexpr int WE_ARRIVALS = 18;  // per CTA 8 softmax warps, + MMA thread, + producer
  static constexpr uint32_t TM_O = 384, TM_COLS = 512;
  static_assert(OFF_KV % 1024 == 0 && OFF_STAGE % 1024 == 0 && SLOT % 1024 == 0, "atoms");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

enum : int { kSite2Producer = 20, kSite2Mma = 21, kSite2Softmax = 22, kSite2Work = 23 };

// Of every 8 column pairs of a score row, this many are exponentiated with exp2_poly2 on the
// FMA pipe, the rest with ex2.approx on the MUFU unit (16 results per clock per SM: one tile of
// 128 x 128 scores needs 1024 MUFU cycles, as long as the 16 MMAs of a block).
#ifndef MLXP_POLY_2SM
#define MLXP_POLY_2SM 2
#endif
constexpr int kPoly2Sm = MLXP_POLY_2SM;

template <bool kBF16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(384, 1)
    attn_fwd_2sm_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_o, const FwdParams p) {
  using C = Fwd2SmCfg<kBF16>;
  constexpr int D = C::D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + C::OFF_MISC + 4);
  volatile int* work_slot = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8);
  auto BAR = [&](int i) -> uint32_t { return sbase + C::OFF_BAR + 8 * i; };
  const uint32_t rank = cluster_cta_rank();
  // the even CTA's copy of a barrier, as a shared::cluster address
  auto BAR0 = [&](int i) -> uint32_t { return mapa_shared(BAR(i), 0); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = p.n_qblk * p.B * p.H * p.splits;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NQ; ++i) {
      mbar_init(BAR(C::B_QF + i), 1);
      mbar_init(BAR(C::B_QE + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(BAR(C::B_PF + i), C::PF_ARRIVALS);
      mbar_init(BAR(C::B_WF + i), 1);
      mbar_init(BAR(C::B_WE + i), C::WE_ARRIVALS);
    }
    for (int i = 0; i < C::NSLOT; ++i) {
      mbar_init(BAR(C::B_F + i), 1);
      mbar_init(BAR(C::B_E + i), 1);
    }
    mbar_init(BAR(C::B_OF), 1);
    mbar_init(BAR(C::B_DR), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc_pair(smem_u32(tmem_slot), C::TM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx wctx{abort_flag, p.status, p.timeout_ns};

  if (warp >= 8) {
    // ================================ control warpgroup ================================
    setmaxnreg_dec<C::REGS_CONTROL>();
    if (warp == 9 && lane == 0) {
      // =================================== TMA producer ===================================
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_o);
      const uint32_t slot_peer = mapa_shared(smem_u32(const_cast<int*>(work_slot)), 1);
      int nb = 0, n_q = 0, issued_q = 0;
      bool ok = true;
      for (int item = 0; ok; ++item) {
        const int ws = item & 1;
        int idx;
        if (rank == 0) {
          if (item >= 2) {
            ok = mbar_wait_cluster(BAR(C::B_WE + ws), ((item >> 1) - 1) & 1, wctx, kSite2Work);
            if (!ok) break;
          }
          idx = (int)atomicAdd(p.work_counter, 1u);
          work_slot[ws] = idx;
          st_shared_cluster_u32(slot_peer + 4 * ws, (uint32_t)idx);
          mbar_arrive_cluster(mapa_shared(BAR(C::B_WF + ws), 0));
          mbar_arrive_cluster(mapa_shared(BAR(C::B_WF + ws), 1));
        } else {
          ok = mbar_wait_cluster(BAR(C::B_WF + ws), (item >> 1) & 1, wctx, kSite2Work);
          if (!ok) break;
          idx = work_slot[ws];
          mbar_arrive_cluster(BAR0(C::B_WE + ws));
        }
        if (idx >= n_items) break;
        const WorkItem w = decode_item(p, idx, C::BN);
        if (w.hi <= w.lo) continue;
#if MLXP_TRACE
        if (rank == 0 && idx < 8192) {
          uint32_t smid;
          asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
          g_mlxp_cta_trace[idx * 4 + 0] = (long long)global_timer_ns();
          g_mlxp_cta_trace[idx * 4 + 2] = smid;
          g_mlxp_cta_trace[idx * 4 + 3] = w.hi - w.lo;
        }
#endif
        int c1, c2, c3;
        const int qb = n_q % C::NQ;
        if (n_q >= C::NQ) {
          ok = mbar_wait(BAR(C::B_QE + qb), ((n_q / C::NQ) - 1) & 1, wctx, kSite2Producer);
          if (!ok) break;
        }
        if (rank == 0) mbar_arrive_expect_tx(BAR(C::B_QF + qb), 2 * C::Q_TILE);
        tma_coords(p.cq, w.q0 + 128 * (int)rank, w.h, w.b, c1, c2, c3);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
          tma_load_4d_pair(sbase + C::OFF_Q + qb * C::Q_TILE + kb * C::BOX_Q, &tm_q,
                           BAR0(C::B_QF + qb), kb * 64, c1, c2, c3);
        ++n_q;
        issued_q = n_q;
        const int hk = w.h / p.kv_group;
        const int n_blk = w.hi - w.lo + 2;
        for (int bi = 0; bi < n_blk && ok; ++bi) {
          const int x = w.lo - 2 + bi, g = nb + bi, s = g % C::NSLOT;
          if (g >= C::NSLOT) {
            ok = mbar_wait(BAR(C::B_E + s), ((g / C::NSLOT) - 1) & 1, wctx, kSite2Producer);
            if (!ok) break;
          }
          const bool has_qk = x + 2 < w.hi, has_pv = x >= w.lo;
          if (rank == 0) {
            const uint32_t bytes = (has_qk ? 2 * C::K_HALF : 0) + (has_pv ? 2 * C::V_HALF : 0);
            if (bytes) mbar_arrive_expect_tx(BAR(C::B_F + s), bytes);
            else mbar_arrive(BAR(C::B_F + s));
          }
          const uint32_t sl = sbase + C::OFF_KV + s * C::SLOT;
          if (has_qk) {
            tma_coords(p.ck, (x + 2) * C::BN + 64 * (int)rank, hk, w.b, c1, c2, c3);
#pragma unroll
            for (int kb = 0; kb < 2; ++kb)
              tma_load_4d_pair(sl + kb * C::BOX_KH, &tm_k, BAR0(C::B_F + s), kb * 64, c1, c2, c3);
          }
          if (has_pv) {
            tma_coords(p.cv, x * C::BN, hk, w.b, c1, c2, c3);
            tma_load_4d_pair(sl + C::K_HALF, &tm_v, BAR0(C::B_F + s), 64 * (int)rank, c1, c2, c3);
          }
        }
        nb += n_blk;
      }
      if (!ok && rank == 0) {
        // Abort: the loads of both CTAs count on this CTA's barriers; let every phase that
        // may still receive bytes complete (bounded) before the pair releases shared memory.
        if (issued_q > 0) {
          for (int q = (issued_q > C::NQ ? issued_q - C::NQ : 0); q < issued_q; ++q)
            mbar_wait_drain(BAR(C::B_QF + q % C::NQ), (q / C::NQ) & 1, p.status, p.timeout_ns);
        }
        for (int g = (nb > C::NSLOT ? nb - C::NSLOT : 0); g < nb; ++g)
          mbar_wait_drain(BAR(C::B_F + g % C::NSLOT), (g / C::NSLOT) & 1, p.status, p.timeout_ns);
      }
    } else if (warp == 8 && lane == 0 && rank == 0) {
      // ==================================== MMA issuer ====================================
      constexpr uint32_t id_qk = make_idesc_f16(256, C::BN, kBF16, false);
      constexpr uint32_t id_pv = make_idesc_f16(256, D, kBF16, true);
      const uint32_t q_lo = ((sbase + C::OFF_Q) >> 4) | (1u << 16);
      const uint32_t kv_lo = ((sbase + C::OFF_KV) >> 4) | (1u << 16);
      int nb = 0, ns = 0, np = 0, n_q = 0;
      bool ok = true;
      for (int item = 0; ok; ++item) {
        const int ws = item & 1;
        ok = mbar_wait_cluster(BAR(C::B_WF + ws), (item >> 1) & 1, wctx, kSite2Work);
        if (!ok) break;
        const int idx = work_slot[ws];
        mbar_arrive_cluster(BAR0(C::B_WE + ws));
        if (idx >= n_items) break;
        const WorkItem w = decode_item(p, idx, C::BN);
        if (w.hi <= w.lo) continue;
        const int qb = n_q % C::NQ;
        ok = mbar_wait_cluster(BAR(C::B_QF + qb), (n_q / C::NQ) & 1, wctx, kSite2Mma);
        if (!ok) break;
        ++n_q;
        const uint32_t qa = q_lo + (uint32_t)((qb * C::Q_TILE) >> 4);
        const int n_blk = w.hi - w.lo + 2;
        for (int bi = 0; bi < n_blk; ++bi) {
          const int x = w.lo - 2 + bi, g = nb + bi, s = g % C::NSLOT;
          const bool has_qk = x + 2 < w.hi, has_pv = x >= w.lo;
          MLXP_TR(true, 2, g, 0);
          ok = mbar_wait_cluster(BAR(C::B_F + s), (g / C::NSLOT) & 1, wctx, kSite2Mma);
          MLXP_TR(true, 2, g, 1);
          if (ok && has_pv) {
            ok = mbar_wait_cluster(BAR(C::B_PF + (np & 1)), (np >> 1) & 1, wctx, kSite2Mma);
            ++np;
          }
          MLXP_TR(true, 2, g, 2);
          if (!ok) break;
          tc_fence_after();
          const uint32_t s_pv = tmem + (uint32_t)(((ns + x - w.lo) % 3) * 128);
          const uint32_t s_qk = tmem + (uint32_t)(((ns + x + 2 - w.lo) % 3) * 128);
          const uint32_t ka = kv_lo + (uint32_t)((s * C::SLOT) >> 4);
          // V half: MN-major (head-dim columns contiguous), one 64-column chunk per CTA
          const uint32_t va = ka + (uint32_t)(C::K_HALF >> 4);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            if (has_pv)  // P of keys 16 kk .. 16 kk + 15: half kk / 4, packed column 8 (kk % 4)
              mma_ts_pair(tmem + C::TM_O, s_pv + (uint32_t)(64 * (kk >> 2) + 8 * (kk & 3)),
                          sdesc(va + (uint32_t)((kk * 16 * 128) >> 4)), id_pv,
                          (x > w.lo || kk > 0) ? 1u : 0u);
            if (has_qk)
              mma_ss_pair(s_qk, sdesc(qa + (uint32_t)(((kk >> 2) * C::BOX_Q + (kk & 3) * 32) >> 4)),
                          sdesc(ka + (uint32_t)(((kk >> 2) * C::BOX_KH + (kk & 3) * 32) >> 4)),
                          id_qk, kk > 0 ? 1u : 0u);
          }
          tc_commit_pair(BAR(C::B_E + s), 3);
          MLXP_TR(true, 2, g, 3);
          if (has_pv && x == w.hi - 1) tc_commit_pair(BAR(C::B_OF), 3);
          if (has_qk && x + 2 == w.hi - 1) tc_commit_pair(BAR(C::B_QE + qb), 3);
        }
        if (!ok) break;
        nb += n_blk;
        ns += w.hi - w.lo;
      }
      // every MMA issued by this thread completes before TMEM and shared memory are released
      tc_commit_pair(BAR(C::B_DR), 1);
      mbar_wait_drain(BAR(C::B_DR), 0, p.status, p.timeout_ns);
    }
    // warps 10-11 and the odd CTA's warp 8: spare
  } else {
    // ============================= softmax + epilogue (8 warps) =============================
    setmaxnreg_inc<C::REGS_SOFTMAX>();
    const int lg = warp & 3;  // TMEM lane group
    const int hc = warp >> 2;  // column half of S / O
    const int row = lg * 32 + lane;
    const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
    const uint32_t tO = tmem + lane_off + C::TM_O + 64 * hc;
    float* xm = reinterpret_cast<float*>(smem + C::OFF_XM);
    float* xl = reinterpret_cast<float*>(smem + C::OFF_XL);
    const float sl2 = p.scale_log2;
    const int pair_bar = 1 + lg;  // warps lg and lg + 4
    int nb = 0, ns = 0, np = 0, n_o = 0;
    bool ok = true;
    for (int item = 0; ok; ++item) {
      const int ws = item & 1;
      ok = mbar_wait_cluster(BAR(C::B_WF + ws), (item >> 1) & 1, wctx, kSite2Work);
      ok = named_bar_and(7, 256, ok);  // all softmax warps leave the item loop together
      if (!ok) break;
      const int idx = work_slot[ws];
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(BAR0(C::B_WE + ws));
      if (idx >= n_items) break;
      const WorkItem w = decode_item(p, idx, C::BN);
      const int tlo = rank ? w.lo1 : w.lo0, thi = rank ? w.hi1 : w.hi0;
      const long long r0 = w.q0 + 128 * (int)rank;
      const long long r1 = (r0 + 128 < p.Sq) ? r0 + 128 : p.Sq;
      const int qrow = (int)r0 + row;
      int flo = 0, fhi = 0;
      if (r1 > r0) full_tile_range(p.mask, r0, r1, C::BN, flo, fhi);
      float m = -INFINITY, l = 0.f;
      const int n_t = w.hi > w.lo ? w.hi - w.lo : 0;

      for (int it = 0; it < n_t; ++it) {
        const int x = w.lo + it;
        const int g = nb + it;  // block that computed S(x)
        MLXP_TR(lg == 0 && lane == 0, hc, np, 0);
        if (ok) ok = mbar_wait(BAR(C::B_E + g % C::NSLOT), (g / C::NSLOT) & 1, wctx, kSite2Softmax);
        MLXP_TR(lg == 0 && lane == 0, hc, np, 1);
        tc_fence_after();
        const uint32_t tS = tmem + lane_off + (uint32_t)(((ns + it) % 3) * 128) + 64 * hc;
        const bool in_range = x >= tlo && x < thi;  // uniform over the CTA
        float s[64];
        float mh = -INFINITY;
        if (ok && in_range) {
          if (x < flo || x >= fhi) {
            // boundary tile: mask this half's two 32-column chunks in TMEM first
            const long long c0 = (long long)x * C::BN;
            int c_lo, c_hi;
            row_col_interval(p.mask, qrow, c0, C::BN, c_lo, c_hi);
            const int lo_min = __reduce_min_sync(0xffffffffu, c_lo);
            const int lo_max = __reduce_max_sync(0xffffffffu, c_lo);
            const int hi_min = __reduce_min_sync(0xffffffffu, c_hi);
            const int hi_max = __reduce_max_sync(0xffffffffu, c_hi);
            const int width = (c_hi >= c_lo) ? c_hi - c_lo + 1 : 0;
            bool stored = false;
#pragma unroll 1
            for (int k = 0; k < 2; ++k) {
              const int k0 = 64 * hc + 32 * k, k1 = k0 + 31;
              if (lo_max <= k0 && hi_min >= k1) continue;
              if (hi_max < k0 || lo_min > k1) {
                tmem_fill_x32(tS + 32 * k, 0xff800000u);
              } else {
                uint32_t r[32];
                tmem_ld_x32(tS + 32 * k, r);
                tmem_wait_ld();
                reg_fence(r);
                const int lo = c_lo - k0;
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  r[i] = ((unsigned)(i - lo) < (unsigned)width) ? r[i] : 0xff800000u;
                tmem_st_x32(tS + 32 * k, r);
              }
              stored = true;
            }
            if (stored) tmem_wait_st();
          }
          uint32_t ra[32], rb[32];
          tmem_ld_x32(tS, ra);
          tmem_ld_x32(tS + 32, rb);
          tmem_wait_ld();
          reg_fence(ra);
          reg_fence(rb);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            s[c] = __uint_as_float(ra[c]);
            s[32 + c] = __uint_as_float(rb[c]);
          }
          float mx0 = max3(s[0], s[1], s[2]), mx1 = max3(s[3], s[4], s[5]);
          float mx2 = max3(s[6], s[7], s[8]), mx3 = max3(s[9], s[10], s[11]);
#pragma unroll
          for (int c = 12; c < 60; c += 8) {
            mx0 = max3(mx0, s[c], s[c + 1]);
            mx1 = max3(mx1, s[c + 2], s[c + 3]);
            mx2 = max3(mx2, s[c + 4], s[c + 5]);
            mx3 = max3(mx3, s[c + 6], s[c + 7]);
          }
          mx0 = max3(mx0, s[60], s[61]);
          mx1 = max3(mx1, s[62], s[63]);
          mh = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        }
        float* xmp = xm + (it & 1) * 256;
        xmp[hc * 128 + row] = mh;
        MLXP_TR(lg == 0 && lane == 0, hc, np, 2);
        ok = named_bar_and(pair_bar, 64, ok);  // the two halves of each row go on together
        MLXP_TR(lg == 0 && lane == 0, hc, np, 3);
        if (!ok) break;
        uint32_t pk[32];
        float alpha = 1.f;
        float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
        bool resc = false;
        if (in_range) {
          const float mloc = fmaxf(mh, xmp[(hc ^ 1) * 128 + row]) * sl2;
          const float m_new = fmaxf(m, mloc);
          resc = m_new > m + 8.0f;
          if (resc) {
            alpha = ex2_approx(m - m_new);
            m = m_new;
          }
          const float neg_mu = (m == -INFINITY) ? 0.f : -m;
          const float2 sl2v = make_float2(sl2, sl2), negm = make_float2(neg_mu, neg_mu);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float2 xv = fma2(make_float2(s[2 * c], s[2 * c + 1]), sl2v, negm);
            float2 e;
            if ((c & 7) < kPoly2Sm) {
              e = exp2_poly2(xv);
            } else {
              e.x = ex2_approx(xv.x);
              e.y = ex2_approx(xv.y);
            }
            if (c & 1)
              acc1 = add2(acc1, e);
            else
              acc0 = add2(acc0, e);
            pk[c] = pack2<kBF16>(e.x, e.y);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) pk[c] = 0u;
        }
        MLXP_TR(lg == 0 && lane == 0, hc, np, 4);
        tmem_st_x32(tS, pk);
        MLXP_TR(lg == 0 && lane == 0, hc, np, 6);
        if (in_range && x > tlo && __any_sync(0xffffffffu, resc) && ok) {
          // O holds PV(x-1) once block x-1 is done (its commit); PV(x) waits for our P.
          ok = mbar_wait(BAR(C::B_E + (g + 1) % C::NSLOT), ((g + 1) / C::NSLOT) & 1, wctx,
                         kSite2Softmax);
          if (ok) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
              uint32_t ov[32];
              tmem_ld_x32(tO + c * 32, ov);
              tmem_wait_ld();
              reg_fence(ov);
#pragma unroll
              for (int i = 0; i < 32; ++i)
                ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
              tmem_st_x32(tO + c * 32, ov);
            }
          }
        }
        tmem_wait_st();
        MLXP_TR(lg == 0 && lane == 0, hc, np, 7);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(BAR(C::B_PF + (np & 1)));
          else mbar_arrive_remote(BAR0(C::B_PF + (np & 1)));
        }
        MLXP_TR(lg == 0 && lane == 0, hc, np, 5);
        ++np;
        if (in_range) l = l * alpha + ((acc0.x + acc1.x) + (acc0.y + acc1.y));
      }
      if (n_t > 0) {
        nb += n_t + 2;
        ns += n_t;
      }
      // ------------------------------------ epilogue ------------------------------------
      if (ok && n_t > 0) {
        ok = mbar_wait(BAR(C::B_OF), n_o & 1, wctx, kSite2Softmax);
        ++n_o;
      }
      ok = named_bar_and(7, 256, ok);
      if (!ok) break;
      tc_fence_after();
      xl[hc * 128 + row] = l;
      named_bar_sync(pair_bar, 64);
      const float lt = xl[row] + xl[128 + row];
      const bool has_rows = qrow < p.Sq;
      const bool valid = thi > tlo && lt > 0.f && m != -INFINITY;
      const float inv_l = valid ? 1.0f / lt : 0.f;
      if (hc == 0 && has_rows && p.lse != nullptr)
        p.lse[(long long)w.split * p.lse_split + ((long long)w.b * p.H + w.h) * p.Sq + qrow] =
            valid ? (m + log2f(lt)) * 0.69314718055994531f : -INFINITY;
      // O of this half (64 columns) leaves through the half's staging box: one box of 64
      // bf16/fp16 columns, or two passes of 32 fp32 columns (split partials).
      const uint32_t stage = sbase + C::OFF_STAGE + hc * C::STAGE_BYTES;
      const uint32_t row_base = stage + (uint32_t)row * 128u;
      const uint32_t sw = (uint32_t)(row & 7);
      const bool elected = (lg == 0 && lane == 0);
      const bool f32 = p.out_f32 != 0;
      const int half_bar = 5 + hc;
      int c1, c2, c3;
      tma_coords(p.co, (int)r0, w.h, w.split * p.o_split_b + w.b, c1, c2, c3);
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t ov[32];
        if (n_t > 0) {
          tmem_ld_x32(tO + c * 32, ov);
          tmem_wait_ld();
          reg_fence(ov);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = 0u;
        }
        if (f32 || c == 0) {
          if (elected) bulk_wait_group_read0();  // the previous store has read the box
          named_bar_sync(half_bar, 128);
        }
        if (f32) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            st_shared_v4(row_base + ((((uint32_t)i) ^ sw) << 4),
                         __float_as_uint(__uint_as_float(ov[4 * i]) * inv_l),
                         __float_as_uint(__uint_as_float(ov[4 * i + 1]) * inv_l),
                         __float_as_uint(__uint_as_float(ov[4 * i + 2]) * inv_l),
                         __float_as_uint(__uint_as_float(ov[4 * i + 3]) * inv_l));
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t k = (uint32_t)(c * 4 + i);
            st_shared_v4(row_base + ((k ^ sw) << 4),
                         pack2<kBF16>(__uint_as_float(ov[8 * i + 0]) * inv_l,
                                      __uint_as_float(ov[8 * i + 1]) * inv_l),
                         pack2<kBF16>(__uint_as_float(ov[8 * i + 2]) * inv_l,
                                      __uint_as_float(ov[8 * i + 3]) * inv_l),
                         pack2<kBF16>(__uint_as_float(ov[8 * i + 4]) * inv_l,
                                      __uint_as_float(ov[8 * i + 5]) * inv_l),
                         pack2<kBF16>(__uint_as_float(ov[8 * i + 6]) * inv_l,
                                      __uint_as_float(ov[8 * i + 7]) * inv_l));
          }
        }
        if (f32 || c == 1) {
          fence_proxy_async_smem();
          named_bar_sync(half_bar, 128);
          if (elected) {
            tma_store_4d(&tm_o, stage, f32 ? 64 * hc + 32 * c : 64 * hc, c1, c2, c3);
            bulk_commit_group();
          }
        }
      }
#if MLXP_TRACE
      if (rank == 0 && hc == 0 && lg == 0 && lane == 0 && idx < 8192)
        g_mlxp_cta_trace[idx * 4 + 1] = (long long)global_timer_ns();
#endif
    }
    if (lg == 0 && lane == 0) bulk_wait_group0();  // every store of O has completed
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the other may still address its memory
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TM_COLS);
  }
  // the last CTA to finish resets the launch's work counter for the next launch
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.work_counter + 1, 1u) == gridDim.x - 1) {
      atomicExch(p.work_counter, 0u);
      atomicExch(p.work_counter + 1, 0u);
      __threadfence();
    }
  }
}

}  // namespace mlxp
