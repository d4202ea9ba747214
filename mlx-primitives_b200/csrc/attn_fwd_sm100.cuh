// attn_fwd_sm100.cuh — bf16/fp16 attention forward on the 5th-generation tensor cores (sm_100a).
//
// One CTA computes 256 query rows (two 128-row Q tiles, "tile 0" and "tile 1") of one
// (batch, head) against a range of 128-key K/V tiles:
//
//   warp 9        TMA producer: Q once, then K and V tiles into two smem rings (128B swizzle).
//   warp 8        MMA issuer (one thread): S_t = Q_t K^T (SS form, fp32 accumulate in TMEM),
//                 then O_t += P_t V (TS form: P_t read from TMEM, V from smem).
//   warps 0-3     softmax for tile 0, warps 4-7 softmax for tile 1: one thread owns one query
//                 row (TMEM lane), reads its 128 scores with tcgen05.ld, masks boundary tiles,
//                 updates the running max/sum, writes P (bf16/fp16, packed two per 32-bit
//                 column) back over the S columns with tcgen05.st, and rescales O in TMEM only
//                 when the running max grew by more than 2^8 (exact: the final 1/l uses the
//                 same stale max as the exponentials).  The same warps run the epilogue.
//
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D); P_t aliases
// the first 64 columns of S_t.  The two tiles ping-pong: while softmax works on S_0 the tensor
// core runs PV_1 / QK_1 and vice versa.  The MMA issue order per tile is PV_t(j), QK_t(j+1):
// tcgen05.mma instructions from one thread execute in order, so QK_t(j+1) may overwrite the
// S/P columns right after PV_t(j) is issued, and the commit after QK_t(j+1) also certifies that
// PV_t(j) finished — which is what lets the softmax warps rescale O without another barrier.
//
// Every wait is bounded (mbar_wait); when one gives up the CTA drains its in-flight TMA
// loads and MMAs (bounded again), frees TMEM and returns, leaving the error in the device
// status word.
#pragma once

#include "attn_common.cuh"
#include "sm100_ptx.cuh"

namespace mlxp {

template <int D, int NSK, int NSV>
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
  static constexpr int OFF_V = OFF_K + NSK * KV_TILE;
  static constexpr int OFF_BAR = OFF_V + NSV * KV_TILE;
  // barrier indices
  static constexpr int B_Q = 0;
  static constexpr int B_KF = 1;
  static constexpr int B_KE = B_KF + NSK;
  static constexpr int B_VF = B_KE + NSK;
  static constexpr int B_VE = B_VF + NSV;
  static constexpr int B_SF = B_VE + NSV;  // 2: S_t ready
  static constexpr int B_PF = B_SF + 2;    // 2: P_t ready (128 arrivals)
  static constexpr int B_OF = B_PF + 2;    // 2: final PV_t complete
  static constexpr int B_DR = B_OF + 2;    // 1: MMA drain
  static constexpr int NBAR = B_DR + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to align the base to 1024 B
  // Three warpgroups: WG0/WG1 softmax (tiles 0/1), WG2 = MMA warp, TMA warp, two spare warps.
  // Registers are split per SM sub-partition, so the launch gets 65536/384 -> 168 per thread
  // and setmaxnreg moves them to the softmax warpgroups: 2*128*208 + 128*80 = 63488 <= 384*168.
  static constexpr int THREADS = 384;
  static constexpr int REGS_SOFTMAX = 208;
  static constexpr int REGS_CONTROL = 80;
  static_assert(2 * 128 * REGS_SOFTMAX + 128 * REGS_CONTROL <= THREADS * 168, "register split");
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
  kSiteSelfTest = 7
};

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

template <int D, bool kBF16, int NSK, int NSV>
__global__ void __launch_bounds__(384, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  using C = Sm100Cfg<D, NSK, NSV>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + C::OFF_MISC + 4);
  auto BAR = [&](int i) -> uint32_t { return sbase + C::OFF_BAR + 8 * i; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work item: (b, h) major so that CTAs sharing K/V run together (L2 reuse); within a
  // (b, h), the heaviest query block first when the mask is causal.
  const int per_bh = p.n_qblk * p.splits;
  const int bh = blockIdx.x / per_bh;
  const int rem = blockIdx.x - bh * per_bh;
  const int split = rem % p.splits;
  int qb = rem / p.splits;
  if (p.heavy_first) qb = p.n_qblk - 1 - qb;
  const int h = bh % p.H;
  const int b = bh / p.H;
  const int q0 = qb * 256;

  int lo_t[2], hi_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const long long r0 = q0 + t * 128;
    const long long r1 = (r0 + 128 < p.Sq) ? r0 + 128 : p.Sq;
    kv_tile_range(p.mask, r0, r1, C::BN, lo_t[t], hi_t[t]);
    if (p.splits > 1) {
      const int s_lo = split * p.tiles_per_split, s_hi = s_lo + p.tiles_per_split;
      if (lo_t[t] < s_lo) lo_t[t] = s_lo;
      if (hi_t[t] > s_hi) hi_t[t] = s_hi;
      if (hi_t[t] < lo_t[t]) hi_t[t] = lo_t[t];
    }
  }
  const bool act0 = hi_t[0] > lo_t[0], act1 = hi_t[1] > lo_t[1];
  int lo = 0, hi = 0;
  if (act0 && act1) {
    lo = min(lo_t[0], lo_t[1]);
    hi = max(hi_t[0], hi_t[1]);
  } else if (act0) {
    lo = lo_t[0];
    hi = hi_t[0];
  } else if (act1) {
    lo = lo_t[1];
    hi = hi_t[1];
  }
  const int n_tiles = hi - lo;

  if (threadIdx.x == 0) {
    mbar_init(BAR(C::B_Q), 1);
    for (int i = 0; i < NSK; ++i) {
      mbar_init(BAR(C::B_KF + i), 1);
      mbar_init(BAR(C::B_KE + i), 1);
    }
    for (int i = 0; i < NSV; ++i) {
      mbar_init(BAR(C::B_VF + i), 1);
      mbar_init(BAR(C::B_VE + i), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(BAR(C::B_SF + t), 1);
      mbar_init(BAR(C::B_PF + t), 128);
      mbar_init(BAR(C::B_OF + t), 1);
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
  if (warp >= 8) {
    // ================================ control warpgroup ================================
    setmaxnreg_dec<C::REGS_CONTROL>();
    if (warp == 9) {
    // =================================== TMA producer ===================================
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const uint32_t sQ = sbase + C::OFF_Q, sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
      int c1, c2, c3;
      mbar_arrive_expect_tx(BAR(C::B_Q), (act0 + act1) * C::Q_TILE);
      for (int t = 0; t < 2; ++t) {
        if (!(t ? act1 : act0)) continue;
        tma_coords(p.cq, q0 + t * 128, h, b, c1, c2, c3);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_4d(sQ + t * C::Q_TILE + kb * C::BOX_Q, &tm_q, BAR(C::B_Q), kb * 64, c1, c2,
                      c3);
      }
      int issued_k = 0, issued_v = 0;
      bool ok = true;
      for (int f = 0; f < n_tiles && ok; ++f) {
        const int j = lo + f;
        const int ks = f % NSK;
        if (f >= NSK) ok = mbar_wait(BAR(C::B_KE + ks), ((f / NSK) - 1) & 1, wctx, kSiteProducer);
        if (!ok) break;
        mbar_arrive_expect_tx(BAR(C::B_KF + ks), C::KV_TILE);
        tma_coords(p.ck, j * C::BN, h, b, c1, c2, c3);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_4d(sK + ks * C::KV_TILE + kb * C::BOX_KV, &tm_k, BAR(C::B_KF + ks), kb * 64,
                      c1, c2, c3);
        issued_k = f + 1;
        const int vs = f % NSV;
        if (f >= NSV) ok = mbar_wait(BAR(C::B_VE + vs), ((f / NSV) - 1) & 1, wctx, kSiteProducer);
        if (!ok) break;
        mbar_arrive_expect_tx(BAR(C::B_VF + vs), C::KV_TILE);
        tma_coords(p.cv, j * C::BN, h, b, c1, c2, c3);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_4d(sV + vs * C::KV_TILE + kb * C::BOX_KV, &tm_v, BAR(C::B_VF + vs), kb * 64,
                      c1, c2, c3);
        issued_v = f + 1;
      }
      if (!ok) {
        // Abort: let every load already issued land before the CTA releases its smem.
        mbar_wait_drain(BAR(C::B_Q), 0, p.status, p.timeout_ns);
        for (int f = (issued_k > NSK ? issued_k - NSK : 0); f < issued_k; ++f)
          mbar_wait_drain(BAR(C::B_KF + f % NSK), (f / NSK) & 1, p.status, p.timeout_ns);
        for (int f = (issued_v > NSV ? issued_v - NSV : 0); f < issued_v; ++f)
          mbar_wait_drain(BAR(C::B_VF + f % NSV), (f / NSV) & 1, p.status, p.timeout_ns);
      }
    }
  } else if (warp == 8) {
    // ==================================== MMA issuer ====================================
    if (lane == 0 && n_tiles > 0) {
      const uint32_t sQ = sbase + C::OFF_Q, sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
      constexpr uint32_t idesc_qk = make_idesc_f16(128, C::BN, kBF16, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(128, D, kBF16, true);
      auto issue_qk = [&](int t, int ks) {
        const uint32_t d = tmem + (t ? C::TM_S1 : C::TM_S0);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad =
                make_sdesc_sw128(sQ + t * C::Q_TILE + kb * C::BOX_Q + kk * 32, 16, 1024);
            const uint64_t bd =
                make_sdesc_sw128(sK + ks * C::KV_TILE + kb * C::BOX_KV + kk * 32, 16, 1024);
            mma_ss(d, ad, bd, idesc_qk, (kb | kk) ? 1u : 0u);
          }
        }
      };
      auto issue_pv = [&](int t, int vs, bool acc) {
        const uint32_t d = tmem + (t ? C::TM_O1 : C::TM_O0);
        const uint32_t a = tmem + (t ? C::TM_S1 : C::TM_S0);
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk) {
          const uint64_t bd =
              make_sdesc_sw128(sV + vs * C::KV_TILE + kk * 16 * 128, C::BOX_KV, 1024);
          mma_ts(d, a + kk * 8, bd, idesc_pv, (acc || kk > 0) ? 1u : 0u);
        }
      };
      auto active = [&](int t, int j) { return j >= lo_t[t] && j < hi_t[t]; };

      int pcount[2] = {0, 0};
      bool ok = mbar_wait(BAR(C::B_Q), 0, wctx, kSiteMmaLoad);
      if (ok) ok = mbar_wait(BAR(C::B_KF + 0), 0, wctx, kSiteMmaLoad);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if (active(t, lo)) {
            issue_qk(t, 0);
            tc_commit(BAR(C::B_SF + t));
          }
        tc_commit(BAR(C::B_KE + 0));
      }
      for (int f = 0; f < n_tiles && ok; ++f) {
        const int j = lo + f;
        const int vs = f % NSV;
        const bool has_next = f + 1 < n_tiles;
        const int ksn = (f + 1) % NSK;
        bool k_ready = false;
        ok = mbar_wait(BAR(C::B_VF + vs), (f / NSV) & 1, wctx, kSiteMmaLoad);
        if (!ok) break;
        tc_fence_after();
        for (int t = 0; t < 2 && ok; ++t) {
          if (active(t, j)) {
            ok = mbar_wait(BAR(C::B_PF + t), pcount[t] & 1, wctx, kSiteMmaP);
            if (!ok) break;
            ++pcount[t];
            tc_fence_after();
            issue_pv(t, vs, j > lo_t[t]);
            if (j == hi_t[t] - 1) tc_commit(BAR(C::B_OF + t));
          }
          if (has_next && active(t, j + 1)) {
            if (!k_ready) {
              ok = mbar_wait(BAR(C::B_KF + ksn), ((f + 1) / NSK) & 1, wctx, kSiteMmaLoad);
              if (!ok) break;
              tc_fence_after();
              k_ready = true;
            }
            issue_qk(t, ksn);
            tc_commit(BAR(C::B_SF + t));
          }
        }
        if (!ok) break;
        tc_commit(BAR(C::B_VE + vs));
        if (has_next) {
          if (!k_ready) {  // neither tile uses this key tile: consume it anyway
            ok = mbar_wait(BAR(C::B_KF + ksn), ((f + 1) / NSK) & 1, wctx, kSiteMmaLoad);
            if (!ok) break;
          }
          tc_commit(BAR(C::B_KE + ksn));
        }
      }
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
    const int qrow = q0 + t * 128 + row;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + (t ? C::TM_S1 : C::TM_S0);
    const uint32_t tO = tmem + lane_off + (t ? C::TM_O1 : C::TM_O0);
    const int tlo = lo_t[t], thi = hi_t[t];
    const long long r0 = q0 + t * 128;
    const long long r1 = (r0 + 128 < p.Sq) ? r0 + 128 : p.Sq;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;

    for (int it = 0; it < thi - tlo; ++it) {
      const int j = tlo + it;
      ok = mbar_wait(BAR(C::B_SF + t), it & 1, wctx, kSiteSoftmaxS);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t r0v[32], r1v[32], r2v[32], r3v[32];
      tmem_ld_x32(tS + 0, r0v);
      tmem_ld_x32(tS + 32, r1v);
      tmem_ld_x32(tS + 64, r2v);
      tmem_ld_x32(tS + 96, r3v);
      tmem_wait_ld();
      reg_fence(r0v);
      reg_fence(r1v);
      reg_fence(r2v);
      reg_fence(r3v);
      float s[128];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        s[c] = __uint_as_float(r0v[c]);
        s[32 + c] = __uint_as_float(r1v[c]);
        s[64 + c] = __uint_as_float(r2v[c]);
        s[96 + c] = __uint_as_float(r3v[c]);
      }
      const long long c0 = (long long)j * C::BN;
      if (!tile_is_full(p.mask, r0, r1, c0, c0 + C::BN)) {
        int c_lo, c_hi;
        row_col_interval(p.mask, qrow, c0, C::BN, c_lo, c_hi);
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] = (c < c_lo || c > c_hi) ? -INFINITY : s[c];
      }
      float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
      for (int c = 4; c < 128; c += 4) {
        mx0 = fmaxf(mx0, s[c]);
        mx1 = fmaxf(mx1, s[c + 1]);
        mx2 = fmaxf(mx2, s[c + 2]);
        mx3 = fmaxf(mx3, s[c + 3]);
      }
      const float mloc = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
      const float m_new = fmaxf(m, mloc);
      const bool resc = m_new > m + 8.0f;
      float alpha = 1.f;
      if (resc) {
        alpha = ex2_approx(m - m_new);
        m = m_new;
      }
      const float neg_mu = (m == -INFINITY) ? 0.f : -m;
      float rs0 = 0.f, rs1 = 0.f;
      {
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float a0 = ex2_approx(fmaf(s[2 * c], sl2, neg_mu));
          const float a1 = ex2_approx(fmaf(s[2 * c + 1], sl2, neg_mu));
          rs0 += a0;
          rs1 += a1;
          pk[c] = pack2<kBF16>(a0, a1);
        }
        tmem_st_x32(tS + 0, pk);
      }
      {
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float a0 = ex2_approx(fmaf(s[64 + 2 * c], sl2, neg_mu));
          const float a1 = ex2_approx(fmaf(s[64 + 2 * c + 1], sl2, neg_mu));
          rs0 += a0;
          rs1 += a1;
          pk[c] = pack2<kBF16>(a0, a1);
        }
        tmem_st_x32(tS + 32, pk);
      }
      if (it > 0 && __any_sync(0xffffffffu, resc)) {
        // O_t holds PV_t(j-1) (complete: it was issued before QK_t(j), whose commit we saw);
        // PV_t(j) is not issued before the arrive below, so it sees the rescaled O.
#pragma unroll
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
      l = l * alpha + (rs0 + rs1);
    }

    // ------------------------------------ epilogue ------------------------------------
    const bool has_rows = qrow < p.Sq;
    const int n_it = thi - tlo;
    if (ok && n_it > 0) {
      ok = mbar_wait(BAR(C::B_OF + t), 0, wctx, kSiteSoftmaxO);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      if (n_it > 0) tc_fence_after();
      const float inv_l = (n_it > 0 && l > 0.f) ? 1.0f / l : 0.f;
      const float lse_v =
          (n_it > 0 && l > 0.f) ? (m + log2f(l)) * 0.69314718055994531f : -INFINITY;
      if (has_rows && p.lse != nullptr)
        p.lse[(long long)split * p.lse_split + ((long long)b * p.H + h) * p.Sq + qrow] = lse_v;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ov[32];
        if (n_it > 0) {
          tmem_ld_x32(tO + c * 32, ov);
          tmem_wait_ld();
          reg_fence(ov);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = 0u;
        }
        if (has_rows) {
          const long long off = (long long)split * p.o_split + (long long)b * p.o_sb +
                                (long long)h * p.o_sh + (long long)qrow * p.o_ss + c * 32;
          if (p.out_f32) {
            float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.o) + off);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_float4(__uint_as_float(ov[4 * i]) * inv_l,
                                   __uint_as_float(ov[4 * i + 1]) * inv_l,
                                   __uint_as_float(ov[4 * i + 2]) * inv_l,
                                   __uint_as_float(ov[4 * i + 3]) * inv_l);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.o) + off);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 w;
              w.x = pack2<kBF16>(__uint_as_float(ov[8 * i + 0]) * inv_l,
                                 __uint_as_float(ov[8 * i + 1]) * inv_l);
              w.y = pack2<kBF16>(__uint_as_float(ov[8 * i + 2]) * inv_l,
                                 __uint_as_float(ov[8 * i + 3]) * inv_l);
              w.z = pack2<kBF16>(__uint_as_float(ov[8 * i + 4]) * inv_l,
                                 __uint_as_float(ov[8 * i + 5]) * inv_l);
              w.w = pack2<kBF16>(__uint_as_float(ov[8 * i + 6]) * inv_l,
                                 __uint_as_float(ov[8 * i + 7]) * inv_l);
              dst[i] = w;
            }
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // teardown barrier (pairs with the control warpgroup's)
  }
}

}  // namespace mlxp
