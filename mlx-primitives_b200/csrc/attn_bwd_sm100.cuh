// attn_bwd_sm100.cuh — attention backward (dQ, dK, dV) on the 5th-generation tensor cores,
// head_dim 128, bf16/fp16 inputs, fp32 accumulation in TMEM.
//
// One CTA per (key tile of 128 keys, batch, K/V head); it keeps K_j and V_j in shared memory
// and dK_j, dV_j in TMEM while it walks the 64-row query tiles (of every query head of a
// grouped K/V head) that see the tile.  With the forward's log-sum-exp (as L2 = L * log2(e))
// and Delta = rowsum(dO * O) prepared by bwd_tc_prep_kernel, one step (query tile i) is
//   S^T  = K Q_i^T          (SS, M 128 keys x N 64 queries x K 128)    TMEM [0, 64)
//   dP^T = V dO_i^T         (SS)                                         TMEM [64, 128)
//   P^T  = exp2(S^T * scale * log2(e) - L2_i),  dS^T = P^T (dP^T - Delta_i)   (softmax warps)
//   dV  += P^T dO_i         (TS: P^T bf16 from TMEM [128, 160), dO MN-major)   TMEM [192, 320)
//   dK  += dS^T Q_i         (TS: dS^T from TMEM [160, 192), Q MN-major)         TMEM [320, 448)
//   dQ_i^T = K^T dS_i^T     (SS: K as an MN-major A, dS^T from shared memory)   TMEM [448, 512)
// and dQ_i^T leaves through a shared-memory box and TMA reduce-add (fp32) into a zeroed
// accumulator that bwd_tc_post_kernel scales and converts.  The MMA order is
//   S_0 dP_0 | P_0 ready | S_1 dP_1 dV_0 dK_0 dQ_0 | P_1 ready | S_2 dP_2 dV_1 dK_1 dQ_1 | ...
// so the softmax warps compute step i+1 while the tensor core runs dV_i, dK_i and dQ_i; they
// wait for dK_i (which reads the previous P^T / dS^T columns) only before storing.
//
//   warps 0-3  softmax: thread = key row (TMEM lane), 64 queries per step
//   warps 4-7  dQ writer (thread = head-dim row of dQ^T), then the dK / dV epilogue
//   warp 8     TMA producer (K, V once; Q_i, dO_i, L2_i, Delta_i per step, two stages)
//   warp 9     MMA issuer (one thread)
// Every mbarrier wait is bounded; on a timeout the CTA stops, drains (bounded) and frees TMEM.
#pragma once

#include "attn_common.cuh"
#include "sm100_ptx.cuh"

namespace mlxp {

struct BwdTcParams {
  int B, H, Sq, Skv, kv_group, n_kt, Sq_pad;
  const float* lse2;   // [B * H][Sq_pad]: L * log2(e); +inf for rows without keys and padding
  const float* delta;  // [B * H][Sq_pad]: rowsum(dO * O); 0 in padding
  void* dk;
  void* dv;
  long long dk_sb, dk_sh, dk_ss, dv_sb, dv_sh, dv_ss;
  float scale, scale_log2;
  MaskSpec mask;
  TmaCoordMap cq, ck, cv, cdo, cdq;
  int* status;
  unsigned long long timeout_ns;
};

struct BwdTcCfg {
  static constexpr int D = 128, BN = 128, BM = 64, KB = 2;
  static constexpr int K_TILE = BN * D * 2;   // 32 KB
  static constexpr int BOX_K = BN * 128;      // one 64-column box of K / V
  static constexpr int Q_TILE = BM * D * 2;   // 16 KB
  static constexpr int BOX_Q = BM * 128;      // one 64-column box of Q / dO
  static constexpr int DS_TILE = BN * 128;    // dS^T: 128 key rows x 64 queries (bf16)
  static constexpr int DQ_BOX = BM * 128;     // dQ staging: 4 boxes of 64 rows x 32 fp32
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + K_TILE;
  static constexpr int OFF_QS = OFF_V + K_TILE;             // 2 stages x (Q, dO)
  static constexpr int OFF_LD = OFF_QS + 2 * 2 * Q_TILE;    // 2 stages x (L2, Delta) 512 B
  static constexpr int OFF_DS = OFF_LD + 1024;              // 2 x dS^T
  static constexpr int OFF_DQ = OFF_DS + 2 * DS_TILE;       // dQ staging (32 KB)
  static constexpr int OFF_BAR = OFF_DQ + 4 * DQ_BOX;
  enum {
    B_KVF = 0, B_QF = 1, B_QE = 3, B_SF = 5, B_PF = 6, B_PDF = 7, B_DSF = 8, B_DQF = 10,
    B_DQE = 11, B_ACC = 12, NBAR = 13
  };
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
  static constexpr int THREADS = 320;
  static constexpr uint32_t TM_S = 0, TM_DP = 64, TM_P = 128, TM_DS = 160, TM_DV = 192,
                            TM_DK = 320, TM_DQ = 448, TM_COLS = 512;
  static_assert(OFF_DS % 1024 == 0 && OFF_DQ % 1024 == 0 && OFF_QS % 1024 == 0, "atoms");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

enum : int { kSiteBwdProducer = 10, kSiteBwdMma = 11, kSiteBwdSoftmax = 12, kSiteBwdWriter = 13 };

// L2 and Delta in the padded layout the TMA kernel copies from, one warp per padded row.
template <typename T>
__global__ void __launch_bounds__(256) bwd_tc_prep_kernel(const BwdParams p, int D, int Sq_pad,
                                                          float* lse2, float* delta) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= (long long)p.B * p.H * Sq_pad) return;
  const long long i = row % Sq_pad, bh = row / Sq_pad;
  const long long h = bh % p.H, b = bh / p.H;
  if (i >= p.Sq) {
    if (lane == 0) {
      lse2[row] = INFINITY;
      delta[row] = 0.f;
    }
    return;
  }
  const T* o = static_cast<const T*>(p.o) + b * p.o_sb + h * p.o_sh + i * p.o_ss;
  const T* g = static_cast<const T*>(p.dout) + b * p.do_sb + h * p.do_sh + i * p.do_ss;
  float a = 0.f;
  for (int d = lane; d < D; d += 32) a = fmaf(bwd_ld(o + d), bwd_ld(g + d), a);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
  if (lane == 0) {
    const float L = p.lse[bh * p.Sq + i];
    lse2[row] = L == -INFINITY ? INFINITY : L * 1.4426950408889634f;
    delta[row] = a;
  }
}

// dq = scale * accumulator (fp32 [B][H][Sq][D] contiguous), in the output type and strides.
template <typename T>
__global__ void __launch_bounds__(256) bwd_tc_post_kernel(const BwdParams p, int D,
                                                          const float* acc) {
  const long long n = (long long)p.B * p.H * p.Sq * D;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const long long d = e % D, r = e / D;
    const long long i = r % p.Sq, bh = r / p.Sq;
    const long long h = bh % p.H, b = bh / p.H;
    bwd_st<T>(static_cast<T*>(p.dq) + b * p.dq_sb + h * p.dq_sh + i * p.dq_ss + d,
              acc[e] * p.scale);
  }
}

template <bool kBF16>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_do,
                          const __grid_constant__ CUtensorMap tm_dq, const BwdTcParams p) {
  using C = BwdTcCfg;
  using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + C::OFF_MISC + 4);
  auto BAR = [&](int i) -> uint32_t { return sbase + C::OFF_BAR + 8 * i; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // work: key tile (heaviest first for causal masks: small j sees the most query tiles)
  const int Hkv = p.H / p.kv_group;
  const int j = blockIdx.x / (p.B * Hkv);
  const int bhk = blockIdx.x - j * (p.B * Hkv);
  const int hk = bhk % Hkv, b = bhk / Hkv;
  const int c0 = j * C::BN;
  long long qlo, qhi;
  q_index_range(p.mask, c0, c0 + C::BN < p.Skv ? c0 + C::BN : p.Skv, p.Sq, qlo, qhi);
  const int qt_lo = (int)(qlo / C::BM), qt_hi = (int)((qhi + C::BM - 1) / C::BM);
  const int per_head = qt_hi > qt_lo ? qt_hi - qt_lo : 0;
  const int n_steps = per_head * p.kv_group;

  if (threadIdx.x == 0) {
    mbar_init(BAR(C::B_KVF), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(BAR(C::B_QF + s), 1);
      mbar_init(BAR(C::B_QE + s), 1);
      mbar_init(BAR(C::B_DSF + s), 1);
    }
    mbar_init(BAR(C::B_SF), 1);
    mbar_init(BAR(C::B_PF), 128);
    mbar_init(BAR(C::B_PDF), 1);
    mbar_init(BAR(C::B_DQF), 1);
    mbar_init(BAR(C::B_DQE), 128);
    mbar_init(BAR(C::B_ACC), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), C::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx wctx{abort_flag, p.status, p.timeout_ns};
  auto step_qh = [&](int i, int& h, int& q0) {
    const int g = i / per_head;
    h = hk * p.kv_group + g;
    q0 = (qt_lo + (i - g * per_head)) * C::BM;
  };

  if (warp == 8) {
    // =================================== TMA producer ===================================
    if (lane == 0 && n_steps > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      int c1, c2, c3;
      mbar_arrive_expect_tx(BAR(C::B_KVF), 2 * C::K_TILE);
      tma_coords(p.ck, c0, hk, b, c1, c2, c3);
#pragma unroll
      for (int kb = 0; kb < C::KB; ++kb)
        tma_load_4d(sbase + C::OFF_K + kb * C::BOX_K, &tm_k, BAR(C::B_KVF), kb * 64, c1, c2, c3);
      tma_coords(p.cv, c0, hk, b, c1, c2, c3);
#pragma unroll
      for (int kb = 0; kb < C::KB; ++kb)
        tma_load_4d(sbase + C::OFF_V + kb * C::BOX_K, &tm_v, BAR(C::B_KVF), kb * 64, c1, c2, c3);
      bool ok = true;
      int issued = 0;
      for (int i = 0; i < n_steps; ++i) {
        const int s = i & 1;
        if (i >= 2) {
          ok = mbar_wait(BAR(C::B_QE + s), ((i >> 1) - 1) & 1, wctx, kSiteBwdProducer);
          if (!ok) break;
        }
        int h, q0;
        step_qh(i, h, q0);
        const uint32_t st = sbase + C::OFF_QS + s * 2 * C::Q_TILE;
        mbar_arrive_expect_tx(BAR(C::B_QF + s), 2 * C::Q_TILE + 512);
        tma_coords(p.cq, q0, h, b, c1, c2, c3);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_4d(st + kb * C::BOX_Q, &tm_q, BAR(C::B_QF + s), kb * 64, c1, c2, c3);
        tma_coords(p.cdo, q0, h, b, c1, c2, c3);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_4d(st + C::Q_TILE + kb * C::BOX_Q, &tm_do, BAR(C::B_QF + s), kb * 64, c1, c2,
                      c3);
        const long long r = ((long long)b * p.H + h) * p.Sq_pad + q0;
        const uint32_t ld = sbase + C::OFF_LD + s * 512;
        bulk_copy_g2s(ld, p.lse2 + r, 256, BAR(C::B_QF + s));
        bulk_copy_g2s(ld + 256, p.delta + r, 256, BAR(C::B_QF + s));
        ++issued;
      }
      // Let every load already issued land before the CTA releases its shared memory (a
      // normal run consumed all of them already: these waits then return at once).
      mbar_wait_drain(BAR(C::B_KVF), 0, p.status, p.timeout_ns);
      for (int i = (issued > 2 ? issued - 2 : 0); i < issued; ++i)
        mbar_wait_drain(BAR(C::B_QF + (i & 1)), (i >> 1) & 1, p.status, p.timeout_ns);
    }
  } else if (warp == 9) {
    // ==================================== MMA issuer ====================================
    if (lane == 0) {
      constexpr uint32_t id_s = make_idesc_f16_ab(128, C::BM, kBF16, false, false);
      constexpr uint32_t id_acc = make_idesc_f16_ab(128, C::D, kBF16, false, true);
      constexpr uint32_t id_dq = make_idesc_f16_ab(128, C::BM, kBF16, true, true);
      const uint32_t k_lo = ((sbase + C::OFF_K) >> 4) | (1u << 16);
      const uint32_t v_lo = ((sbase + C::OFF_V) >> 4) | (1u << 16);
      const uint32_t k_mn = ((sbase + C::OFF_K) >> 4) | ((uint32_t)(C::BOX_K >> 4) << 16);
      bool ok = n_steps > 0 ? mbar_wait(BAR(C::B_KVF), 0, wctx, kSiteBwdMma) : true;
      auto issue_sdp = [&](int i) {
        const int s = i & 1;
        const uint32_t q_lo = ((sbase + C::OFF_QS + s * 2 * C::Q_TILE) >> 4) | (1u << 16);
        const uint32_t o_lo = q_lo + (uint32_t)(C::Q_TILE >> 4);
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t ka = (uint32_t)((kb * C::BOX_K + kk * 32) >> 4);
            const uint32_t qa = (uint32_t)((kb * C::BOX_Q + kk * 32) >> 4);
            mma_ss(tmem + C::TM_S, sdesc(k_lo + ka), sdesc(q_lo + qa), id_s, (kb | kk) ? 1u : 0u);
          }
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t ka = (uint32_t)((kb * C::BOX_K + kk * 32) >> 4);
            const uint32_t qa = (uint32_t)((kb * C::BOX_Q + kk * 32) >> 4);
            mma_ss(tmem + C::TM_DP, sdesc(v_lo + ka), sdesc(o_lo + qa), id_s, (kb | kk) ? 1u : 0u);
          }
        tc_commit(BAR(C::B_SF));
      };
      if (ok && n_steps > 0) {
        ok = mbar_wait(BAR(C::B_QF), 0, wctx, kSiteBwdMma);
        if (ok) {
          tc_fence_after();
          issue_sdp(0);
        }
      }
      for (int i = 0; i < n_steps && ok; ++i) {
        const int s = i & 1;
        ok = mbar_wait(BAR(C::B_PF), i & 1, wctx, kSiteBwdMma);
        if (!ok) break;
        tc_fence_after();
        if (i + 1 < n_steps) {
          ok = mbar_wait(BAR(C::B_QF + ((i + 1) & 1)), ((i + 1) >> 1) & 1, wctx, kSiteBwdMma);
          if (!ok) break;
          tc_fence_after();
          issue_sdp(i + 1);
        }
        // dV += P^T dO_i, dK += dS^T Q_i (MN-major B: 64-column chunks 8 KB apart)
        const uint32_t qm = ((sbase + C::OFF_QS + s * 2 * C::Q_TILE) >> 4) |
                            ((uint32_t)(C::BOX_Q >> 4) << 16);
        const uint32_t om = qm + (uint32_t)(C::Q_TILE >> 4);
#pragma unroll
        for (int kk = 0; kk < C::BM / 16; ++kk)
          mma_ts(tmem + C::TM_DV, tmem + C::TM_P + kk * 8, sdesc(om + (uint32_t)(kk * 16 * 128 >> 4)),
                 id_acc, (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < C::BM / 16; ++kk)
          mma_ts(tmem + C::TM_DK, tmem + C::TM_DS + kk * 8,
                 sdesc(qm + (uint32_t)(kk * 16 * 128 >> 4)), id_acc, (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(BAR(C::B_PDF));
        // dQ_i^T = K^T dS_i^T: A = K (MN-major, 64-row chunks of head_dim 16 KB apart),
        // B = dS^T from shared memory (MN-major), K steps of 16 keys
        if (i >= 1) {
          ok = mbar_wait(BAR(C::B_DQE), (i - 1) & 1, wctx, kSiteBwdMma);
          if (!ok) break;
          tc_fence_after();
        }
        const uint32_t ds = ((sbase + C::OFF_DS + s * C::DS_TILE) >> 4) |
                            ((uint32_t)(C::DS_TILE >> 4) << 16);
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk)
          mma_ss(tmem + C::TM_DQ, sdesc(k_mn + (uint32_t)(kk * 16 * 128 >> 4)),
                 sdesc(ds + (uint32_t)(kk * 16 * 128 >> 4)), id_dq, kk > 0 ? 1u : 0u);
        tc_commit(BAR(C::B_DQF));
        tc_commit(BAR(C::B_DSF + s));
        tc_commit(BAR(C::B_QE + s));
      }
      tc_commit(BAR(C::B_ACC));  // every MMA issued above is complete when this arrives
      mbar_wait_drain(BAR(C::B_ACC), 0, p.status, p.timeout_ns);
    }
  } else if (warp < 4) {
    // ===================================== softmax ======================================
    const int k = warp * 32 + lane;  // key row of the tile = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const long long kpos = (long long)c0 + k + p.mask.kv_off;
    const bool key_ok = c0 + k < p.Skv;
    bool ok = true;
    for (int i = 0; i < n_steps && ok; ++i) {
      const int s = i & 1;
      int h, q0;
      step_qh(i, h, q0);
      // admissible local queries [qa, qb) of this key
      long long qa = 0, qb = C::BM;
      const long long base = q0 + p.mask.q_off;  // position of local query 0
      if (p.mask.causal && kpos - base > qa) qa = kpos - base;
      if (p.mask.wr >= 0 && kpos - p.mask.wr - base > qa) qa = kpos - p.mask.wr - base;
      if (p.mask.wl >= 0 && kpos + p.mask.wl - base + 1 < qb) qb = kpos + p.mask.wl - base + 1;
      if (!key_ok || qb < qa) qb = qa;
      const uint32_t lo = (uint32_t)qa, width = (uint32_t)(qb - qa);
      ok = mbar_wait(BAR(C::B_SF), i & 1, wctx, kSiteBwdSoftmax) &&
           mbar_wait(BAR(C::B_QF + s), (i >> 1) & 1, wctx, kSiteBwdSoftmax);
      if (!ok) break;
      tc_fence_after();
      const float* l2 = reinterpret_cast<const float*>(smem + C::OFF_LD + s * 512);
      const float* dl = l2 + 64;
      uint32_t pp[32], dd[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sr[32], dr[32];
        tmem_ld_x32(lane_base + C::TM_S + 32 * half, sr);
        tmem_ld_x32(lane_base + C::TM_DP + 32 * half, dr);
        tmem_wait_ld();
        reg_fence(sr);
        reg_fence(dr);
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float pv[2], dv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int q = 32 * half + c + e;
            const float x = fmaf(__uint_as_float(sr[c + e]), p.scale_log2, -l2[q]);
            const float pr = ((uint32_t)q - lo < width) ? ex2_approx(x) : 0.f;
            pv[e] = pr;
            dv[e] = pr * (__uint_as_float(dr[c + e]) - dl[q]);
          }
          pp[16 * half + c / 2] = pack2<kBF16>(pv[0], pv[1]);
          dd[16 * half + c / 2] = pack2<kBF16>(dv[0], dv[1]);
        }
      }
      // the previous step's P^T / dS^T columns are free once dK_{i-1} completed
      if (i >= 1) {
        ok = mbar_wait(BAR(C::B_PDF), (i - 1) & 1, wctx, kSiteBwdSoftmax);
        if (!ok) break;
        tc_fence_after();
      }
      tmem_st_x32(lane_base + C::TM_P, pp);
      tmem_st_x32(lane_base + C::TM_DS, dd);
      // dS^T row k into this step's shared-memory buffer (MN-major B, 128-byte swizzle)
      if (i >= 2) {
        ok = mbar_wait(BAR(C::B_DSF + s), ((i >> 1) - 1) & 1, wctx, kSiteBwdSoftmax);
        if (!ok) break;
      }
      const uint32_t row = sbase + C::OFF_DS + s * C::DS_TILE + k * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        st_shared_v4(row + ((c ^ (k & 7)) << 4), dd[4 * c], dd[4 * c + 1], dd[4 * c + 2],
                     dd[4 * c + 3]);
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR(C::B_PF));
    }
  } else {
    // ============================ dQ writer, then dK / dV ==============================
    const int d = (warp - 4) * 32 + lane;  // dQ^T lane = head-dim row; dK/dV lane = key row
    const uint32_t lane_base = tmem + ((uint32_t)((warp - 4) * 32) << 16);
    const bool leader = warp == 4 && lane == 0;
    bool ok = true;
    for (int i = 0; i < n_steps && ok; ++i) {
      int h, q0;
      step_qh(i, h, q0);
      ok = mbar_wait(BAR(C::B_DQF), i & 1, wctx, kSiteBwdWriter);
      ok = named_bar_and(1, 128, ok);  // the 128 writers agree before their named barriers
      if (!ok) break;
      tc_fence_after();
      uint32_t v0[32], v1[32];
      tmem_ld_x32(lane_base + C::TM_DQ, v0);
      tmem_ld_x32(lane_base + C::TM_DQ + 32, v1);
      tmem_wait_ld();
      reg_fence(v0);
      reg_fence(v1);
      tc_fence_before();
      mbar_arrive(BAR(C::B_DQE));
      // staging: box d/32 holds 64 query rows x 32 fp32 (128 B), 128-byte swizzle
      if (leader) bulk_wait_group_read0();  // the previous reduce has read the staging
      named_bar_sync(1, 128);
      const uint32_t box = sbase + C::OFF_DQ + (d >> 5) * C::DQ_BOX;
      const int chunk = (d & 31) >> 2, within = (d & 3) * 4;
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(box + q * 128 + ((chunk ^ (q & 7)) << 4) + within),
                     "r"(v0[q]) : "memory");
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(box + (q + 32) * 128 + ((chunk ^ (q & 7)) << 4) + within),
                     "r"(v1[q]) : "memory");
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (leader) {
        int c1, c2, c3;
        tma_coords(p.cdq, q0, h, b, c1, c2, c3);
#pragma unroll
        for (int bx = 0; bx < 4; ++bx)
          tma_reduce_add_4d(&tm_dq, sbase + C::OFF_DQ + bx * C::DQ_BOX, bx * 32, c1, c2, c3);
        bulk_commit_group();
      }
    }
    if (leader) bulk_wait_group0();
    // dK, dV of the tile: thread = key row
    if (ok && n_steps > 0) ok = mbar_wait(BAR(C::B_ACC), 0, wctx, kSiteBwdWriter);
    if (ok) {
      tc_fence_after();
      const int key = c0 + d;
      T* dvr = static_cast<T*>(p.dv) + b * p.dv_sb + hk * p.dv_sh + (long long)key * p.dv_ss;
      T* dkr = static_cast<T*>(p.dk) + b * p.dk_sb + hk * p.dk_sh + (long long)key * p.dk_ss;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        T* dst = which ? dkr : dvr;
        const float mul = which ? p.scale : 1.f;
#pragma unroll 1
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t r[32];
          if (n_steps > 0) {
            tmem_ld_x32(lane_base + (which ? C::TM_DK : C::TM_DV) + 32 * cb, r);
            tmem_wait_ld();
            reg_fence(r);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = 0u;
          }
          if (key < p.Skv) {
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
              uint4 u;
              u.x = pack2<kBF16>(__uint_as_float(r[e]) * mul, __uint_as_float(r[e + 1]) * mul);
              u.y = pack2<kBF16>(__uint_as_float(r[e + 2]) * mul, __uint_as_float(r[e + 3]) * mul);
              u.z = pack2<kBF16>(__uint_as_float(r[e + 4]) * mul, __uint_as_float(r[e + 5]) * mul);
              u.w = pack2<kBF16>(__uint_as_float(r[e + 6]) * mul, __uint_as_float(r[e + 7]) * mul);
              *reinterpret_cast<uint4*>(dst + 32 * cb + e) = u;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TM_COLS);
  }
}

}  // namespace mlxp
