// attn_bwd_sm100.cuh — attention backward (dQ, dK, dV) on the 5th-generation tensor cores,
// head_dim 64 or 128, bf16/fp16 inputs, fp32 accumulation in TMEM.
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
// accumulator that bwd_tc_post_kernel scales and converts.  The softmax warps signal twice per
// step: once they have loaded S^T_i and dP^T_i into registers (the tensor core then computes
// S^T_{i+1}, dP^T_{i+1} into the same columns while they work), and once P^T_i, dS^T_i are
// stored (then dV_i, dK_i, dQ_i run while they start step i+1).  MMA order:
//   S_0 dP_0 | consumed 0 | S_1 dP_1 | ready 0 | dV_0 dK_0 dQ_0 | consumed 1 | S_2 dP_2 | ...
// Before storing P^T_{i+1} / dS^T_{i+1} the softmax warps wait for dK_i, the last reader of
// those columns.  (Measured with one softmax warpgroup and S/dP not overlapped: 5500 cycles
// per step, 3000 of them the softmax compute; see the history of this file.)
//
//   warps 0-7  softmax: thread = key row (TMEM lane); warps w and w + 4 share the lanes and
//              take queries 0-31 and 32-63 of the step
//   warps 8-11 dQ writer (thread = head-dim row of dQ^T), then the dK / dV epilogue
//   warp 12    TMA producer (K, V once; Q_i, dO_i, L2_i, Delta_i per step, two stages)
//   warp 13    MMA issuer (one thread)
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

// head_dim 64: dQ^T = K^T dS^T keeps M = 128 (the tensor core's row count for one CTA) with an
// A operand whose second 64-row chunk (head-dim rows 64-127) is a zero tile in shared memory;
// those accumulator lanes hold zeros and are never read.
template <int D_>
struct BwdTcCfg {
  static constexpr int D = D_, BN = 128, BM = 64, KB = D / 64;
  static constexpr int K_TILE = BN * D * 2;   // K or V tile
  static constexpr int BOX_K = BN * 128;      // one 64-column box of K / V
  static constexpr int Q_TILE = BM * D * 2;   // Q or dO tile
  static constexpr int BOX_Q = BM * 128;      // one 64-column box of Q / dO
  static constexpr int DS_TILE = BN * 128;    // dS^T: 128 key rows x 64 queries (bf16)
  static constexpr int NQS = 3;               // Q / dO stages
  static constexpr int DQ_BOX = 32 * 128;     // dQ staging: D/32 boxes of 32 rows x 32 fp32
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + K_TILE;
  static constexpr int OFF_ZERO = OFF_V + K_TILE;           // head_dim 64: 16 KB of zeros
  static constexpr int OFF_QS = OFF_ZERO + (D == 64 ? BOX_K : 0);  // NQS stages x (Q, dO)
  static constexpr int OFF_LD = OFF_QS + NQS * 2 * Q_TILE;  // NQS stages x (L2, Delta) 512 B
  static constexpr int OFF_DS = OFF_LD + 2048;              // 2 x dS^T
  static constexpr int OFF_DQ = OFF_DS + 2 * DS_TILE;       // dQ staging (16 KB, half a step)
  static constexpr int OFF_BAR = OFF_DQ + (D / 32) * DQ_BOX;
  enum {
    B_KVF = 0, B_QF = 1, B_QE = 4, B_SF = 7, B_PF = 8, B_PDF = 9, B_DSF = 10, B_DQF = 12,
    B_DQE = 13, B_ACC = 14, B_SC = 15, NBAR = 16
  };
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
  static constexpr int THREADS = 448;
  static constexpr uint32_t TM_S = 0, TM_DP = 64, TM_P = 128, TM_DS = 160, TM_DV = 192,
                            TM_DK = 192 + D, TM_DQ = 192 + 2 * D, TM_COLS = 512;
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(OFF_DS % 1024 == 0 && OFF_DQ % 1024 == 0 && OFF_QS % 1024 == 0, "atoms");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

enum : int { kSiteBwdProducer = 10, kSiteBwdMma = 11, kSiteBwdSoftmax = 12, kSiteBwdWriter = 13 };

// L2 and Delta in the padded layout the TMA kernel copies from, one warp per padded row
// (each lane reads D/32 consecutive elements of O and dO).
template <typename T, int D>
__global__ void __launch_bounds__(256) bwd_tc_prep_kernel(const BwdParams p, int Sq_pad,
                                                          float* lse2, float* delta) {
  constexpr int E = D / 32;
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
  const T* o = static_cast<const T*>(p.o) + b * p.o_sb + h * p.o_sh + i * p.o_ss + E * lane;
  const T* g = static_cast<const T*>(p.dout) + b * p.do_sb + h * p.do_sh + i * p.do_ss + E * lane;
  using V = typename std::conditional<E == 4, uint2, uint32_t>::type;
  float a = 0.f;
  if (((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(g)) & (2 * E - 1)) == 0) {
    const V uo = *reinterpret_cast<const V*>(o), ug = *reinterpret_cast<const V*>(g);
    const T* eo = reinterpret_cast<const T*>(&uo);
    const T* eg = reinterpret_cast<const T*>(&ug);
#pragma unroll
    for (int e = 0; e < E; ++e) a = fmaf(bwd_ld(eo + e), bwd_ld(eg + e), a);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) a = fmaf(bwd_ld(o + e), bwd_ld(g + e), a);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
  if (lane == 0) {
    const float L = p.lse[bh * p.Sq + i];
    lse2[row] = L == -INFINITY ? INFINITY : L * 1.4426950408889634f;
    delta[row] = a;
  }
}

// dq = scale * accumulator (fp32 [B][H][Sq][D] contiguous), in the output type and strides;
// 8 consecutive elements per thread (one 16-byte store when VEC: dq rows 16-byte aligned).
template <typename T, int D, bool VEC>
__global__ void __launch_bounds__(256) bwd_tc_post_kernel(const BwdParams p, const float* acc) {
  const long long n8 = (long long)p.B * p.H * p.Sq * (D / 8);
  for (long long e8 = (long long)blockIdx.x * blockDim.x + threadIdx.x; e8 < n8;
       e8 += (long long)gridDim.x * blockDim.x) {
    const int d0 = (int)(e8 % (D / 8)) * 8;
    const long long r = e8 / (D / 8);
    const long long i = r % p.Sq, bh = r / p.Sq;
    const long long h = bh % p.H, b = bh / p.H;
    const float4 x0 = *reinterpret_cast<const float4*>(acc + e8 * 8);
    const float4 x1 = *reinterpret_cast<const float4*>(acc + e8 * 8 + 4);
    const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    T* dst = static_cast<T*>(p.dq) + b * p.dq_sb + h * p.dq_sh + i * p.dq_ss + d0;
    if constexpr (VEC) {
      uint4 u;
      u.x = pack2<std::is_same<T, __nv_bfloat16>::value>(v[0] * p.scale, v[1] * p.scale);
      u.y = pack2<std::is_same<T, __nv_bfloat16>::value>(v[2] * p.scale, v[3] * p.scale);
      u.z = pack2<std::is_same<T, __nv_bfloat16>::value>(v[4] * p.scale, v[5] * p.scale);
      u.w = pack2<std::is_same<T, __nv_bfloat16>::value>(v[6] * p.scale, v[7] * p.scale);
      *reinterpret_cast<uint4*>(dst) = u;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) bwd_st<T>(dst + e, v[e] * p.scale);
    }
  }
}

template <bool kBF16, int D>
__global__ void __launch_bounds__(448, 1)
    attn_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_do,
                          const __grid_constant__ CUtensorMap tm_dq, const BwdTcParams p) {
  using C = BwdTcCfg<D>;
  using T = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  int* abort_flag = reinterpret_cast<int*>(smem + C::OFF_MISC + 4);
  auto BAR = [&](int i) -> uint32_t { return sbase + C::OFF_BAR + 8 * i; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // work: (batch, K/V head) major, key tile minor — the CTAs running at the same time share
  // the Q, dO and dQ-accumulator rows of a few heads in L2 (key-tile-major order re-read Q and
  // dO from DRAM for every key tile: 7.8 GB of reads for config 2); within a head the small j
  // (most query tiles under a causal mask) come first
  const int Hkv = p.H / p.kv_group;
  const int bhk = blockIdx.x / p.n_kt;
  const int j = blockIdx.x - bhk * p.n_kt;
  const int hk = bhk % Hkv, b = bhk / Hkv;
  const int c0 = j * C::BN;
  long long qlo, qhi;
  q_index_range(p.mask, c0, c0 + C::BN < p.Skv ? c0 + C::BN : p.Skv, p.Sq, qlo, qhi);
  const int qt_lo = (int)(qlo / C::BM), qt_hi = (int)((qhi + C::BM - 1) / C::BM);
  const int per_head = qt_hi > qt_lo ? qt_hi - qt_lo : 0;
  const int n_steps = per_head * p.kv_group;

  if (threadIdx.x == 0) {
    mbar_init(BAR(C::B_KVF), 1);
    for (int s = 0; s < C::NQS; ++s) {
      mbar_init(BAR(C::B_QF + s), 1);
      mbar_init(BAR(C::B_QE + s), 1);
    }
    for (int s = 0; s < 2; ++s) mbar_init(BAR(C::B_DSF + s), 1);
    mbar_init(BAR(C::B_SF), 1);
    mbar_init(BAR(C::B_PF), 256);
    mbar_init(BAR(C::B_SC), 256);
    mbar_init(BAR(C::B_PDF), 1);
    mbar_init(BAR(C::B_DQF), 1);
    mbar_init(BAR(C::B_DQE), 128);
    mbar_init(BAR(C::B_ACC), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 13) {
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

  if (warp == 12) {
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
        const int s = i % C::NQS;
        if (i >= C::NQS) {
          ok = mbar_wait(BAR(C::B_QE + s), ((i / C::NQS) - 1) & 1, wctx, kSiteBwdProducer);
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
      for (int i = (issued > C::NQS ? issued - C::NQS : 0); i < issued; ++i)
        mbar_wait_drain(BAR(C::B_QF + i % C::NQS), (i / C::NQS) & 1, p.status, p.timeout_ns);
    }
  } else if (warp == 13) {
    // ==================================== MMA issuer ====================================
    if (lane == 0) {
      constexpr uint32_t id_s = make_idesc_f16_ab(128, C::BM, kBF16, false, false);
      constexpr uint32_t id_acc = make_idesc_f16_ab(128, C::D, kBF16, false, true);
      constexpr uint32_t id_dq = make_idesc_f16_ab(128, C::BM, kBF16, true, true);
      const uint32_t k_lo = ((sbase + C::OFF_K) >> 4) | (1u << 16);
      const uint32_t v_lo = ((sbase + C::OFF_V) >> 4) | (1u << 16);
      // dQ^T's A = K^T (MN-major, two 64-row chunks of head dim: K's second box, or the zero
      // tile for head_dim 64)
      constexpr uint32_t a_lbo = (D == 128 ? C::BOX_K : C::OFF_ZERO - C::OFF_K);
      const uint32_t k_mn = ((sbase + C::OFF_K) >> 4) | ((a_lbo >> 4) << 16);
      bool ok = n_steps > 0 ? mbar_wait(BAR(C::B_KVF), 0, wctx, kSiteBwdMma) : true;
      auto issue_sdp = [&](int i) {
        const int s = i % C::NQS;
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
        const int s = i % C::NQS, sb = i & 1;  // Q / dO stage, dS buffer
        if (i + 1 < n_steps) {  // S^T_{i+1}, dP^T_{i+1} once the softmax warps hold S^T_i, dP^T_i
          ok = mbar_wait(BAR(C::B_SC), i & 1, wctx, kSiteBwdMma) &&
               mbar_wait(BAR(C::B_QF + (i + 1) % C::NQS), ((i + 1) / C::NQS) & 1, wctx,
                         kSiteBwdMma);
          if (!ok) break;
          tc_fence_after();
          issue_sdp(i + 1);
        }
        ok = mbar_wait(BAR(C::B_PF), i & 1, wctx, kSiteBwdMma);
        if (!ok) break;
        tc_fence_after();
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
        const uint32_t ds = ((sbase + C::OFF_DS + sb * C::DS_TILE) >> 4) |
                            ((uint32_t)(C::DS_TILE >> 4) << 16);
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk)
          mma_ss(tmem + C::TM_DQ, sdesc(k_mn + (uint32_t)(kk * 16 * 128 >> 4)),
                 sdesc(ds + (uint32_t)(kk * 16 * 128 >> 4)), id_dq, kk > 0 ? 1u : 0u);
        // one commit: its completion also frees dS buffer sb and Q/dO stage s, which the dQ
        // writer passes on (commits in the MMA stream are not free)
        tc_commit(BAR(C::B_DQF));
      }
      tc_commit(BAR(C::B_ACC));  // every MMA issued above is complete when this arrives
      mbar_wait_drain(BAR(C::B_ACC), 0, p.status, p.timeout_ns);
    }
  } else if (warp < 8) {
    // ===================================== softmax ======================================
    if constexpr (D == 64) {  // the zero half of dQ^T's A operand (fenced before the first PF)
      for (int e = threadIdx.x; e < C::BOX_K / 16; e += 256)
        st_shared_v4(sbase + C::OFF_ZERO + 16 * e, 0u, 0u, 0u, 0u);
    }
    const int k = (warp & 3) * 32 + lane;  // key row of the tile = TMEM lane
    const int hc = warp >> 2;              // query half: local queries 32 * hc .. 32 * hc + 31
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const long long kpos = (long long)c0 + k + p.mask.kv_off;
    const bool key_ok = c0 + k < p.Skv;
    bool ok = true;
    for (int i = 0; i < n_steps && ok; ++i) {
      const int s = i % C::NQS, sb = i & 1;  // Q / dO stage, dS buffer
      int h, q0;
      step_qh(i, h, q0);
      // admissible queries [qa, qb) of this key, local to this warp's 32 columns
      long long qa = 0, qb = C::BM;
      const long long base = q0 + p.mask.q_off;  // position of local query 0
      if (p.mask.causal && kpos - base > qa) qa = kpos - base;
      if (p.mask.wr >= 0 && kpos - p.mask.wr - base > qa) qa = kpos - p.mask.wr - base;
      if (p.mask.wl >= 0 && kpos + p.mask.wl - base + 1 < qb) qb = kpos + p.mask.wl - base + 1;
      if (!key_ok || qb < qa) qb = qa;
      const uint32_t lo = (uint32_t)(qa - 32 * hc), width = (uint32_t)(qb - qa);
      ok = mbar_wait(BAR(C::B_SF), i & 1, wctx, kSiteBwdSoftmax) &&
           mbar_wait(BAR(C::B_QF + s), (i / C::NQS) & 1, wctx, kSiteBwdSoftmax);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[32], dr[32];
      tmem_ld_x32(lane_base + C::TM_S + 32 * hc, sr);
      tmem_ld_x32(lane_base + C::TM_DP + 32 * hc, dr);
      tmem_wait_ld();
      reg_fence(sr);
      reg_fence(dr);
      tc_fence_before();
      mbar_arrive(BAR(C::B_SC));  // S^T_i, dP^T_i are in registers: their columns may be reused
      const float4* l2 = reinterpret_cast<const float4*>(smem + C::OFF_LD + s * 512) + 8 * hc;
      const float4* dl = l2 + 16;
      uint32_t pp[16], dd[16];
#pragma unroll
      for (int c = 0; c < 32; c += 4) {
        const float4 L4 = l2[c / 4], D4 = dl[c / 4];
        const float Ls[4] = {L4.x, L4.y, L4.z, L4.w}, Ds[4] = {D4.x, D4.y, D4.z, D4.w};
        float pv[4], dv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = fmaf(__uint_as_float(sr[c + e]), p.scale_log2, -Ls[e]);
          const float pr = ((uint32_t)(c + e) - lo < width) ? ex2_approx(x) : 0.f;
          pv[e] = pr;
          dv[e] = pr * (__uint_as_float(dr[c + e]) - Ds[e]);
        }
        pp[c / 2] = pack2<kBF16>(pv[0], pv[1]);
        pp[c / 2 + 1] = pack2<kBF16>(pv[2], pv[3]);
        dd[c / 2] = pack2<kBF16>(dv[0], dv[1]);
        dd[c / 2 + 1] = pack2<kBF16>(dv[2], dv[3]);
      }
      // the previous step's P^T / dS^T columns are free once dK_{i-1} completed
      if (i >= 1) {
        ok = mbar_wait(BAR(C::B_PDF), (i - 1) & 1, wctx, kSiteBwdSoftmax);
        if (!ok) break;
        tc_fence_after();
      }
      tmem_st_x16(lane_base + C::TM_P + 16 * hc, pp);
      tmem_st_x16(lane_base + C::TM_DS + 16 * hc, dd);
      // dS^T row k, this half, into the step's shared-memory buffer (MN-major B, 128-byte
      // swizzle: 16-byte chunk c of row k at chunk c ^ (k % 8))
      if (i >= 2) {
        ok = mbar_wait(BAR(C::B_DSF + sb), ((i >> 1) - 1) & 1, wctx, kSiteBwdSoftmax);
        if (!ok) break;
      }
      const uint32_t row = sbase + C::OFF_DS + sb * C::DS_TILE + k * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        st_shared_v4(row + (((4 * hc + c) ^ (k & 7)) << 4), dd[4 * c], dd[4 * c + 1],
                     dd[4 * c + 2], dd[4 * c + 3]);
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR(C::B_PF));
    }
  } else {
    // ============================ dQ writer, then dK / dV ==============================
    const int d = (warp - 8) * 32 + lane;  // dQ^T lane = head-dim row; dK/dV lane = key row
    const uint32_t lane_base = tmem + ((uint32_t)((warp - 8) * 32) << 16);
    const bool leader = warp == 8 && lane == 0;
    bool ok = true;
    for (int i = 0; i < n_steps && ok; ++i) {
      int h, q0;
      step_qh(i, h, q0);
      ok = mbar_wait(BAR(C::B_DQF), i & 1, wctx, kSiteBwdWriter);
      ok = named_bar_and(1, 128, ok);  // the 128 writers agree before their named barriers
      if (!ok) break;
      if (leader) {  // every MMA of step i is complete: its dS buffer and Q/dO stage are free
        mbar_arrive(BAR(C::B_DSF + (i & 1)));
        mbar_arrive(BAR(C::B_QE + i % C::NQS));
      }
      tc_fence_after();
      const bool rows = warp - 8 < D / 32;  // warp-uniform: this warp's head-dim rows exist
      uint32_t v0[32], v1[32];
      if (rows) {
        tmem_ld_x32(lane_base + C::TM_DQ, v0);
        tmem_ld_x32(lane_base + C::TM_DQ + 32, v1);
        tmem_wait_ld();
        reg_fence(v0);
        reg_fence(v1);
      }
      tc_fence_before();
      mbar_arrive(BAR(C::B_DQE));
      // staging: queries 0-31, then 32-63; box d/32 holds 32 query rows x 32 fp32 (128 B),
      // 128-byte swizzle
      const uint32_t box = sbase + C::OFF_DQ + (d >> 5) * C::DQ_BOX;
      const int chunk = (d & 31) >> 2, within = (d & 3) * 4;
      int c1, c2, c3;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        if (leader) bulk_wait_group_read0();  // the previous reduce has read the staging
        named_bar_sync(1, 128);
        if (rows) {
#pragma unroll
          for (int q = 0; q < 32; ++q)
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(box + q * 128 + ((chunk ^ (q & 7)) << 4) + within),
                         "r"(half ? v1[q] : v0[q]) : "memory");
        }
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        if (leader) {
          tma_coords(p.cdq, q0 + 32 * half, h, b, c1, c2, c3);
#pragma unroll
          for (int bx = 0; bx < D / 32; ++bx)
            tma_reduce_add_4d(&tm_dq, sbase + C::OFF_DQ + bx * C::DQ_BOX, bx * 32, c1, c2, c3);
          bulk_commit_group();
        }
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
        for (int cb = 0; cb < D / 32; ++cb) {
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
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TM_COLS);
  }
}

}  // namespace mlxp
