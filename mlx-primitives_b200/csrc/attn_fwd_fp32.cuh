// attn_fwd_fp32.cuh — fp32 attention forward on CUDA cores (FFMA), the tight-parity variant.
//
// The reference's fp32 paths (flash.py:257-316 tiled online softmax, flash.py:329-408 Metal
// per-query kernel) accumulate in fp32 and rescale exactly on every new maximum; this kernel
// does the same (no lazy rescale), with scores scaled into the log2 domain once.
//
// CTA = 64 query rows x one (batch, head); 256 threads as a 16 x 16 grid: thread (ty, tx) owns
// query rows 4*ty .. 4*ty+3 (scores, running max/sum and output accumulators), the key columns
// tx + 16*c of each key tile, and the EPT = D/16 consecutive output columns EPT*tx .. of the
// head dimension.  Shared-memory operands are read as 16-byte vectors (4 head-dim elements of
// Q and K per load, 4 keys of P per load, EPT consecutive columns of V), so a thread does
// 64 FMAs per 8 vector loads instead of 16 per 8 scalar ones.  Row reductions are 16-lane
// shuffles (the 16 threads of a row group share a warp).  K and V tiles are double-buffered:
// tile j+1 is copied with cp.async while tile j is computed.  Key splits (several CTAs per query
// block) are merged by the split that finishes last, in the same launch.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "attn_common.cuh"
#include "sm100_ptx.cuh"

namespace mlxp {


template <int D>
struct F32Cfg {
  static constexpr int BM = 64;
  static constexpr int BN = (D >= 128) ? 32 : 64;
  static constexpr int NC = BN / 16;   // key columns per thread
  static constexpr int EPT = D / 16;   // consecutive output columns per thread (2, 4 or 8)
  static constexpr int SQ = D;         // row pitch (floats) of Q in smem
  static constexpr int SK = D + 4;     // K pitch: rows of different tx lanes 16 bytes apart mod 128
  static constexpr int SV = D;
  static constexpr int SP = BN + 4;    // P pitch (16-byte aligned rows)
  static constexpr int KV_FLOATS = BN * SK + BN * SV;  // one stage of K and V
  static constexpr int SMEM_FLOATS = BM * SQ + 2 * KV_FLOATS + BM * SP;
  static constexpr int SMEM_BYTES = SMEM_FLOATS * 4;
  static_assert(D % 32 == 0 && D <= 128, "head_dim 32, 64 or 128");
};

template <int N>
__device__ __forceinline__ void lds_vec(const float* p, float* out) {
  if constexpr (N == 2) {
    const float2 v = *reinterpret_cast<const float2*>(p);
    out[0] = v.x; out[1] = v.y;
  } else {
#pragma unroll
    for (int j = 0; j < N; j += 4) {
      const float4 v = *reinterpret_cast<const float4*>(p + j);
      out[j] = v.x; out[j + 1] = v.y; out[j + 2] = v.z; out[j + 3] = v.w;
    }
  }
}

template <int D>
__global__ void __launch_bounds__(256) attn_fwd_fp32_kernel(const FwdParamsF32 p) {
  using C = F32Cfg<D>;
  extern __shared__ __align__(16) float fsm[];
  float* Qs = fsm;
  float* KVs = Qs + C::BM * C::SQ;  // [2][K tile, V tile]
  float* Ps = KVs + 2 * C::KV_FLOATS;

  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;
  const int n_qblk = (p.Sq + C::BM - 1) / C::BM;
  const int split = blockIdx.x % p.splits;
  const int blk = blockIdx.x / p.splits;
  // causal: query blocks heaviest first across all (batch, head) units (longest-processing-time
  // order, so that the last wave holds the lightest blocks); otherwise unit-major, so that the
  // blocks reading the same K/V run side by side
  int bh, qb;
  if (p.mask.causal) {
    const int BH = p.B * p.H;
    const int qrank = blk / BH;
    bh = blk - qrank * BH;
    qb = n_qblk - 1 - qrank;
  } else {
    bh = blk / n_qblk;
    qb = blk - bh * n_qblk;
  }
  const int h = bh % p.H, b = bh / p.H;
  const int q0 = qb * C::BM;

  const float* qg = p.q + (long long)b * p.q_sb + (long long)h * p.q_sh;
  const int hk = h / p.kv_group;  // K/V head of this query head
  const float* kg = p.k + (long long)b * p.k_sb + (long long)hk * p.k_sh;
  const float* vg = p.v + (long long)b * p.v_sb + (long long)hk * p.v_sh;

  // Q tile -> smem (rows past Sq are zero)
  for (int i = tid; i < C::BM * (D / 4); i += 256) {
    const int r = i / (D / 4), c4 = i % (D / 4);
    float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < p.Sq) val = *reinterpret_cast<const float4*>(qg + (long long)(q0 + r) * p.q_ss + c4 * 4);
    *reinterpret_cast<float4*>(Qs + r * C::SQ + c4 * 4) = val;
  }

  const long long r0 = q0;
  const long long r1 = (q0 + C::BM < p.Sq) ? q0 + C::BM : p.Sq;
  int tlo, thi;
  kv_tile_range(p.mask, r0, r1, C::BN, tlo, thi);
  if (p.splits > 1) {  // this split's share of the block's key tiles
    const int n = thi - tlo;
    const int lo = tlo + (int)((long long)n * split / p.splits);
    thi = tlo + (int)((long long)n * (split + 1) / p.splits);
    tlo = lo;
  }

  float m[4], l[4], acc[4][C::EPT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int d = 0; d < C::EPT; ++d) acc[i][d] = 0.f;
  }
  const float sl2 = p.scale_log2;

  // K and V of key tile jt into stage buf (rows past Skv are zero-filled; their source address
  // stays row 0, which exists whenever the kernel runs)
  auto load_kv = [&](int jt, int buf) {
    const int c0 = jt * C::BN;
    float* Kb = KVs + buf * C::KV_FLOATS;
    float* Vb = Kb + C::BN * C::SK;
    for (int i = tid; i < C::BN * (D / 4); i += 256) {
      const int r = i / (D / 4), c4 = i % (D / 4);
      const bool in = c0 + r < p.Skv;
      const long long row = in ? c0 + r : 0;
      cp_async_piece<16>(smem_u32(Kb + r * C::SK + c4 * 4), kg + row * p.k_ss + c4 * 4, in ? 16 : 0);
      cp_async_piece<16>(smem_u32(Vb + r * C::SV + c4 * 4), vg + row * p.v_ss + c4 * 4, in ? 16 : 0);
    }
    cp_async_commit();
  };
  if (tlo < thi) load_kv(tlo, 0);

  for (int jt = tlo; jt < thi; ++jt) {
    const int c0 = jt * C::BN;
    const int buf = (jt - tlo) & 1;
    __syncthreads();  // previous tile fully consumed (and Q stored, first time)
    if (jt + 1 < thi) {
      load_kv(jt + 1, buf ^ 1);  // overlaps this tile's compute
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // tile jt is visible to every thread
    const float* Ks = KVs + buf * C::KV_FLOATS;
    const float* Vs = Ks + C::BN * C::SK;

    float s[4][C::NC];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < C::NC; ++c) s[i][c] = 0.f;
    // fully unrolled (as the P.V loop below): the shared-memory loads of later steps issue
    // early (config 1, unroll 2 / 4 / 8 / full: 23.5 / 24.3 / 24.9 / 25.5 TFLOPS)
#pragma unroll
    for (int d = 0; d < D; d += 4) {
      float qv[4][4], kv[C::NC][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) lds_vec<4>(Qs + (ty * 4 + i) * C::SQ + d, qv[i]);
#pragma unroll
      for (int c = 0; c < C::NC; ++c) lds_vec<4>(Ks + (tx + 16 * c) * C::SK + d, kv[c]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < C::NC; ++c)
#pragma unroll
          for (int e = 0; e < 4; ++e) s[i][c] = fmaf(qv[i][e], kv[c][e], s[i][c]);
    }

    const bool full = tile_is_full(p.mask, r0, r1, c0, c0 + C::BN);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = q0 + ty * 4 + i;
      int c_lo = 0, c_hi = C::BN - 1;
      if (!full) row_col_interval(p.mask, row, c0, C::BN, c_lo, c_hi);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < C::NC; ++c) {
        const int col = tx + 16 * c;
        s[i][c] = (col < c_lo || col > c_hi) ? -INFINITY : s[i][c] * sl2;
        mx = fmaxf(mx, s[i][c]);
      }
      if (p.bias != nullptr && row < p.Sq) {  // additive bias (log2 units: times log2(e))
        const float* br = p.bias + (long long)b * p.bias_sb + (long long)h * p.bias_sh +
                          (long long)row * p.bias_sq + c0;
        mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < C::NC; ++c) {
          const int col = tx + 16 * c;
          if (c0 + col < p.Skv) s[i][c] += __ldg(br + col) * 1.4426950408889634f;
          mx = fmaxf(mx, s[i][c]);
        }
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off, 16));
      const float m_new = fmaxf(m[i], mx);
      const float alpha = (m[i] == -INFINITY) ? 0.f : exp2f(m[i] - m_new);
      const float mu = (m_new == -INFINITY) ? 0.f : m_new;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < C::NC; ++c) {
        const float e = exp2f(s[i][c] - mu);
        rs += e;
        Ps[(ty * 4 + i) * C::SP + tx + 16 * c] = e;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off, 16);
      l[i] = l[i] * alpha + rs;
      m[i] = m_new;
#pragma unroll
      for (int d = 0; d < C::EPT; ++d) acc[i][d] *= alpha;
    }
    __syncthreads();

#pragma unroll
    for (int k4 = 0; k4 < C::BN; k4 += 4) {
      float pv[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) lds_vec<4>(Ps + (ty * 4 + i) * C::SP + k4, pv[i]);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        float vv[C::EPT];
        lds_vec<C::EPT>(Vs + (k4 + kk) * C::SV + C::EPT * tx, vv);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int d = 0; d < C::EPT; ++d) acc[i][d] = fmaf(pv[i][kk], vv[d], acc[i][d]);
      }
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = q0 + ty * 4 + i;
    if (row >= p.Sq) continue;
    const float inv_l = (l[i] > 0.f) ? 1.0f / l[i] : 0.f;
    float* og = p.o + split * p.o_split + (long long)b * p.o_sb + (long long)h * p.o_sh +
                (long long)row * p.o_ss + C::EPT * tx;
    if ((reinterpret_cast<uintptr_t>(og) & 7) == 0) {
#pragma unroll
      for (int d = 0; d < C::EPT; d += 2)
        *reinterpret_cast<float2*>(og + d) = make_float2(acc[i][d] * inv_l, acc[i][d + 1] * inv_l);
    } else {
#pragma unroll
      for (int d = 0; d < C::EPT; ++d) og[d] = acc[i][d] * inv_l;
    }
    if (p.lse != nullptr && tx == 0)
      p.lse[split * p.lse_split + ((long long)b * p.H + h) * p.Sq + row] =
          (l[i] > 0.f) ? (m[i] + log2f(l[i])) * 0.69314718055994531f : -INFINITY;
  }

  // Key splits: the split that completes the query block's count merges every split's partial
  // (w_s = exp(lse_s - max) / sum, O = sum_s w_s O_s, LSE = max + log(sum): the arithmetic of
  // lse_merge_kernel), reading the partials through L2.
  if (p.splits > 1 && p.blk_cnt != nullptr) {
    __shared__ int s_last;
    __threadfence();  // this split's partial is visible device-wide before it counts
    __syncthreads();
    if (tid == 0) {
      const unsigned prev = atomicAdd(p.blk_cnt + blk, 1u);
      const int last = prev == (unsigned)(p.splits - 1);
      if (last) p.blk_cnt[blk] = 0u;  // every split has counted: ready for the next launch
      s_last = last;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      const int row = q0 + ty * 4 + i;
      if (row >= p.Sq) continue;
      const long long r = ((long long)b * p.H + h) * p.Sq + row;
      float mx = -INFINITY;
      for (int sp = 0; sp < p.splits; ++sp) mx = fmaxf(mx, __ldcg(p.lse + sp * p.lse_split + r));
      float* of = p.o_final + (long long)b * p.of_sb + (long long)h * p.of_sh +
                  (long long)row * p.of_ss + C::EPT * tx;
      if (mx == -INFINITY) {
#pragma unroll
        for (int d = 0; d < C::EPT; ++d) of[d] = 0.f;
        if (p.lse_final != nullptr && tx == 0) p.lse_final[r] = -INFINITY;
        continue;
      }
      float wsum = 0.f;
      for (int sp = 0; sp < p.splits; ++sp) wsum += expf(__ldcg(p.lse + sp * p.lse_split + r) - mx);
      float a[C::EPT];
#pragma unroll
      for (int d = 0; d < C::EPT; ++d) a[d] = 0.f;
      const float* pb = p.o + (long long)b * p.o_sb + (long long)h * p.o_sh +
                        (long long)row * p.o_ss + C::EPT * tx;
      for (int sp = 0; sp < p.splits; ++sp) {
        const float w = expf(__ldcg(p.lse + sp * p.lse_split + r) - mx);
        const float* ps = pb + sp * p.o_split;
#pragma unroll
        for (int d = 0; d < C::EPT; d += 2) {
          const float2 v2 = __ldcg(reinterpret_cast<const float2*>(ps + d));
          a[d] = fmaf(w, v2.x, a[d]);
          a[d + 1] = fmaf(w, v2.y, a[d + 1]);
        }
      }
      const float inv = 1.0f / wsum;
#pragma unroll
      for (int d = 0; d < C::EPT; ++d) of[d] = a[d] * inv;
      if (p.lse_final != nullptr && tx == 0) p.lse_final[r] = mx + logf(wsum);
    }
  }
}

// ------------------------------------------------------------------------------------------
// LSE merge: one warp per (b, h, s) row.
// ------------------------------------------------------------------------------------------
template <typename OutT>
__device__ __forceinline__ void store_elem(OutT* p, float v);
template <>
__device__ __forceinline__ void store_elem<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store_elem<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ void store_elem<__half>(__half* p, float v) {
  *p = __float2half_rn(v);
}

template <typename OutT>
__global__ void __launch_bounds__(256) lse_merge_kernel(const float* __restrict__ o_parts,
                                                        const float* __restrict__ lse_parts,
                                                        int n_parts, OutT* o, float* lse_out,
                                                        int B, int H, int S, int D,
                                                        long long o_sb, long long o_sh,
                                                        long long o_ss) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long n_rows = (long long)B * H * S;
  if (row >= n_rows) return;
  const long long part_rows = n_rows;
  float mx = -INFINITY;
  for (int i = 0; i < n_parts; ++i) mx = fmaxf(mx, lse_parts[i * part_rows + row]);
  const long long s = row % S;
  const long long bh = row / S;
  const long long hh = bh % H, bb = bh / H;
  OutT* orow = o + bb * o_sb + hh * o_sh + s * o_ss;
  if (mx == -INFINITY) {
    for (int d = lane; d < D; d += 32) store_elem<OutT>(orow + d, 0.f);
    if (lse_out != nullptr && lane == 0) lse_out[row] = -INFINITY;
    return;
  }
  float wsum = 0.f;
  for (int i = 0; i < n_parts; ++i) wsum += expf(lse_parts[i * part_rows + row] - mx);
  const float inv = 1.0f / wsum;
  for (int d = lane; d < D; d += 32) {
    float a = 0.f;
    for (int i = 0; i < n_parts; ++i) {
      const float w = expf(lse_parts[i * part_rows + row] - mx);
      a = fmaf(w, o_parts[(i * part_rows + row) * D + d], a);
    }
    store_elem<OutT>(orow + d, a * inv);
  }
  if (lse_out != nullptr && lane == 0) lse_out[row] = mx + logf(wsum);
}

// (o_acc, lse_acc) <- merge((o_acc, lse_acc), (o_new, lse_new)), all fp32 contiguous.
__global__ void __launch_bounds__(256) lse_merge_acc_kernel(float* __restrict__ o_acc,
                                                            float* __restrict__ lse_acc,
                                                            const float* __restrict__ o_new,
                                                            const float* __restrict__ lse_new,
                                                            long long n_rows, int D) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const float la = lse_acc[row], ln = lse_new[row];
  const float mx = fmaxf(la, ln);
  if (ln == -INFINITY) return;  // nothing to add
  const float ea = (la == -INFINITY) ? 0.f : expf(la - mx);
  const float en = expf(ln - mx);
  const float sum = ea + en;
  const float wa = ea / sum, wn = en / sum;
  float* oa = o_acc + row * D;
  const float* on = o_new + row * D;
  for (int d = lane; d < D; d += 32) oa[d] = fmaf(wa, oa[d], wn * on[d]);
  __syncwarp();
  if (lane == 0) lse_acc[row] = mx + logf(sum);
}

template <typename OutT>
__global__ void __launch_bounds__(256) cast_rows_kernel(const float* __restrict__ src, OutT* dst,
                                                        long long n_rows, int H, int S, int D,
                                                        long long o_sb, long long o_sh,
                                                        long long o_ss) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const long long s = row % S, bh = row / S, hh = bh % H, bb = bh / H;
  OutT* orow = dst + bb * o_sb + hh * o_sh + s * o_ss;
  for (int d = lane; d < D; d += 32) store_elem<OutT>(orow + d, src[row * D + d]);
}

// Fills O with zeros and LSE with -inf (no admissible keys at all, e.g. Skv == 0).
template <typename OutT>
__global__ void __launch_bounds__(256) fill_empty_kernel(OutT* o, float* lse, long long n_rows,
                                                         int H, int S, int D, long long o_sb,
                                                         long long o_sh, long long o_ss) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const long long s = row % S, bh = row / S, hh = bh % H, bb = bh / H;
  OutT* orow = o + bb * o_sb + hh * o_sh + s * o_ss;
  for (int d = lane; d < D; d += 32) store_elem<OutT>(orow + d, 0.f);
  if (lse != nullptr && lane == 0) lse[row] = -INFINITY;
}

// Self-test of the bounded wait: thread 0 initialises an mbarrier that nothing arrives on and
// every thread waits on it with the given limit.
__global__ void wait_selftest_kernel(int* status, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const WaitCtx w{&abort_flag, status, timeout_ns};
  (void)mbar_wait(smem_u32(&bar), 0, w, 7);
}

}  // namespace mlxp
