// attn_bwd.cuh — attention backward (dQ, dK, dV) on CUDA cores, fp32 arithmetic.
//
// The reference differentiates its forward with MLX autodiff (mlx_primitives/attention/
// flash.py:52-316 under mx.grad / mx.vjp, checked by tests/gradients/
// test_numerical_gradients.py:20-270); here the gradient of the same function is computed
// from the forward's saved output O and log-sum-exp L (natural log, one per query row):
//   P_ij  = exp(scale * q_i . k_j - L_i)             (admissible (i, j); 0 otherwise)
//   dV_j  = sum_i P_ij dO_i
//   dP_ij = dO_i . v_j,   Delta_i = dO_i . O_i,   dS_ij = P_ij (dP_ij - Delta_i)
//   dQ_i  = scale * sum_j dS_ij k_j,   dK_j = scale * sum_i dS_ij q_i
// Masks are the forward's (attn_common.cuh, absolute positions).  Grouped K/V heads sum the
// dK/dV contributions of every query head that reads them.
//
// Three launches: bwd_delta_kernel (Delta), bwd_dkdv_kernel (one CTA per (batch, K/V head,
// 64-key tile), looping over the query tiles and query heads that see the tile) and
// bwd_dq_kernel (one CTA per (batch, head, 64-query tile), looping over key tiles).  Each
// output element has exactly one writer: no atomics, deterministic.  CTA = 256 threads as a
// 16 x 16 grid with 4 x (BN/16) register micro-tiles, as in the fp32 forward kernel.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "attn_common.cuh"

namespace mlxp {

struct BwdParams {
  int B, H, Sq, Skv, kv_group;
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  const float* lse;  // [B][H][Sq]
  float* delta;      // [B][H][Sq] (workspace)
  void* dq;
  void* dk;
  void* dv;
  long long q_sb, q_sh, q_ss, k_sb, k_sh, k_ss, v_sb, v_sh, v_ss, o_sb, o_sh, o_ss;
  long long do_sb, do_sh, do_ss, dq_sb, dq_sh, dq_ss, dk_sb, dk_sh, dk_ss, dv_sb, dv_sh, dv_ss;
  float scale, scale_log2;
  MaskSpec mask;
};

template <typename T>
__device__ __forceinline__ float bwd_ld(const T* p) {
  if constexpr (sizeof(T) == 4) return *p;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(*p);
  else return __half2float(*p);
}
template <typename T>
__device__ __forceinline__ void bwd_st(T* p, float v) {
  if constexpr (sizeof(T) == 4) *p = v;
  else if constexpr (std::is_same<T, __nv_bfloat16>::value) *p = __float2bfloat16_rn(v);
  else *p = __float2half_rn(v);
}

// Admissible query-index range [lo, hi) of the key indices [c0, c1) (c1 > c0), within [0, Sq).
__host__ __device__ inline void q_index_range(const MaskSpec& m, long long c0, long long c1,
                                              long long Sq, long long& lo, long long& hi) {
  const long long kmin = c0 + m.kv_off, kmax = c1 - 1 + m.kv_off;
  lo = 0;
  hi = Sq;
  if (m.causal && kmin - m.q_off > lo) lo = kmin - m.q_off;                 // qpos >= kpos
  if (m.wr >= 0 && kmin - m.wr - m.q_off > lo) lo = kmin - m.wr - m.q_off;  // kpos - qpos <= wr
  if (m.wl >= 0 && kmax + m.wl - m.q_off + 1 < hi) hi = kmax + m.wl - m.q_off + 1;
  if (hi < lo) hi = lo;
}

// Delta_i = dO_i . O_i: one warp per (b, h, i) row.
template <typename T>
__global__ void __launch_bounds__(256) bwd_delta_kernel(const BwdParams p, int D) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= (long long)p.B * p.H * p.Sq) return;
  const long long i = row % p.Sq, bh = row / p.Sq;
  const long long h = bh % p.H, b = bh / p.H;
  const T* o = static_cast<const T*>(p.o) + b * p.o_sb + h * p.o_sh + i * p.o_ss;
  const T* g = static_cast<const T*>(p.dout) + b * p.do_sb + h * p.do_sh + i * p.do_ss;
  float a = 0.f;
  for (int d = lane; d < D; d += 32) a = fmaf(bwd_ld(o + d), bwd_ld(g + d), a);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
  if (lane == 0) p.delta[row] = a;
}

template <int D>
struct BwdCfg {
  static constexpr int BM = 64;      // query rows per tile
  static constexpr int BN = 64;      // key rows per tile
  static constexpr int ND = D / 16;  // head-dim columns per thread
  static constexpr int SP = D + 1;   // padded pitch of rows read by column (K, V / Q, dO)
  static constexpr int ST = BN + 1;  // pitch of the P / dS tiles
  static_assert(D % 16 == 0 && D <= 128, "head_dim multiple of 16, <= 128");
};

// Rows [r0, r0 + n) of a [seq][D] operand (element strides) -> fp32 smem with pitch `pitch`;
// rows past `limit` are zero.
template <typename T, int D>
__device__ __forceinline__ void bwd_load_rows(float* dst, int pitch, const T* src, long long ss,
                                              long long r0, int n, long long limit) {
  for (int idx = threadIdx.x; idx < n * D; idx += blockDim.x) {
    const int r = idx / D, c = idx - r * D;
    const long long row = r0 + r;
    dst[r * pitch + c] = row < limit ? bwd_ld(src + row * ss + c) : 0.f;
  }
}

// s[i][c] = sum_d A[ty*4+i][d] * B[tx+16c][d]  (A pitch pa, B pitch pb)
template <int D>
__device__ __forceinline__ void bwd_tile_dot(float (&s)[4][4], const float* A, int pa,
                                             const float* Bm, int pb, int ty, int tx) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) s[i][c] = 0.f;
#pragma unroll 4
  for (int d = 0; d < D; ++d) {
    float a[4], bb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = A[(ty * 4 + i) * pa + d];
#pragma unroll
    for (int c = 0; c < 4; ++c) bb[c] = Bm[(tx + 16 * c) * pb + d];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[i][c] = fmaf(a[i], bb[c], s[i][c]);
  }
}

// P and dS of one (64 query x 64 key) tile: thread (ty, tx) holds queries ty*4+i (local
// rows of the query tile starting at q0) and keys tx+16c (of the key tile starting at c0).
template <int D>
__device__ __forceinline__ void bwd_p_ds(const BwdParams& p, const float* Qs, const float* dOs,
                                         const float* Ks, const float* Vs, const float* Ls,
                                         const float* Dl, long long q0, long long c0, int ty,
                                         int tx, float (&P)[4][4], float (&dS)[4][4]) {
  using C = BwdCfg<D>;
  bwd_tile_dot<D>(P, Qs, C::SP, Ks, C::SP, ty, tx);
  float dP[4][4];
  bwd_tile_dot<D>(dP, dOs, C::SP, Vs, C::SP, ty, tx);
  const bool full = tile_is_full(p.mask, q0, q0 + C::BM, c0, c0 + C::BN);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = ty * 4 + i;
    int c_lo = 0, c_hi = C::BN - 1;
    if (!full) row_col_interval(p.mask, q0 + r, c0, C::BN, c_lo, c_hi);
    const float L2 = Ls[r];  // LSE in log2 units; -inf for rows without keys (and past Sq)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int col = tx + 16 * c;
      const bool ok = col >= c_lo && col <= c_hi && L2 != -INFINITY;
      const float pr = ok ? exp2f(fmaf(P[i][c], p.scale_log2, -L2)) : 0.f;
      P[i][c] = pr;
      dS[i][c] = pr * (dP[i][c] - Dl[r]);
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(256) bwd_dkdv_kernel(const BwdParams p) {
  using C = BwdCfg<D>;
  extern __shared__ float bsm[];
  float* Ks = bsm;                        // [BN][SP]
  float* Vs = Ks + C::BN * C::SP;         // [BN][SP]
  float* Qs = Vs + C::BN * C::SP;         // [BM][SP]
  float* dOs = Qs + C::BM * C::SP;        // [BM][SP]
  float* Ps = dOs + C::BM * C::SP;        // [BM][ST]
  float* dSs = Ps + C::BM * C::ST;        // [BM][ST]
  float* Ls = dSs + C::BM * C::ST;        // [BM] (log2 units)
  float* Dl = Ls + C::BM;                 // [BM]

  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int n_kt = (p.Skv + C::BN - 1) / C::BN;
  const int Hkv = p.H / p.kv_group;
  const int kt = blockIdx.x % n_kt;
  const int bhk = blockIdx.x / n_kt;
  const int hk = bhk % Hkv, b = bhk / Hkv;
  const long long c0 = (long long)kt * C::BN;

  const T* kg = static_cast<const T*>(p.k) + b * p.k_sb + hk * p.k_sh;
  const T* vg = static_cast<const T*>(p.v) + b * p.v_sb + hk * p.v_sh;
  bwd_load_rows<T, D>(Ks, C::SP, kg, p.k_ss, c0, C::BN, p.Skv);
  bwd_load_rows<T, D>(Vs, C::SP, vg, p.v_ss, c0, C::BN, p.Skv);

  float adk[4][C::ND], adv[4][C::ND];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int d = 0; d < C::ND; ++d) adk[i][d] = adv[i][d] = 0.f;

  long long qlo, qhi;
  q_index_range(p.mask, c0, c0 + C::BN < p.Skv ? c0 + C::BN : p.Skv, p.Sq, qlo, qhi);
  const int t_lo = (int)(qlo / C::BM), t_hi = (int)((qhi + C::BM - 1) / C::BM);
  for (int g = 0; g < p.kv_group; ++g) {
    const int h = hk * p.kv_group + g;
    const T* qg = static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
    const T* dog = static_cast<const T*>(p.dout) + b * p.do_sb + h * p.do_sh;
    const float* lg = p.lse + ((long long)b * p.H + h) * p.Sq;
    const float* dg = p.delta + ((long long)b * p.H + h) * p.Sq;
    for (int qt = t_lo; qt < t_hi; ++qt) {
      const long long q0 = (long long)qt * C::BM;
      __syncthreads();  // previous tile's smem fully consumed (K/V stored, first time)
      bwd_load_rows<T, D>(Qs, C::SP, qg, p.q_ss, q0, C::BM, p.Sq);
      bwd_load_rows<T, D>(dOs, C::SP, dog, p.do_ss, q0, C::BM, p.Sq);
      if (tid < C::BM) {
        const long long r = q0 + tid;
        Ls[tid] = r < p.Sq ? lg[r] * 1.4426950408889634f : -INFINITY;
        Dl[tid] = r < p.Sq ? dg[r] : 0.f;
      }
      __syncthreads();
      float P[4][4], dS[4][4];
      bwd_p_ds<D>(p, Qs, dOs, Ks, Vs, Ls, Dl, q0, c0, ty, tx, P, dS);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          Ps[(ty * 4 + i) * C::ST + tx + 16 * c] = P[i][c];
          dSs[(ty * 4 + i) * C::ST + tx + 16 * c] = dS[i][c];
        }
      __syncthreads();
      // dV[key ty*4+i][d] += sum_q P[q][key] dO[q][d];  dK likewise with dS and Q
#pragma unroll 4
      for (int qq = 0; qq < C::BM; ++qq) {
        float pv[4], sv[4], gv[C::ND], qv[C::ND];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pv[i] = Ps[qq * C::ST + ty * 4 + i];
          sv[i] = dSs[qq * C::ST + ty * 4 + i];
        }
#pragma unroll
        for (int d = 0; d < C::ND; ++d) {
          gv[d] = dOs[qq * C::SP + tx + 16 * d];
          qv[d] = Qs[qq * C::SP + tx + 16 * d];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int d = 0; d < C::ND; ++d) {
            adv[i][d] = fmaf(pv[i], gv[d], adv[i][d]);
            adk[i][d] = fmaf(sv[i], qv[d], adk[i][d]);
          }
      }
    }
  }
  T* dkg = static_cast<T*>(p.dk) + b * p.dk_sb + hk * p.dk_sh;
  T* dvg = static_cast<T*>(p.dv) + b * p.dv_sb + hk * p.dv_sh;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const long long key = c0 + ty * 4 + i;
    if (key >= p.Skv) continue;
#pragma unroll
    for (int d = 0; d < C::ND; ++d) {
      bwd_st<T>(dkg + key * p.dk_ss + tx + 16 * d, adk[i][d] * p.scale);
      bwd_st<T>(dvg + key * p.dv_ss + tx + 16 * d, adv[i][d]);
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(256) bwd_dq_kernel(const BwdParams p) {
  using C = BwdCfg<D>;
  extern __shared__ float bsm[];
  float* Qs = bsm;                        // [BM][SP]
  float* dOs = Qs + C::BM * C::SP;        // [BM][SP]
  float* Ks = dOs + C::BM * C::SP;        // [BN][SP]
  float* Vs = Ks + C::BN * C::SP;         // [BN][SP]
  float* dSs = Vs + C::BN * C::SP;        // [BM][ST]
  float* Ls = dSs + C::BM * C::ST;        // [BM]
  float* Dl = Ls + C::BM;                 // [BM]

  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int n_qt = (p.Sq + C::BM - 1) / C::BM;
  const int qt = blockIdx.x % n_qt;
  const int bh = blockIdx.x / n_qt;
  const int h = bh % p.H, b = bh / p.H;
  const int hk = h / p.kv_group;
  const long long q0 = (long long)qt * C::BM;

  const T* qg = static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
  const T* dog = static_cast<const T*>(p.dout) + b * p.do_sb + h * p.do_sh;
  const T* kg = static_cast<const T*>(p.k) + b * p.k_sb + hk * p.k_sh;
  const T* vg = static_cast<const T*>(p.v) + b * p.v_sb + hk * p.v_sh;
  bwd_load_rows<T, D>(Qs, C::SP, qg, p.q_ss, q0, C::BM, p.Sq);
  bwd_load_rows<T, D>(dOs, C::SP, dog, p.do_ss, q0, C::BM, p.Sq);
  if (tid < C::BM) {
    const long long r = q0 + tid;
    const long long row = ((long long)b * p.H + h) * p.Sq + r;
    Ls[tid] = r < p.Sq ? p.lse[row] * 1.4426950408889634f : -INFINITY;
    Dl[tid] = r < p.Sq ? p.delta[row] : 0.f;
  }

  float adq[4][C::ND];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int d = 0; d < C::ND; ++d) adq[i][d] = 0.f;

  const long long r1 = q0 + C::BM < p.Sq ? q0 + C::BM : p.Sq;
  int tlo, thi;
  kv_tile_range(p.mask, q0, r1, C::BN, tlo, thi);
  for (int jt = tlo; jt < thi; ++jt) {
    const long long c0 = (long long)jt * C::BN;
    __syncthreads();
    bwd_load_rows<T, D>(Ks, C::SP, kg, p.k_ss, c0, C::BN, p.Skv);
    bwd_load_rows<T, D>(Vs, C::SP, vg, p.v_ss, c0, C::BN, p.Skv);
    __syncthreads();
    float P[4][4], dS[4][4];
    bwd_p_ds<D>(p, Qs, dOs, Ks, Vs, Ls, Dl, q0, c0, ty, tx, P, dS);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) dSs[(ty * 4 + i) * C::ST + tx + 16 * c] = dS[i][c];
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < C::BN; ++kk) {
      float sv[4], kv[C::ND];
#pragma unroll
      for (int i = 0; i < 4; ++i) sv[i] = dSs[(ty * 4 + i) * C::ST + kk];
#pragma unroll
      for (int d = 0; d < C::ND; ++d) kv[d] = Ks[kk * C::SP + tx + 16 * d];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int d = 0; d < C::ND; ++d) adq[i][d] = fmaf(sv[i], kv[d], adq[i][d]);
    }
  }
  T* dqg = static_cast<T*>(p.dq) + b * p.dq_sb + h * p.dq_sh;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const long long r = q0 + ty * 4 + i;
    if (r >= p.Sq) continue;
#pragma unroll
    for (int d = 0; d < C::ND; ++d) bwd_st<T>(dqg + r * p.dq_ss + tx + 16 * d, adq[i][d] * p.scale);
  }
}

template <int D>
constexpr int bwd_dkdv_smem() {
  using C = BwdCfg<D>;
  return 4 * (4 * C::BN * C::SP + 2 * C::BM * C::ST + 2 * C::BM);
}
template <int D>
constexpr int bwd_dq_smem() {
  using C = BwdCfg<D>;
  return 4 * (4 * C::BN * C::SP + C::BM * C::ST + 2 * C::BM);
}

}  // namespace mlxp
