// paged_attn.cuh — attention over a paged K/V pool (block tables), CUDA cores, split over keys.
//
// The reference's paged_attention (mlx_primitives/cache/paged_attention.py:44-320) gathers the
// pool blocks of each sequence into a dense (batch, max_blocks * block_size, heads, dim) copy
// and runs masked dense attention.  Here nothing is gathered: every CTA takes one query row
// (batch b, query i) and a contiguous share of that sequence's block-table slots, and reads each
// block straight from the pool (key t of slot n is at position n * block_size + t).  Decode
// (one query row) is HBM-bound: every K/V byte of the context is read once, in 8- or 16-byte
// vectors per lane, with a batch of K and V rows in flight per warp before any is used.
//
// Lanes and keys.  A warp owns one head at a time.  Each lane holds 4 consecutive elements of
// a row, so a row takes LPR = head_dim / 4 lanes and one warp-wide load covers KPW = 32 / LPR
// keys (1 for head_dim 128, 2 for 64, 4 for 32).  The LPR lanes of a key group finish the dot
// product with log2(LPR) xor-shuffles and keep their own online softmax over the keys they
// see; the KPW groups are merged by log-sum-exp at the end of the share.
//
// Admissible key positions of row i, as in the reference (paged_attention.py:161-199, 271-313):
// position < context_lens[b]; the slot's block id >= 0 (ids >= num_blocks count as missing too,
// so the pool is never read out of range); and, when causal with more than one query row,
// position <= i.  ALiBi adds slope[h] * (position - q_pos) to the scaled score, with
// q_pos = context_lens[b] for one query row and i otherwise.  A row with no admissible key
// writes zeros and LSE -inf.
//
// Output: with one share per row the CTA writes the row in the output type directly; with
// several it writes a normalised fp32 partial and its log-sum-exp in lse_merge_kernel's layout
// ([share][batch][head][query] rows), and that kernel combines the shares.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace mlxp {

struct PagedParams {
  const void* q;
  const void* k_pool;
  const void* v_pool;
  const int* block_tables;
  const int* context_lens;
  const float* alibi;             // nullable, [H] (natural units of the scaled score)
  void* o;                        // direct output (one share), element type of q
  float* o_part;                  // several shares: [share][B][H][Sq][D] fp32
  float* lse_part;                // several shares: [share][B][H][Sq]
  long long q_sb, q_sh, q_ss;     // element strides of q (batch, head, query)
  long long o_sb, o_sh, o_ss;     // element strides of o
  long long p_sb, p_st, p_sh;     // element strides of both pools (block, token, head)
  long long bt_stride;            // elements between block-table rows
  int B, H, Sq, D, kv_group, num_blocks, block_size, max_blocks;
  int blocks_per_split, causal;
  float scale_log2;               // scale * log2(e)
};

template <int BYTES>
struct RawVec;
template <>
struct RawVec<8> { using type = uint2; };
template <>
struct RawVec<16> { using type = uint4; };

// Four consecutive elements of a K or V row, kept in the storage type until used.
template <typename T>
struct Quad {
  using V = typename RawVec<4 * (int)sizeof(T)>::type;
  V v;
  __device__ __forceinline__ void load(const T* p) { v = __ldg(reinterpret_cast<const V*>(p)); }
  __device__ __forceinline__ void zero() { v = V{}; }
  __device__ __forceinline__ float operator[](int e) const {
    return to_f<T>(reinterpret_cast<const T*>(&v)[e]);
  }
};

// grid (B * Sq, shares), 256 threads = 8 warps; warp w handles heads w, w + 8, ...
// LPR = head_dim / 4 lanes per key row; NB K and V rows per lane in flight per batch.
template <typename T, int LPR>
__global__ void __launch_bounds__(256, 3) paged_attn_kernel(const PagedParams p) {
  constexpr int KPW = 32 / LPR;                 // keys per warp-wide load
  constexpr int NB = 16 / sizeof(T);            // loads per batch: 32 registers of K and V
  constexpr int KEYS = NB * KPW;                // keys per batch
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane / LPR;                     // key group of this lane
  const int c = (lane % LPR) * 4;               // first element of the lane's quad
  const int row = blockIdx.x;                   // b * Sq + i
  const int split = blockIdx.y;
  const int b = row / p.Sq, i = row - b * p.Sq;
  const int ctx = p.context_lens[b];
  int kv_end = ctx;                             // admissible positions are < kv_end
  if (p.causal && p.Sq > 1 && i + 1 < kv_end) kv_end = i + 1;
  const int q_pos = (p.Sq == 1) ? ctx : i;
  const int n0 = split * p.blocks_per_split;
  const int n1 = min(p.max_blocks, n0 + p.blocks_per_split);
  const int* bt = p.block_tables + (long long)b * p.bt_stride;
  const T* kp = static_cast<const T*>(p.k_pool);
  const T* vp = static_cast<const T*>(p.v_pool);
  for (int h = warp; h < p.H; h += 8) {
    float q[4], o[4] = {0.f, 0.f, 0.f, 0.f};
    {
      Quad<T> qv;
      qv.load(static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh + i * p.q_ss + c);
#pragma unroll
      for (int e = 0; e < 4; ++e) q[e] = qv[e] * p.scale_log2;
    }
    const float slope2 = p.alibi ? __ldg(p.alibi + h) * 1.4426950408889634f : 0.f;
    const long long head_off = (long long)(h / p.kv_group) * p.p_sh + c;
    float m = -INFINITY, l = 0.f;
    for (int n = n0; n < n1; ++n) {
      const int pos0 = n * p.block_size;
      if (pos0 >= kv_end) break;
      const int blk = __ldg(bt + n);
      if (blk < 0 || blk >= p.num_blocks) continue;
      const int nt = min(p.block_size, kv_end - pos0);
      const T* kb = kp + (long long)blk * p.p_sb + head_off;
      const T* vb = vp + (long long)blk * p.p_sb + head_off;
      for (int t0 = 0; t0 < nt; t0 += KEYS) {
        Quad<T> kr[NB], vr[NB];
#pragma unroll
        for (int u = 0; u < NB; ++u) {
          const int t = t0 + u * KPW + g;
          if (t < nt) {
            kr[u].load(kb + (long long)t * p.p_st);
            vr[u].load(vb + (long long)t * p.p_st);
          } else {
            kr[u].zero();
            vr[u].zero();
          }
        }
        float s[NB];
#pragma unroll
        for (int u = 0; u < NB; ++u) {
          float a = 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) a = fmaf(q[e], kr[u][e], a);
          s[u] = a;
        }
#pragma unroll
        for (int off = LPR / 2; off > 0; off >>= 1) {
#pragma unroll
          for (int u = 0; u < NB; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
        }
        float m_blk = -INFINITY;
#pragma unroll
        for (int u = 0; u < NB; ++u) {
          const int t = t0 + u * KPW + g;
          s[u] = (t < nt) ? fmaf(slope2, (float)(pos0 + t - q_pos), s[u]) : -INFINITY;
          m_blk = fmaxf(m_blk, s[u]);
        }
        const float m_new = fmaxf(m, m_blk);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = ex2_approx(m - m_use);  // 0 while m = -inf
        l *= alpha;
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] *= alpha;
#pragma unroll
        for (int u = 0; u < NB; ++u) {
          const float pw = ex2_approx(s[u] - m_use);  // 0 for masked keys
          l += pw;
#pragma unroll
          for (int e = 0; e < 4; ++e) o[e] = fmaf(pw, vr[u][e], o[e]);
        }
        m = m_new;
      }
    }
    // merge the KPW key groups (lanes g * LPR + j, same j) by log-sum-exp
    if (KPW > 1) {
      float mt = m;
#pragma unroll
      for (int off = LPR; off < 32; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float f = ex2_approx(m - (mt == -INFINITY ? 0.f : mt));
      l *= f;
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] *= f;
#pragma unroll
      for (int off = LPR; off < 32; off <<= 1) {
        l += __shfl_xor_sync(0xffffffffu, l, off);
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] += __shfl_xor_sync(0xffffffffu, o[e], off);
      }
      m = mt;
    }
    const bool valid = l > 0.f;
    const float inv_l = valid ? 1.f / l : 0.f;
    if (lane < LPR) {
      if (p.o_part == nullptr) {
        T* op = static_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh + i * p.o_ss + c;
#pragma unroll
        for (int e = 0; e < 4; ++e) op[e] = from_f<T>(o[e] * inv_l);
      } else {
        const long long prow = (((long long)split * p.B + b) * p.H + h) * p.Sq + i;
        float4 v4 = make_float4(o[0] * inv_l, o[1] * inv_l, o[2] * inv_l, o[3] * inv_l);
        *reinterpret_cast<float4*>(p.o_part + prow * p.D + c) = v4;
        if (lane == 0) p.lse_part[prow] = valid ? (m + __log2f(l)) * 0.69314718055994531f : -INFINITY;
      }
    }
  }
}

}  // namespace mlxp
