// paged_attn.cuh — attention over a paged K/V pool (block tables), CUDA cores, split over keys.
//
// The reference's paged_attention (mlx_primitives/cache/paged_attention.py:44-320) gathers the
// pool blocks of each sequence into a dense (batch, max_blocks * block_size, heads, dim) copy
// and runs masked dense attention.  Here nothing is gathered: the kernel reads each block
// straight from the pool through the block table (key t of slot n is at position
// n * block_size + t).  Decode (one query row) is HBM-bound: every K/V byte of the context is
// read once.
//
// Work: one CTA per (query row (batch b, query i), head h, share of the block-table slots);
// its 4 warps take the share's slots round-robin.  Each warp streams its keys through a
// private 4-stage shared-memory ring filled by cp.async (every lane copies, and later reads
// back, exactly its own 8- or 16-byte pieces, so no barrier is needed between copy and use):
// three chunks of K and V are in flight per warp while the fourth is being used.
//
// Lanes and keys.  Each lane holds 4 consecutive elements of a row, so a row takes
// LPR = head_dim / 4 lanes and one chunk step covers KPW = 32 / LPR keys (1 for head_dim 128,
// 2 for 64, 4 for 32); a chunk is 8 such steps.  The LPR lanes of a key group finish the dot
// product with log2(LPR) xor-shuffles and keep their own online softmax; the KPW groups, then
// the 4 warps, are merged by log-sum-exp at the end.
//
// Admissible key positions of row i, as in the reference (paged_attention.py:161-199, 271-313):
// position < context_lens[b]; the slot's block id >= 0 (ids >= num_blocks count as missing too,
// so the pool is never read out of range); and, when causal with more than one query row,
// position <= i.  ALiBi adds slope[h] * (position - q_pos) to the scaled score, with
// q_pos = context_lens[b] for one query row and i otherwise.  A row with no admissible key
// gets zeros.
//
// Output: with one share per (row, head) the CTA writes the output row directly.  With several,
// each CTA writes its normalised fp32 partial and log2-sum-exp, bumps the (row, head) counter,
// and the CTA that arrives last merges all shares (from L2) and writes the output row — no
// second launch.  The counters are zeroed by the host before the launch.
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
  void* o;                        // output, element type of q
  float* o_part;                  // several shares: [share][B * Sq][H][D] fp32
  float* lse_part;                // several shares: [share][B * Sq][H] (log2 units)
  unsigned* counters;             // several shares: [B * Sq][H], zero at launch
  long long q_sb, q_sh, q_ss;     // element strides of q (batch, head, query)
  long long o_sb, o_sh, o_ss;     // element strides of o
  long long p_sb, p_st, p_sh;     // element strides of both pools (block, token, head)
  long long bt_stride;            // elements between block-table rows
  int B, H, Sq, D, kv_group, num_blocks, block_size, max_blocks;
  int blocks_per_split, splits, causal;
  float scale_log2;               // scale * log2(e)
};

constexpr int kPagedWarps = 4;
constexpr int kPagedStages = 4;
constexpr int kPagedSteps = 8;    // key steps (of KPW keys) per chunk

template <typename T>
__host__ __device__ constexpr int paged_stage_bytes(int D) {
  return 2 * kPagedSteps * (32 / (D / 4)) * D * (int)sizeof(T);  // K and V of one chunk
}
template <typename T>
__host__ __device__ constexpr int paged_smem_bytes(int D) {
  return kPagedWarps * kPagedStages * paged_stage_bytes<T>(D) + kPagedWarps * (D + 2) * 4;
}

// 4 * sizeof(T) bytes global -> shared; src_bytes = 0 writes zeros without reading global.
template <int BYTES>
__device__ __forceinline__ void cp_async_piece(uint32_t dst, const void* src, int src_bytes) {
  if constexpr (BYTES == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                 "r"(src_bytes) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(dst), "l"(src),
                 "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <typename T>
__device__ __forceinline__ void quad_to_f(const T* p, float (&x)[4]) {
  if constexpr (sizeof(T) == 4) {
    const float4 u = *reinterpret_cast<const float4*>(p);
    x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = to_f<T>(e[i]);
  }
}

// Walk over a warp's chunks: its block-table slots n = n0 + warp + j * kPagedWarps in order,
// missing blocks skipped, each block cut into chunks of `keys` positions.
struct PagedCursor {
  int n, t0, nt, pos0;
  long long base;  // element offset of the block (blk * p_sb) in the pools
  bool valid;
};

__device__ __forceinline__ void paged_next_block(const PagedParams& p, const int* bt, int n1,
                                                 int kv_end, PagedCursor& c) {
  for (;;) {
    c.n += kPagedWarps;
    c.pos0 = c.n * p.block_size;
    if (c.n >= n1 || c.pos0 >= kv_end) {
      c.valid = false;
      return;
    }
    const int blk = __ldg(bt + c.n);
    if (blk < 0 || blk >= p.num_blocks) continue;
    c.nt = min(p.block_size, kv_end - c.pos0);
    c.t0 = 0;
    c.base = (long long)blk * p.p_sb;
    c.valid = true;
    return;
  }
}

template <typename T, int LPR>
__global__ void __launch_bounds__(128) paged_attn_kernel(const PagedParams p) {
  constexpr int KPW = 32 / LPR;          // keys per step
  constexpr int KEYS = kPagedSteps * KPW;
  constexpr int D = LPR * 4;
  constexpr int PIECE = 4 * (int)sizeof(T);
  constexpr int STAGE = paged_stage_bytes<T>(D);
  constexpr int STEP = KPW * D * (int)sizeof(T);  // bytes of one step's rows
  extern __shared__ __align__(16) unsigned char psm[];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane / LPR;              // key group of this lane
  const int c = (lane % LPR) * 4;        // first element of the lane's quad
  const int h = blockIdx.x % p.H;
  const int row = blockIdx.x / p.H;      // b * Sq + i
  const int split = blockIdx.y;
  const int b = row / p.Sq, i = row - b * p.Sq;
  const int ctx = p.context_lens[b];
  int kv_end = ctx;                      // admissible positions are < kv_end
  if (p.causal && p.Sq > 1 && i + 1 < kv_end) kv_end = i + 1;
  const int q_pos = (p.Sq == 1) ? ctx : i;
  const int n0 = split * p.blocks_per_split;
  const int n1 = min(p.max_blocks, n0 + p.blocks_per_split);
  const int* bt = p.block_tables + (long long)b * p.bt_stride;
  const T* kp = static_cast<const T*>(p.k_pool) + (long long)(h / p.kv_group) * p.p_sh + c;
  const T* vp = static_cast<const T*>(p.v_pool) + (long long)(h / p.kv_group) * p.p_sh + c;
  unsigned char* ring = psm + warp * kPagedStages * STAGE;
  const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
  // this lane's piece of step u inside a stage: K at lane_off + u * STEP, V STAGE / 2 further
  const int lane_off = (g * D + c) * (int)sizeof(T);

  float q[4], o[4] = {0.f, 0.f, 0.f, 0.f};
  {
    float qv[4];
    quad_to_f<T>(static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh + i * p.q_ss + c, qv);
#pragma unroll
    for (int e = 0; e < 4; ++e) q[e] = qv[e] * p.scale_log2;
  }
  const float slope2 = p.alibi ? __ldg(p.alibi + h) * 1.4426950408889634f : 0.f;
  float m = -INFINITY, l = 0.f;

  PagedCursor pc{n0 + warp - kPagedWarps, 0, 0, 0, 0, false};
  paged_next_block(p, bt, n1, kv_end, pc);
  PagedCursor cc = pc;
  auto issue = [&](const PagedCursor& cur, int stage) {
    const uint32_t st = ring_s + stage * STAGE + lane_off;
#pragma unroll
    for (int u = 0; u < kPagedSteps; ++u) {
      const int t = cur.t0 + u * KPW + g;
      const bool ok = cur.valid && t < cur.nt;
      const long long off = ok ? cur.base + (long long)t * p.p_st : 0;
      cp_async_piece<PIECE>(st + u * STEP, kp + off, ok ? PIECE : 0);
      cp_async_piece<PIECE>(st + STAGE / 2 + u * STEP, vp + off, ok ? PIECE : 0);
    }
  };
  auto advance = [&](PagedCursor& cur) {
    if (!cur.valid) return;
    cur.t0 += KEYS;
    if (cur.t0 >= cur.nt) paged_next_block(p, bt, n1, kv_end, cur);
  };
#pragma unroll
  for (int s = 0; s < kPagedStages - 1; ++s) {
    issue(pc, s);
    cp_async_commit();
    advance(pc);
  }
  int stage = 0;
  while (cc.valid) {
    issue(pc, (stage + kPagedStages - 1) % kPagedStages);  // refills the stage used last
    cp_async_commit();
    advance(pc);
    cp_async_wait<kPagedStages - 1>();  // this lane's pieces of `stage` have landed
    const unsigned char* st = ring + stage * STAGE + lane_off;
    float s[kPagedSteps];
#pragma unroll
    for (int u = 0; u < kPagedSteps; ++u) {
      float kx[4];
      quad_to_f<T>(reinterpret_cast<const T*>(st + u * STEP), kx);
      float a = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) a = fmaf(q[e], kx[e], a);
      s[u] = a;
    }
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) {
#pragma unroll
      for (int u = 0; u < kPagedSteps; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
    }
    float m_blk = -INFINITY;
#pragma unroll
    for (int u = 0; u < kPagedSteps; ++u) {
      const int t = cc.t0 + u * KPW + g;
      s[u] = (t < cc.nt) ? fmaf(slope2, (float)(cc.pos0 + t - q_pos), s[u]) : -INFINITY;
      m_blk = fmaxf(m_blk, s[u]);
    }
    const float m_new = fmaxf(m, m_blk);
    const float m_use = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = ex2_approx(m - m_use);  // 0 while m = -inf
    l *= alpha;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] *= alpha;
#pragma unroll
    for (int u = 0; u < kPagedSteps; ++u) {
      const float pw = ex2_approx(s[u] - m_use);  // 0 for masked keys (their V rows are zero)
      float vx[4];
      quad_to_f<T>(reinterpret_cast<const T*>(st + STAGE / 2 + u * STEP), vx);
      l += pw;
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = fmaf(pw, vx[e], o[e]);
    }
    m = m_new;
    advance(cc);
    stage = (stage + 1) % kPagedStages;
  }
  cp_async_wait<0>();

  // merge the KPW key groups of the warp (lanes g * LPR + j, same j) by log-sum-exp
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
  // merge the warps through shared memory (after the rings: [warp][D + 2] floats)
  float* red = reinterpret_cast<float*>(psm + kPagedWarps * kPagedStages * STAGE);
  if (lane < LPR) {
#pragma unroll
    for (int e = 0; e < 4; ++e) red[warp * (D + 2) + c + e] = o[e];
    if (lane == 0) {
      red[warp * (D + 2) + D] = m;
      red[warp * (D + 2) + D + 1] = l;
    }
  }
  __syncthreads();
  if (warp != 0) return;
  float mt = -INFINITY;
#pragma unroll
  for (int w = 0; w < kPagedWarps; ++w) mt = fmaxf(mt, red[w * (D + 2) + D]);
  const float mu = mt == -INFINITY ? 0.f : mt;
  float lt = 0.f, ot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < kPagedWarps; ++w) {
    const float f = ex2_approx(red[w * (D + 2) + D] - mu);
    lt = fmaf(red[w * (D + 2) + D + 1], f, lt);
    if (lane < LPR) {
#pragma unroll
      for (int e = 0; e < 4; ++e) ot[e] = fmaf(red[w * (D + 2) + c + e], f, ot[e]);
    }
  }
  const float inv = lt > 0.f ? 1.f / lt : 0.f;
  T* op = static_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh + i * p.o_ss + c;
  if (p.splits == 1) {
    if (lane < LPR) {
#pragma unroll
      for (int e = 0; e < 4; ++e) op[e] = from_f<T>(ot[e] * inv);
    }
    return;
  }
  const long long stride = (long long)p.B * p.Sq * p.H;  // rows of one share
  const long long r0 = (long long)row * p.H + h;
  const long long prow = split * stride + r0;
  if (lane < LPR)
    *reinterpret_cast<float4*>(p.o_part + prow * p.D + c) =
        make_float4(ot[0] * inv, ot[1] * inv, ot[2] * inv, ot[3] * inv);
  if (lane == 0) p.lse_part[prow] = lt > 0.f ? mt + __log2f(lt) : -INFINITY;
  __threadfence();
  __syncwarp();
  if (lane == 0) s_last = atomicAdd(p.counters + r0, 1u) == (unsigned)(p.splits - 1);
  __syncwarp();
  if (!s_last) return;
  // the last share of (row, h) to finish: every other share is written, merge them all
  __threadfence();
  float mx = -INFINITY;
  for (int s2 = lane; s2 < p.splits; s2 += 32) mx = fmaxf(mx, __ldcg(p.lse_part + s2 * stride + r0));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float mu2 = mx == -INFINITY ? 0.f : mx;
  float wsum = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
  for (int s2 = 0; s2 < p.splits; ++s2) {
    const float w = ex2_approx(__ldcg(p.lse_part + s2 * stride + r0) - mu2);
    wsum += w;
    if (lane < LPR) {
      const float4 v4 = __ldcg(reinterpret_cast<const float4*>(p.o_part + (s2 * stride + r0) * p.D + c));
      acc[0] = fmaf(w, v4.x, acc[0]);
      acc[1] = fmaf(w, v4.y, acc[1]);
      acc[2] = fmaf(w, v4.z, acc[2]);
      acc[3] = fmaf(w, v4.w, acc[3]);
    }
  }
  const float inv2 = wsum > 0.f ? 1.f / wsum : 0.f;
  if (lane < LPR) {
#pragma unroll
    for (int e = 0; e < 4; ++e) op[e] = from_f<T>(acc[e] * inv2);
  }
}

}  // namespace mlxp
