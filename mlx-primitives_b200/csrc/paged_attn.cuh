// paged_attn.cuh — attention over a paged K/V pool (block tables), CUDA cores, split over keys.
//
// The reference's paged_attention (mlx_primitives/cache/paged_attention.py:44-320) gathers the
// pool blocks of each sequence into a dense (batch, max_blocks * block_size, heads, dim) copy
// and runs masked dense attention.  Here nothing is gathered: the kernel reads each block
// straight from the pool through the block table (key t of slot n is at position
// n * block_size + t).  Decode (one query row) is HBM-bound: every K/V byte of the context is
// read once.
//
// Work: the (query row, head, block-table slot) space, flattened with the slot innermost, is
// cut into G equal contiguous ranges, one per CTA ("stream-K"): with G = the resident CTA count
// every SM gets the same number of blocks and the whole grid runs as one wave.  A CTA's range
// covers the tail of one (row, head) pair, whole pairs and the head of another; for each pair
// segment its 4 warps take the segment's slots round-robin.  Each warp streams its keys through a
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
// Output: a segment that covers its whole pair writes the output row directly.  Otherwise the
// CTA writes the segment's normalised fp32 partial and log2-sum-exp into the pair's slot for
// that CTA, adds the segment's block count to the pair's counter, and the CTA whose addition
// completes the pair merges all its partials (from L2) and writes the output row — no second
// launch.  The counters are zeroed by the host before the launch.
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
  float* o_part;                  // [pair][slot][D] fp32, slot = CTA - first CTA of the pair
  float* lse_part;                // [pair][slot] (log2 units)
  unsigned* counters;             // [pair] blocks done, zero at launch (pair = row * H + h)
  long long q_sb, q_sh, q_ss;     // element strides of q (batch, head, query)
  long long o_sb, o_sh, o_ss;     // element strides of o
  long long p_sb, p_st, p_sh;     // element strides of both pools (block, token, head)
  long long bt_stride;            // elements between block-table rows
  int B, H, Sq, D, kv_group, num_blocks, block_size, max_blocks;
  int causal;
  int* status;                    // device status word (bounded waits of the TMA kernel)
  unsigned long long timeout_ns;
  int grid;                       // CTAs; CTA c owns flat slots [c * total / grid, ...)
  int max_parts;                  // partial slots per pair
  long long total;                // pairs * max_blocks
  float scale_log2;               // scale * log2(e)
};

// CTA whose range holds flat slot f: start(c) = floor(c * total / grid) <= f.
__host__ __device__ inline long long paged_cta_of(long long f, long long total, long long grid) {
  return ((f + 1) * grid - 1) / total;
}

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
  int blk;
};

template <int NW>
__device__ __forceinline__ void paged_next_block_w(const PagedParams& p, const int* bt, int n1,
                                                   int kv_end, PagedCursor& c) {
  for (;;) {
    c.n += NW;
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
    c.blk = blk;
    c.valid = true;
    return;
  }
}

__device__ __forceinline__ void paged_next_block(const PagedParams& p, const int* bt, int n1,
                                                 int kv_end, PagedCursor& c) {
  paged_next_block_w<kPagedWarps>(p, bt, n1, kv_end, c);
}

// End of a segment, called by every thread of the CTA: merge the key groups of each warp,
// then the NW warps (through `red`, [NW][D + 2] floats), then write the output row (a whole
// pair) or the segment's partial, and, in the CTA that completes a pair, merge its partials.
// With the CTA's abort flag raised (a bounded wait gave up) nothing is written.
template <typename T, int LPR, int NW>
__device__ __forceinline__ void paged_epilogue(const PagedParams& p, float* red, int* s_last_p,
                                               int warp, int lane, float m, float l, float (&o)[4],
                                               int pair, int b, int h, int i, int n_a, int n_b,
                                               const int* abort_flag) {
  constexpr int KPW = 32 / LPR;
  constexpr int D = LPR * 4;
  const int c = (lane % LPR) * 4;
  const int mb = p.max_blocks;
  int& s_last = *s_last_p;
  // merge the KPW key groups of the warp (lanes g * LPR + j, same j) by log-sum-exp
  if (KPW > 1) {
    float mt = m;
#pragma unroll
    for (int off = LPR; off < 32; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
    const float fct = ex2_approx(m - (mt == -INFINITY ? 0.f : mt));
    l *= fct;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] *= fct;
#pragma unroll
    for (int off = LPR; off < 32; off <<= 1) {
      l += __shfl_xor_sync(0xffffffffu, l, off);
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] += __shfl_xor_sync(0xffffffffu, o[e], off);
    }
    m = mt;
  }
  // merge the warps through shared memory (after the rings: [warp][D + 2] floats)
  if (lane < LPR) {
#pragma unroll
    for (int e = 0; e < 4; ++e) red[warp * (D + 2) + c + e] = o[e];
    if (lane == 0) {
      red[warp * (D + 2) + D] = m;
      red[warp * (D + 2) + D + 1] = l;
    }
  }
  __syncthreads();
  const bool write = abort_flag == nullptr || *reinterpret_cast<const volatile int*>(abort_flag) == 0;
  if (warp == 0 && write) {
    float mt = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mt = fmaxf(mt, red[w * (D + 2) + D]);
    const float mu = mt == -INFINITY ? 0.f : mt;
    float lt = 0.f, ot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float fct = ex2_approx(red[w * (D + 2) + D] - mu);
      lt = fmaf(red[w * (D + 2) + D + 1], fct, lt);
      if (lane < LPR) {
#pragma unroll
        for (int e = 0; e < 4; ++e) ot[e] = fmaf(red[w * (D + 2) + c + e], fct, ot[e]);
      }
    }
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    T* op = static_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh + i * p.o_ss + c;
    if (n_a == 0 && n_b == mb) {  // the whole pair: final output
      if (lane < LPR) {
#pragma unroll
        for (int e = 0; e < 4; ++e) op[e] = from_f<T>(ot[e] * inv);
      }
    } else {
      const long long first = paged_cta_of((long long)pair * mb, p.total, p.grid);
      const long long prow = (long long)pair * p.max_parts + (blockIdx.x - first);
      if (lane < LPR)
        *reinterpret_cast<float4*>(p.o_part + prow * p.D + c) =
            make_float4(ot[0] * inv, ot[1] * inv, ot[2] * inv, ot[3] * inv);
      if (lane == 0) p.lse_part[prow] = lt > 0.f ? mt + __log2f(lt) : -INFINITY;
      __threadfence();
      __syncwarp();
      if (lane == 0)
        s_last = atomicAdd(p.counters + pair, (unsigned)(n_b - n_a)) + (unsigned)(n_b - n_a) ==
                 (unsigned)mb;
      __syncwarp();
      if (s_last) {  // this segment completed the pair: every other partial is written
        __threadfence();
        const long long last = paged_cta_of((long long)pair * mb + mb - 1, p.total, p.grid);
        const int parts = (int)(last - first + 1);
        const long long r0 = (long long)pair * p.max_parts;
        float mx = -INFINITY;
        for (int j = lane; j < parts; j += 32) mx = fmaxf(mx, __ldcg(p.lse_part + r0 + j));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float mu2 = mx == -INFINITY ? 0.f : mx;
        float wsum = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int j = 0; j < parts; ++j) {
          const float w = ex2_approx(__ldcg(p.lse_part + r0 + j) - mu2);
          wsum += w;
          if (lane < LPR) {
            const float4 v4 = __ldcg(reinterpret_cast<const float4*>(p.o_part + (r0 + j) * p.D + c));
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
    }
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
  const int mb = p.max_blocks;
  unsigned char* ring = psm + warp * kPagedStages * STAGE;
  const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
  // this lane's piece of step u inside a stage: K at lane_off + u * STEP, V STAGE / 2 further
  const int lane_off = (g * D + c) * (int)sizeof(T);
  float* red = reinterpret_cast<float*>(psm + kPagedWarps * kPagedStages * STAGE);

  const long long f_end = ((long long)blockIdx.x + 1) * p.total / p.grid;
  for (long long f = (long long)blockIdx.x * p.total / p.grid; f < f_end;) {
    const int pair = (int)(f / mb);                  // row * H + h
    const int n_a = (int)(f - (long long)pair * mb);
    const long long rest = f_end - f;
    const int n_b = rest < (long long)(mb - n_a) ? n_a + (int)rest : mb;
    f += n_b - n_a;
    const int h = pair % p.H;
    const int row = pair / p.H;                      // b * Sq + i
    const int b = row / p.Sq, i = row - b * p.Sq;
    const int ctx = p.context_lens[b];
    int kv_end = ctx;                                // admissible positions are < kv_end
    if (p.causal && p.Sq > 1 && i + 1 < kv_end) kv_end = i + 1;
    const int q_pos = (p.Sq == 1) ? ctx : i;
    const int* bt = p.block_tables + (long long)b * p.bt_stride;
    const T* kp = static_cast<const T*>(p.k_pool) + (long long)(h / p.kv_group) * p.p_sh + c;
    const T* vp = static_cast<const T*>(p.v_pool) + (long long)(h / p.kv_group) * p.p_sh + c;

    float q[4], o[4] = {0.f, 0.f, 0.f, 0.f};
    {
      float qv[4];
      quad_to_f<T>(static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh + i * p.q_ss + c, qv);
#pragma unroll
      for (int e = 0; e < 4; ++e) q[e] = qv[e] * p.scale_log2;
    }
    const float slope2 = p.alibi ? __ldg(p.alibi + h) * 1.4426950408889634f : 0.f;
    float m = -INFINITY, l = 0.f;

    PagedCursor pc{n_a + warp - kPagedWarps, 0, 0, 0, 0, false, 0};
    paged_next_block(p, bt, n_b, kv_end, pc);
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
      if (cur.t0 >= cur.nt) paged_next_block(p, bt, n_b, kv_end, cur);
    };
#pragma unroll
    for (int st = 0; st < kPagedStages - 1; ++st) {
      issue(pc, st);
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

    paged_epilogue<T, LPR, kPagedWarps>(p, red, &s_last, warp, lane, m, l, o, pair, b, h, i, n_a,
                                        n_b, nullptr);
    __syncthreads();  // the rings and the reduction area are reused by the next segment
  }
}


// ------------------------------------------------------------------------------------------
// TMA variant (bf16/fp16, block_size a multiple of 16): the pools are 4-D tensor maps
// {D, kv_heads, block_size, num_blocks}; one chunk = 16 rows of one head of one block, K and V
// each one TMA box, completing on the stage's mbarrier.  Lane 0 of each warp issues its warp's
// loads; the copies bypass the SM's load path, so far more bytes stay in flight per SM than
// cp.async allows.  8 warps, NS stages per warp (24 KB of ring per warp), one CTA per SM.
// Every mbarrier wait is bounded: on a timeout the warp raises the CTA's abort flag, waits
// (bounded) for its copies in flight, and the CTA writes nothing more.
// ------------------------------------------------------------------------------------------
constexpr int kTmaWarps = 8;
constexpr int kTmaRows = 16;   // rows per chunk
constexpr int kSitePaged = 9;  // device-status site of the TMA kernel's waits

template <typename T, int D>
__host__ __device__ constexpr int paged_tma_stages() {
  return (24 * 1024) / (2 * kTmaRows * D * (int)sizeof(T));
}
template <typename T, int D>
__host__ __device__ constexpr int paged_tma_smem() {
  return kTmaWarps * paged_tma_stages<T, D>() * 2 * kTmaRows * D * (int)sizeof(T) +
         kTmaWarps * (D + 2) * 4 + kTmaWarps * paged_tma_stages<T, D>() * 8 + 16;
}

template <typename T, int LPR>
__global__ void __launch_bounds__(32 * kTmaWarps, 1)
    paged_attn_tma_kernel(const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const PagedParams p) {
  constexpr int KPW = 32 / LPR;          // keys per step
  constexpr int D = LPR * 4;
  constexpr int NS = paged_tma_stages<T, D>();
  constexpr int STEPS = kTmaRows / KPW;
  constexpr int HALF = kTmaRows * D * (int)sizeof(T);  // K (or V) bytes of a chunk
  constexpr int STAGE = 2 * HALF;
  constexpr int STEP = KPW * D * (int)sizeof(T);
  static_assert(NS >= 2, "at least two stages");
  extern __shared__ __align__(128) unsigned char psm[];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane / LPR;
  const int c = (lane % LPR) * 4;
  const int mb = p.max_blocks;
  unsigned char* ring = psm + warp * NS * STAGE;
  float* red = reinterpret_cast<float*>(psm + kTmaWarps * NS * STAGE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(psm + kTmaWarps * NS * STAGE + kTmaWarps * (D + 2) * 4);
  int* abort_flag = reinterpret_cast<int*>(bars + kTmaWarps * NS);
  const uint32_t ring_s = smem_u32(ring);
  const uint32_t bar_s = smem_u32(bars + warp * NS);
  const int lane_off = (g * D + c) * (int)sizeof(T);
  if (lane == 0) {
    for (int k = 0; k < NS; ++k) mbar_init(bar_s + 8 * k, 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 0) *abort_flag = 0;
  if (threadIdx.x == 32) {
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  __syncthreads();
  const WaitCtx wctx{abort_flag, p.status, p.timeout_ns};
  uint32_t phase = 0;  // parity of the next completion of each of this warp's stages

  const long long f_end = ((long long)blockIdx.x + 1) * p.total / p.grid;
  for (long long f = (long long)blockIdx.x * p.total / p.grid; f < f_end;) {
    const int pair = (int)(f / mb);
    const int n_a = (int)(f - (long long)pair * mb);
    const long long rest = f_end - f;
    const int n_b = rest < (long long)(mb - n_a) ? n_a + (int)rest : mb;
    f += n_b - n_a;
    const int h = pair % p.H;
    const int row = pair / p.H;
    const int b = row / p.Sq, i = row - b * p.Sq;
    const int hk = h / p.kv_group;
    const int ctx = p.context_lens[b];
    int kv_end = ctx;
    if (p.causal && p.Sq > 1 && i + 1 < kv_end) kv_end = i + 1;
    const int q_pos = (p.Sq == 1) ? ctx : i;
    const int* bt = p.block_tables + (long long)b * p.bt_stride;

    float q[4], o[4] = {0.f, 0.f, 0.f, 0.f};
    {
      float qv[4];
      quad_to_f<T>(static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh + i * p.q_ss + c, qv);
#pragma unroll
      for (int e = 0; e < 4; ++e) q[e] = qv[e] * p.scale_log2;
    }
    const float slope2 = p.alibi ? __ldg(p.alibi + h) * 1.4426950408889634f : 0.f;
    float m = -INFINITY, l = 0.f;

    PagedCursor pc{n_a + warp - kTmaWarps, 0, 0, 0, 0, false, 0};
    paged_next_block_w<kTmaWarps>(p, bt, n_b, kv_end, pc);
    PagedCursor cc = pc;
    auto issue = [&](const PagedCursor& cur, int stage) {
      __syncwarp();  // every lane is done reading the stage being refilled
      if (lane == 0 && cur.valid) {
        fence_proxy_async_smem();
        const uint32_t bar = bar_s + 8 * stage;
        const uint32_t dst = ring_s + stage * STAGE;
        mbar_arrive_expect_tx(bar, STAGE);
        tma_load_4d(dst, &tm_k, bar, 0, hk, cur.t0, cur.blk);
        tma_load_4d(dst + HALF, &tm_v, bar, 0, hk, cur.t0, cur.blk);
      }
    };
    auto advance = [&](PagedCursor& cur) {
      if (!cur.valid) return;
      cur.t0 += kTmaRows;
      if (cur.t0 >= cur.nt) paged_next_block_w<kTmaWarps>(p, bt, n_b, kv_end, cur);
    };
    int inflight = 0;
#pragma unroll 1
    for (int st = 0; st < NS - 1; ++st) {
      if (pc.valid) ++inflight;
      issue(pc, st);
      advance(pc);
    }
    int stage = 0;
    bool ok = true;
    while (cc.valid) {
      if (pc.valid) ++inflight;
      issue(pc, (stage + NS - 1) % NS);
      advance(pc);
      ok = mbar_wait(bar_s + 8 * stage, (phase >> stage) & 1u, wctx, kSitePaged);
      if (!ok) break;
      phase ^= 1u << stage;
      --inflight;
      const unsigned char* st = ring + stage * STAGE + lane_off;
      float sc[STEPS];
#pragma unroll
      for (int u = 0; u < STEPS; ++u) {
        float kx[4];
        quad_to_f<T>(reinterpret_cast<const T*>(st + u * STEP), kx);
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) a = fmaf(q[e], kx[e], a);
        sc[u] = a;
      }
      // Reduce-scatter over the LPR lanes of a key group: each halving step keeps half of the
      // values (the upper half in lanes with that offset bit set) and adds the partner's copy,
      // so STEPS/2 + STEPS/4 + ... + 1 shuffles replace STEPS * log2(LPR).  Afterwards lane
      // holds the full score of step u = (lane >> 1) % STEPS (lanes 2u and 2u + 1 alike).
#pragma unroll
      for (int n = STEPS, off = LPR / 2; n > 1; n >>= 1, off >>= 1) {
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int j = 0; j < n / 2; ++j) {
          const float send = up ? sc[j] : sc[j + n / 2];
          const float keep = up ? sc[j + n / 2] : sc[j];
          sc[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      float sv = sc[0] + __shfl_xor_sync(0xffffffffu, sc[0], 1);
      {
        const int t = cc.t0 + ((lane >> 1) & (STEPS - 1)) * KPW + g;
        sv = (t < cc.nt) ? fmaf(slope2, (float)(cc.pos0 + t - q_pos), sv) : -INFINITY;
      }
      float m_blk = sv;  // over the warp: every key of the chunk
#pragma unroll
      for (int off = 16; off > 1; off >>= 1) m_blk = fmaxf(m_blk, __shfl_xor_sync(0xffffffffu, m_blk, off));
      const float m_new = fmaxf(m, m_blk);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = ex2_approx(m - m_use);
      l *= alpha;
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] *= alpha;
      const float pv = ex2_approx(sv - m_use);  // 0 for masked keys (their rows are finite)
#pragma unroll
      for (int u = 0; u < STEPS; ++u) {
        const float pw = __shfl_sync(0xffffffffu, pv, g * LPR + 2 * u);  // key u * KPW + g
        float vx[4];
        quad_to_f<T>(reinterpret_cast<const T*>(st + HALF + u * STEP), vx);
        l += pw;
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = fmaf(pw, vx[e], o[e]);
      }
      m = m_new;
      advance(cc);
      stage = (stage + 1) % NS;
    }
    if (!ok) {  // wait for this warp's copies still in flight (bounded), then stop writing
      for (int k = 0; k < inflight; ++k) {
        const int sk = (stage + k) % NS;
        if (lane == 0) mbar_wait_drain(bar_s + 8 * sk, (phase >> sk) & 1u, p.status, p.timeout_ns);
        phase ^= 1u << sk;
      }
      __syncwarp();
    }
    paged_epilogue<T, LPR, kTmaWarps>(p, red, &s_last, warp, lane, m, l, o, pair, b, h, i, n_a,
                                      n_b, abort_flag);
    __syncthreads();
    if (*reinterpret_cast<volatile int*>(abort_flag)) break;
  }
}

}  // namespace mlxp
