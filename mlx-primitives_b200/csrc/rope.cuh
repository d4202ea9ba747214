// rope.cuh — rotary position embedding for Q and K ahead of the attention kernel.
//
// The half-split rotation of the reference's rope (mlx_primitives/kernels/rope.py:451-496):
// with h = D / 2, x1 = x[:h], x2 = x[h:] and (cos, sin) of the row's position p,
//   y[:h] = x1 * cos[p] - x2 * sin[p],   y[h:] = x1 * sin[p] + x2 * cos[p],
// p = pos_offset + s for sequence index s; cos/sin are fp32 [n_pos][h].  Computed in fp32 and
// rounded once to the element type.  Memory-bound: every thread moves 16 bytes of each half
// of a row (8 bf16/fp16 or 4 fp32 pairs), the cos/sin rows come from L1/L2; both tensors of a
// Q/K pair are rotated by one launch.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace mlxp {

struct RopeTensor {
  const void* x;
  void* y;
  long long xs[3], ys[3];  // element strides of (batch, head, seq)
  int H, S;
  long long rows;          // B * H * S
  long long pos_offset;
};

struct RopeParams {
  RopeTensor t[2];
  int n;                   // 1 or 2 tensors
  int half;                // D / 2
  const float* cosc;
  const float* sinc;
  long long n_pos;
};

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// One rotated pair (x1, x2) -> (x1 cos - x2 sin, x1 sin + x2 cos), each product and sum rounded
// separately (no contraction into FMAs), so that every kernel that rotates (this one and the
// attention kernel's rotation items) produces the same bits.
__device__ __forceinline__ void rope_pair(float a, float b, float c, float sn, float& y1,
                                          float& y2) {
  y1 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
  y2 = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
}

// VEC pairs per thread: 16 / sizeof(T) (one 16-byte access per half) when half is a multiple
// of it and every row starts on 16 bytes, else 1.  A block handles one token (batch, position)
// at a time: its threads cover the token's heads x (half / VEC) pair groups, so the index
// arithmetic is per token and a token's rows (contiguous in BSHD) are read together.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) rope_kernel(const RopeParams p) {
  const int groups = p.half / VEC;
  const long long ntok0 = p.t[0].rows / (p.t[0].H > 0 ? p.t[0].H : 1);
  const long long ntok = ntok0 + (p.n > 1 ? p.t[1].rows / (p.t[1].H > 0 ? p.t[1].H : 1) : 0);
  for (long long tk = blockIdx.x; tk < ntok; tk += gridDim.x) {
    const int which = tk >= ntok0;
    const RopeTensor& tt = p.t[which];
    const long long tok = which ? tk - ntok0 : tk;
    const long long b = tok / tt.S, s = tok - b * tt.S;
    const long long pos = tt.pos_offset + s;
    const float* crow = p.cosc + pos * p.half;
    const float* srow = p.sinc + pos * p.half;
    const T* xt = static_cast<const T*>(tt.x) + b * tt.xs[0] + s * tt.xs[2];
    T* yt = static_cast<T*>(tt.y) + b * tt.ys[0] + s * tt.ys[2];
    const int per_tok = tt.H * groups;
    for (int i = threadIdx.x; i < per_tok; i += blockDim.x) {
      const int h = i / groups, g = i - h * groups;
      const T* x = xt + h * tt.xs[1];
      T* y = yt + h * tt.ys[1];
      T x1[VEC], x2[VEC], y1[VEC], y2[VEC];
      if constexpr (VEC * sizeof(T) == 16) {
        *reinterpret_cast<uint4*>(x1) = *reinterpret_cast<const uint4*>(x + g * VEC);
        *reinterpret_cast<uint4*>(x2) = *reinterpret_cast<const uint4*>(x + p.half + g * VEC);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          x1[e] = x[g * VEC + e];
          x2[e] = x[p.half + g * VEC + e];
        }
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float a = to_f<T>(x1[e]), bb = to_f<T>(x2[e]);
        const float c = __ldg(crow + g * VEC + e), sn = __ldg(srow + g * VEC + e);
        float r1, r2;
        rope_pair(a, bb, c, sn, r1, r2);
        y1[e] = from_f<T>(r1);
        y2[e] = from_f<T>(r2);
      }
      if constexpr (VEC * sizeof(T) == 16) {
        *reinterpret_cast<uint4*>(y + g * VEC) = *reinterpret_cast<const uint4*>(y1);
        *reinterpret_cast<uint4*>(y + p.half + g * VEC) = *reinterpret_cast<const uint4*>(y2);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          y[g * VEC + e] = y1[e];
          y[p.half + g * VEC + e] = y2[e];
        }
      }
    }
  }
}

}  // namespace mlxp
