// ring_nccl.cuh — sequence-parallel causal attention over NCCL: the C-ABI ring (mlxp_ring_*).
//
// Included at the end of mlxp_attn.cu: it drives the library's own entry points
// (mlxp_attn_fwd_accumulate, mlxp_cast_output) from C++, for callers
// that are not Python.  The schedule is the zig-zag ring of mlx_primitives/attention/ring.py:
// the sequence of S = P * S_local tokens is cut into 2P chunks of C = S_local / 2; rank r holds
// chunks r and 2P-1-r back to back; in P steps every rank attends its two query chunks to the
// K/V shard it holds while the shard moves one rank on (NCCL send to r+1, receive from r-1 on
// a separate stream, so the transfer overlaps the kernels), and folds each (query chunk, key
// chunk) result into an fp32 accumulator, inside the attention kernel, with the LSE form of
// online_softmax_merge
// (mlx_primitives/attention/_online_softmax.py:42-106).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2): a process that already holds an NCCL
// (for instance through torch) shares it, and the library itself has no link-time dependency.
#pragma once

#include <dlfcn.h>
#include <nccl.h>

namespace mlxp {
namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  const char* (*GetErrorString)(ncclResult_t);
};

int nccl_api(const NcclApi** out) {
  static std::mutex mu;
  static NcclApi api;
  static int state = 0;  // 0 not tried, 1 loaded, -1 failed
  static std::string why;
  std::lock_guard<std::mutex> lock(mu);
  if (state == 0) {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      why = e ? e : "libnccl.so.2 not found";
      state = -1;
    } else {
      bool ok = true;
      auto sym = [&](const char* name) {
        void* p = dlsym(h, name);
        if (!p) {
          ok = false;
          why = std::string("missing symbol ") + name;
        }
        return p;
      };
      api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
      api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
      api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
      api.Send = reinterpret_cast<decltype(api.Send)>(sym("ncclSend"));
      api.Recv = reinterpret_cast<decltype(api.Recv)>(sym("ncclRecv"));
      api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(sym("ncclGroupStart"));
      api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(sym("ncclGroupEnd"));
      api.GetErrorString =
          reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
      state = ok ? 1 : -1;
    }
  }
  if (state < 0) return fail(MLXP_ERR_NCCL, "NCCL could not be loaded: %s", why.c_str());
  *out = &api;
  return MLXP_OK;
}

int nccl_fail(const NcclApi* api, ncclResult_t r, const char* what) {
  return fail(MLXP_ERR_NCCL, "%s: %s", what, api->GetErrorString(r));
}

struct RingComm {
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0, device = -1;
  cudaStream_t comm_stream = nullptr;  // NCCL sends / receives
  cudaEvent_t ready = nullptr;         // compute stream -> comm stream
  cudaEvent_t arrived = nullptr;       // comm stream -> compute stream
};

// Copies rows of a strided [B][H][S][D] tensor into a contiguous one, 16 bytes per thread-step.
// Row starts are 16-byte aligned (checked by the caller).
__global__ void __launch_bounds__(256) gather_rows_kernel(const char* __restrict__ src,
                                                          char* __restrict__ dst, long long rows,
                                                          int H, int S, int row_bytes,
                                                          long long sb, long long sh,
                                                          long long ss) {
  const int vec = row_bytes / 16;
  const long long total = rows * vec;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / vec;
    const int c = (int)(i - row * vec);
    const long long s = row % S, bh = row / S;
    const long long h = bh % H, b = bh / H;
    const uint4 x = *reinterpret_cast<const uint4*>(src + b * sb + h * sh + s * ss + 16LL * c);
    *reinterpret_cast<uint4*>(dst + row * row_bytes + 16LL * c) = x;
  }
}

// Workspace of one ring call: two K/V shard buffers (the one being computed on and the one
// being received) and the fp32 accumulators of both query chunks.
struct RingWs {
  size_t kv_bytes = 0;                  // one of K or V, contiguous [B][H][S_local][D]
  size_t off_k[2] = {0, 0}, off_v[2] = {0, 0};
  size_t off_oacc = 0, off_lacc = 0;
  size_t total = 0;
};

RingWs ring_ws_layout(int64_t B, int64_t H, int64_t S_local, int64_t D, int es) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  RingWs w;
  w.kv_bytes = (size_t)B * H * S_local * D * es;
  size_t off = 0;
  for (int i = 0; i < 2; ++i) {
    w.off_k[i] = off;
    off += up(w.kv_bytes);
    w.off_v[i] = off;
    off += up(w.kv_bytes);
  }
  w.off_oacc = off;
  off += up((size_t)B * H * S_local * D * 4);
  w.off_lacc = off;
  off += up((size_t)B * H * S_local * 4);
  w.total = off;
  return w;
}

int ring_check_shape(int dtype, int64_t B, int64_t H, int64_t S_local, int64_t D) {
  if (dtype != MLXP_DTYPE_BF16 && dtype != MLXP_DTYPE_FP16)
    return fail(MLXP_ERR_UNSUPPORTED, "the ring takes bf16/fp16 inputs");
  if (D != 64 && D != 128)
    return fail(MLXP_ERR_UNSUPPORTED, "the ring supports head_dim 64 and 128, got %lld",
                (long long)D);
  if (B < 1 || H < 1 || S_local < 2 || (S_local % 2))
    return fail(MLXP_ERR_INVALID,
                "a zig-zag shard holds two equal chunks: need B, H >= 1 and an even S_local >= 2");
  return MLXP_OK;
}

int ring_fwd(RingComm* rc, const void* q, const void* k, const void* v, void* o, int dtype,
             int64_t B, int64_t H, int64_t S_local, int64_t D, const int64_t qs[4],
             const int64_t ks[4], const int64_t vs[4], const int64_t os[4], float scale,
             void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (!rc || !rc->comm) return fail(MLXP_ERR_INVALID, "ring communicator is null");
  if (int r = ring_check_shape(dtype, B, H, S_local, D)) return r;
  if (!q || !k || !v || !o || !qs || !ks || !vs || !os)
    return fail(MLXP_ERR_INVALID, "q, k, v, o and their strides must be non-null");
  if (!(scale > 0.f) || !std::isfinite(scale))
    return fail(MLXP_ERR_INVALID, "scale must be positive and finite");
  // rows of every 16-bit tensor must start on 16 bytes (K/V are gathered 16 bytes at a time;
  // Q and O go through tensor maps / the cast kernel)
  if (int e = check_out_strides(q, qs, 8, "q")) return e;
  if (int e = check_out_strides(k, ks, 8, "k")) return e;
  if (int e = check_out_strides(v, vs, 8, "v")) return e;
  if (int e = check_out_strides(o, os, 8, "o")) return e;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != rc->device)
    return fail(MLXP_ERR_INVALID, "the ring must be called on the device it was created on (%d)",
                rc->device);
  const NcclApi* api = nullptr;
  if (int r = nccl_api(&api)) return r;
  const int es = 2;
  const RingWs L = ring_ws_layout(B, H, S_local, D, es);
  if (!ws || ws_bytes < L.total)
    return fail(MLXP_ERR_WORKSPACE, "ring workspace of %zu bytes needed, got %zu", L.total,
                ws_bytes);
  if (reinterpret_cast<uintptr_t>(ws) % 256)
    return fail(MLXP_ERR_INVALID, "ring workspace must be 256-byte aligned");
  char* base = static_cast<char*>(ws);
  char* kb[2] = {base + L.off_k[0], base + L.off_k[1]};
  char* vb[2] = {base + L.off_v[0], base + L.off_v[1]};
  float* o_acc = reinterpret_cast<float*>(base + L.off_oacc);
  float* l_acc = reinterpret_cast<float*>(base + L.off_lacc);
  const int64_t C = S_local / 2;
  const int P = rc->nranks, r = rc->rank;
  const int nxt = (r + 1) % P, prv = (r + P - 1) % P;
  const int64_t kv_st[4] = {H * S_local * D, S_local * D, D, 1};  // shard buffers
  const int64_t part_st[4] = {H * C * D, C * D, D, 1};
  const long long rows = B * H * S_local;

  // local K/V -> shard buffer 0; accumulators <- (O = 0, LSE = -inf)
  {
    const unsigned grid = (unsigned)std::min<long long>((rows * D * es / 16 + 255) / 256, 4096);
    gather_rows_kernel<<<grid, 256, 0, stream>>>(static_cast<const char*>(k), kb[0], rows,
                                                 (int)H, (int)S_local, (int)(D * es), ks[0] * es,
                                                 ks[1] * es, ks[2] * es);
    gather_rows_kernel<<<grid, 256, 0, stream>>>(static_cast<const char*>(v), vb[0], rows,
                                                 (int)H, (int)S_local, (int)(D * es), vs[0] * es,
                                                 vs[1] * es, vs[2] * es);
    // both chunks' accumulators: [2][B][H][C][D] and [2][B][H][C], i.e. batch 2B
    Problem pe{MLXP_DTYPE_FP32, 2 * B, H, C, 0, D, 0, -1, -1, 0, 0};
    if (int e = fill_empty(pe, o_acc, l_acc, part_st, stream)) return e;
    cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) return cuda_fail(ce, "ring set-up launch");
  }
  for (int step = 0; step < P; ++step) {
    const int cur = step & 1, src = (r - step + P) % P;
    const bool pass = step + 1 < P;
    if (pass) {
      // The receive buffer was last read by the previous step's kernels and send.
      if (cudaEventRecord(rc->ready, stream) != cudaSuccess ||
          cudaStreamWaitEvent(rc->comm_stream, rc->ready, 0) != cudaSuccess)
        return cuda_fail(cudaGetLastError(), "ring stream ordering");
      ncclResult_t nr = api->GroupStart();
      if (nr == ncclSuccess) nr = api->Send(kb[cur], L.kv_bytes, ncclUint8, nxt, rc->comm, rc->comm_stream);
      if (nr == ncclSuccess) nr = api->Send(vb[cur], L.kv_bytes, ncclUint8, nxt, rc->comm, rc->comm_stream);
      if (nr == ncclSuccess) nr = api->Recv(kb[cur ^ 1], L.kv_bytes, ncclUint8, prv, rc->comm, rc->comm_stream);
      if (nr == ncclSuccess) nr = api->Recv(vb[cur ^ 1], L.kv_bytes, ncclUint8, prv, rc->comm, rc->comm_stream);
      const ncclResult_t ge = api->GroupEnd();
      if (nr != ncclSuccess) return nccl_fail(api, nr, "ring send/recv");
      if (ge != ncclSuccess) return nccl_fail(api, ge, "ring send/recv");
      if (cudaEventRecord(rc->arrived, rc->comm_stream) != cudaSuccess)
        return cuda_fail(cudaGetLastError(), "ring stream ordering");
    }
    const int qchunk[2] = {r, 2 * P - 1 - r}, kchunk[2] = {src, 2 * P - 1 - src};
    for (int qi = 0; qi < 2; ++qi) {
      const char* qv = static_cast<const char*>(q) + qi * C * qs[2] * es;
      for (int ki = 0; ki < 2; ++ki) {
        if (kchunk[ki] > qchunk[qi]) continue;  // every key after every query of the chunk
        const char* kv_ = kb[cur] + ki * C * D * es;
        const char* vv = vb[cur] + ki * C * D * es;
        if (int e = mlxp_attn_fwd_accumulate(qv, kv_, vv, o_acc + qi * B * H * C * D,
                                             l_acc + qi * B * H * C, dtype, B, H, C, C, D, qs,
                                             kv_st, kv_st, part_st, scale, 1, -1, -1,
                                             (int64_t)qchunk[qi] * C, (int64_t)kchunk[ki] * C,
                                             stream))
          return e;
      }
    }
    if (pass && cudaStreamWaitEvent(stream, rc->arrived, 0) != cudaSuccess)
      return cuda_fail(cudaGetLastError(), "ring stream ordering");
  }
  for (int qi = 0; qi < 2; ++qi)
    if (int e = mlxp_cast_output(o_acc + qi * B * H * C * D,
                                 static_cast<char*>(o) + qi * C * os[2] * es, dtype, B, H, C, D,
                                 os, stream))
      return e;
  return MLXP_OK;
}

}  // namespace
}  // namespace mlxp

extern "C" {

int mlxp_ring_unique_id(void* id_out) {
  if (!id_out) return mlxp::fail(MLXP_ERR_INVALID, "id_out is null");
  const mlxp::NcclApi* api = nullptr;
  if (int r = mlxp::nccl_api(&api)) return r;
  ncclUniqueId id;
  const ncclResult_t nr = api->GetUniqueId(&id);
  if (nr != ncclSuccess) return mlxp::nccl_fail(api, nr, "ncclGetUniqueId");
  static_assert(sizeof(id) == 128, "NCCL unique id is 128 bytes");
  std::memcpy(id_out, &id, sizeof(id));
  return MLXP_OK;
}

int mlxp_ring_init(const void* nccl_unique_id, int nranks, int rank, void** comm) {
  if (!nccl_unique_id || !comm || nranks < 1 || rank < 0 || rank >= nranks)
    return mlxp::fail(MLXP_ERR_INVALID, "invalid ring_init arguments (nranks %d, rank %d)",
                      nranks, rank);
  *comm = nullptr;
  const mlxp::NcclApi* api = nullptr;
  if (int r = mlxp::nccl_api(&api)) return r;
  auto* rc = new mlxp::RingComm();
  rc->nranks = nranks;
  rc->rank = rank;
  if (cudaGetDevice(&rc->device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&rc->comm_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&rc->ready, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&rc->arrived, cudaEventDisableTiming) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    mlxp_ring_destroy(rc);
    return mlxp::cuda_fail(e, "ring_init stream/event creation");
  }
  ncclUniqueId id;
  std::memcpy(&id, nccl_unique_id, sizeof(id));
  const ncclResult_t nr = api->CommInitRank(&rc->comm, nranks, id, rank);
  if (nr != ncclSuccess) {
    rc->comm = nullptr;
    mlxp_ring_destroy(rc);
    return mlxp::nccl_fail(api, nr, "ncclCommInitRank");
  }
  *comm = rc;
  return MLXP_OK;
}

size_t mlxp_ring_workspace_size(int dtype, int64_t B, int64_t H, int64_t S_local, int64_t D) {
  if (mlxp::ring_check_shape(dtype, B, H, S_local, D) != MLXP_OK) return 0;
  return mlxp::ring_ws_layout(B, H, S_local, D, 2).total;
}

int mlxp_ring_attn_fwd(void* comm, const void* q, const void* k, const void* v, void* o,
                       int dtype, int64_t B, int64_t H, int64_t S_local, int64_t D,
                       const int64_t q_strides[4], const int64_t k_strides[4],
                       const int64_t v_strides[4], const int64_t o_strides[4], float scale,
                       void* workspace, size_t ws_bytes, void* cuda_stream) {
  return mlxp::ring_fwd(static_cast<mlxp::RingComm*>(comm), q, k, v, o, dtype, B, H, S_local, D,
                        q_strides, k_strides, v_strides, o_strides, scale, workspace, ws_bytes,
                        static_cast<cudaStream_t>(cuda_stream));
}

int mlxp_ring_destroy(void* comm) {
  auto* rc = static_cast<mlxp::RingComm*>(comm);
  if (!rc) return MLXP_OK;
  int status = MLXP_OK;
  if (rc->comm) {
    const mlxp::NcclApi* api = nullptr;
    if (mlxp::nccl_api(&api) == MLXP_OK) {
      const ncclResult_t nr = api->CommDestroy(rc->comm);
      if (nr != ncclSuccess) status = mlxp::nccl_fail(api, nr, "ncclCommDestroy");
    }
  }
  if (rc->ready) cudaEventDestroy(rc->ready);
  if (rc->arrived) cudaEventDestroy(rc->arrived);
  if (rc->comm_stream) cudaStreamDestroy(rc->comm_stream);
  delete rc;
  return status;
}

}  // extern "C"
