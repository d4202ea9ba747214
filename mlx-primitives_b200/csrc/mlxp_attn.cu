// mlxp_attn.cu — host side of libmlxp_attn.so: argument validation, TMA tensor maps, the
// key-split heuristic, kernel launches and the extern "C" entry points of include/mlxp_attn.h.
//
// The library never allocates device memory: splits write to a caller-provided workspace.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <queue>
#include <string>
#include <vector>

#include "../../include/mlxp_attn.h"
#include "attn_common.cuh"
#include "attn_fwd_fp32.cuh"
#include "attn_fwd_sm100.cuh"
#include "rope.cuh"
#include "paged_attn.cuh"
#include "attn_bwd.cuh"
#include "attn_bwd_sm100.cuh"

namespace mlxp {

__device__ int g_dev_status = 0;
// Work counters of the persistent tensor-core kernel: kCounterSlots pairs per device, handed
// out round-robin to launches so that launches in flight on different streams at the same time
// do not share one (each pair is reset by the last CTA of the launch that used it).
constexpr int kCounterSlots = 256;
__device__ unsigned g_work_counters[2 * kCounterSlots];

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MLXP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

std::atomic<unsigned long long> g_timeout_ns{2000000000ull};
// Test hook (mlxp_set_backward_path): 1 = always the CUDA-core backward.
std::atomic<int> g_bwd_force_cuda_cores{0};

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
int* g_status_ptr[kMaxDevices] = {};
unsigned* g_counter_ptr[kMaxDevices] = {};
std::atomic<unsigned> g_counter_seq[kMaxDevices];
int g_num_sms[kMaxDevices] = {};
unsigned long long g_attr_done[kMaxDevices] = {};

int current_device(int& dev) {
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MLXP_ERR_CUDA, "device ordinal %d out of range", dev);
  return MLXP_OK;
}

// Device status word and SM count of the current device (looked up once per device).
int device_info(int** status, int* sms) {
  int dev;
  if (int rc = current_device(dev)) return rc;
  std::lock_guard<std::mutex> g(g_dev_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_dev_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    void* cptr = nullptr;
    e = cudaGetSymbolAddress(&cptr, g_work_counters);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(work counters)");
    g_status_ptr[dev] = static_cast<int*>(ptr);
    g_counter_ptr[dev] = static_cast<unsigned*>(cptr);
    g_num_sms[dev] = n;
  }
  if (status) *status = g_status_ptr[dev];
  if (sms) *sms = g_num_sms[dev];
  return MLXP_OK;
}

// Sets the dynamic shared memory limit of a kernel once per device.
template <typename K>
int ensure_smem_attr(K kernel, int bytes, unsigned long long bit) {
  int dev;
  if (int rc = current_device(dev)) return rc;
  {
    std::lock_guard<std::mutex> g(g_dev_mu);
    if (g_attr_done[dev] & bit) return MLXP_OK;
  }
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  std::lock_guard<std::mutex> g(g_dev_mu);
  g_attr_done[dev] |= bit;
  return MLXP_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
int g_encode_rc = MLXP_OK;
std::string g_encode_err;

int get_encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
      g_encode_rc = MLXP_ERR_CUDA;
      g_encode_err = "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled) failed";
      return;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode_rc != MLXP_OK) return fail(g_encode_rc, "%s", g_encode_err.c_str());
  return MLXP_OK;
}

// Builds a 4-D tensor map over a (b, h, s, d)-strided tensor with a box of 64 d-elements by
// `box_rows` s-rows.  The three outer dims are ordered by stride so that the map is monotonic
// whatever the layout (BHSD: s,h,b; BSHD: h,s,b); size-1 and stride-0 (broadcast) dims are
// given coordinate 0.  The box lands in shared memory as box_rows rows of 128 bytes, 128-byte
// swizzled, for every layout.
int make_tmap(const void* ptr, CUtensorMapDataType dt, int es, int64_t B, int64_t H, int64_t S,
              int64_t D, const int64_t st[4], int box_rows, int box_cols, const char* name,
              CUtensorMap* map, TmaCoordMap* cm) {
  if (int rc = get_encode_fn()) return rc;
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return fail(MLXP_ERR_INVALID, "%s: base address must be 16-byte aligned", name);
  if (st[3] != 1) return fail(MLXP_ERR_INVALID, "%s: head_dim stride must be 1", name);
  struct Dim {
    int64_t size, stride;
    int which;  // 0 = s, 1 = h, 2 = b
    bool unit;
  } dims[3] = {{S, st[2], 0, false}, {H, st[1], 1, false}, {B, st[0], 2, false}};
  bool bcast[3] = {false, false, false};
  for (auto& d : dims) {
    if (d.which != 0 && (d.size == 1 || d.stride == 0)) {
      bcast[d.which] = true;
      d.size = 1;
      d.unit = true;
    } else if (d.which == 0 && d.size == 1) {
      d.unit = true;
    } else {
      if (d.stride <= 0)
        return fail(MLXP_ERR_INVALID, "%s: stride of dim %d must be positive", name, d.which);
      if ((d.stride * es) % 16)
        return fail(MLXP_ERR_INVALID, "%s: strides must be multiples of 16 bytes", name);
    }
  }
  std::stable_sort(dims, dims + 3, [](const Dim& a, const Dim& b) {
    if (a.unit != b.unit) return !a.unit;  // size-1 dims last
    return a.stride < b.stride;
  });
  // benign stride for unit dims: past the span of everything before them
  int64_t span = D * es;
  for (auto& d : dims) {
    if (d.unit) {
      d.stride = ((span + 15) / 16) * 16 / es;
    }
    span = std::max<int64_t>(span, d.stride * es * d.size);
  }
  cuuint64_t gdim[4] = {(cuuint64_t)D, (cuuint64_t)dims[0].size, (cuuint64_t)dims[1].size,
                        (cuuint64_t)dims[2].size};
  cuuint64_t gstride[3] = {(cuuint64_t)(dims[0].stride * es), (cuuint64_t)(dims[1].stride * es),
                           (cuuint64_t)(dims[2].stride * es)};
  cuuint32_t box[4] = {(cuuint32_t)box_cols, 1, 1, 1};
  for (int i = 0; i < 3; ++i)
    if (dims[i].which == 0) box[1 + i] = box_rows;
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(map, dt, 4, const_cast<void*>(ptr), gdim, gstride, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MLXP_ERR_INVALID, "%s: cuTensorMapEncodeTiled failed (code %d)", name, (int)r);
  for (int i = 0; i < 3; ++i) {
    if (dims[i].which == 0) cm->slot_s = (int8_t)(1 + i);
    if (dims[i].which == 1) cm->slot_h = (int8_t)(1 + i);
    if (dims[i].which == 2) cm->slot_b = (int8_t)(1 + i);
  }
  cm->bcast_h = bcast[1];
  cm->bcast_b = bcast[2];
  return MLXP_OK;
}

struct Problem {
  int dtype;
  int64_t B, H, Sq, Skv, D;
  int causal;
  int64_t wl, wr, qoff, kvoff;
  int64_t Hkv = 0;  // K/V heads (grouped / multi-query attention); 0 = H
  int64_t kv_heads() const { return Hkv ? Hkv : H; }
};

MaskSpec mask_of(const Problem& pr) {
  return MaskSpec{pr.causal, (long long)pr.wl, (long long)pr.wr, (long long)pr.qoff,
                  (long long)pr.kvoff, (long long)pr.Skv};
}

int validate(const Problem& pr) {
  if (pr.B <= 0 || pr.H <= 0 || pr.Sq < 0 || pr.Skv < 0 || pr.D <= 0)
    return fail(MLXP_ERR_INVALID, "invalid shape B=%lld H=%lld Sq=%lld Skv=%lld D=%lld",
                (long long)pr.B, (long long)pr.H, (long long)pr.Sq, (long long)pr.Skv,
                (long long)pr.D);
  if (pr.Sq > (1ll << 30) || pr.Skv > (1ll << 30) || pr.B * pr.H > (1ll << 24))
    return fail(MLXP_ERR_INVALID, "shape too large");
  if (pr.wl < -1 || pr.wr < -1) return fail(MLXP_ERR_INVALID, "window must be >= 0 or -1");
  if (pr.kv_heads() < 1 || pr.H % pr.kv_heads())
    return fail(MLXP_ERR_INVALID, "num_heads (%lld) must be divisible by num_kv_heads (%lld)",
                (long long)pr.H, (long long)pr.kv_heads());
  if (pr.dtype == MLXP_DTYPE_BF16 || pr.dtype == MLXP_DTYPE_FP16) {
    if (pr.D != 64 && pr.D != 128)
      return fail(MLXP_ERR_UNSUPPORTED, "bf16/fp16 attention supports head_dim 64 and 128, got %lld",
                  (long long)pr.D);
  } else if (pr.dtype == MLXP_DTYPE_FP32) {
    if (pr.D != 32 && pr.D != 64 && pr.D != 128)
      return fail(MLXP_ERR_UNSUPPORTED, "fp32 attention supports head_dim 32, 64 and 128, got %lld",
                  (long long)pr.D);
  } else {
    return fail(MLXP_ERR_INVALID, "unknown dtype %d", pr.dtype);
  }
  return MLXP_OK;
}

constexpr int kBM2 = 256;  // query rows per tensor-core CTA
constexpr int kBN = 128;   // keys per tensor-core tile

// Scheduling groups of the persistent kernel (FwdParams::n_groups): groups of at least about
// two waves of items — enough to balance, small enough that a group's K/V (2 * Skv * D * 2
// bytes per unit) stays in L2 — spread evenly: floor(units / target) groups of equal size (+-1),
// so that no group is much smaller than the target.
int sched_groups(long long units, long long per_unit, int sms) {
  const long long target = std::max<long long>(1, (2LL * sms + per_unit - 1) / per_unit);
  return (int)std::max<long long>(1, units / target);
}

// Key-range split count, uniform rule for long unmasked key ranges: enough items to fill every
// SM several times, and items short enough (<= 128 key tiles) that the end-of-launch tail stays
// small; each split costs one fp32 partial write and read, so no more splits than that.  (A
// 64-tile cap measured 5-19 % slower: config 4 645 against 678 TFLOPS with 8 instead of 4
// splits, 16K x 16K head_dim 128 957 against 1142 with 2 instead of 1, 4K x 64K 966 against 1031
// with 8 instead of 4.)
constexpr int kMaxTilesPerSplit = 128;
int uniform_splits(const Problem& pr, int sms) {
  const long long n_qblk = (pr.Sq + kBM2 - 1) / kBM2;
  const long long base = n_qblk * pr.B * pr.H;
  const long long kv_tiles = (pr.Skv + kBN - 1) / kBN;
  if (base <= 0 || kv_tiles < 16) return 1;
  int s = 1;
  while (s < 32 && ((kv_tiles + s - 1) / s > kMaxTilesPerSplit || base * s < 4LL * sms) &&
         kv_tiles / (2 * s) >= 8)
    s *= 2;
  return s;
}

// Modelled duration (in key-tile steps) of one launch with `splits` key splits: the items in
// the kernel's own order (item_coords) handed to the earliest free SM, each costing its key
// tiles + a per-item overhead (~2 steps: Q load, first and last steps without the other tile,
// epilogue; measured by tracing item start/end times), + for every query tile split into
// several parts the partial written to and read back from L2 (128 rows x head_dim fp32 each).
double model_launch_steps(const Problem& pr, int splits, int sms) {
  constexpr double kItemOverhead = 2.0;
  const double part_cost = pr.D >= 128 ? 0.35 : 0.18;
  FwdParams p{};
  p.B = (int)pr.B;
  p.H = (int)pr.H;
  p.Sq = (int)pr.Sq;
  p.Skv = (int)pr.Skv;
  p.n_qblk = (int)((pr.Sq + kBM2 - 1) / kBM2);
  p.splits = splits;
  const int kv_tiles = (int)((pr.Skv + kBN - 1) / kBN);
  p.tiles_per_split = (kv_tiles + splits - 1) / splits;
  p.heavy_first = pr.causal ? 1 : 0;
  p.n_groups = sched_groups(pr.B * pr.H, (long long)p.n_qblk * splits, sms);
  const MaskSpec m = mask_of(pr);
  // every unit has the same items: cost per (query block, split), computed once
  std::vector<double> cost((size_t)p.n_qblk * splits, 0.0);
  for (int qb = 0; qb < p.n_qblk; ++qb) {
    int ulo[2], uhi[2], nparts[2];
    for (int t = 0; t < 2; ++t) {
      const long long r0 = (long long)qb * 256 + t * 128;
      const long long r1 = std::min<long long>(r0 + 128, pr.Sq);
      kv_tile_range(m, r0, r1, kBN, ulo[t], uhi[t]);
      nparts[t] = uhi[t] > ulo[t] ? (uhi[t] - 1) / p.tiles_per_split - ulo[t] / p.tiles_per_split + 1 : 0;
    }
    for (int sp = 0; sp < splits; ++sp) {
      const int s_lo = sp * p.tiles_per_split, s_hi = s_lo + p.tiles_per_split;
      int lo = 1 << 30, hi = -1;
      double extra = 0.0;
      for (int t = 0; t < 2; ++t) {
        const int a = std::max(ulo[t], s_lo), b = std::min(uhi[t], s_hi);
        if (b <= a) continue;
        lo = std::min(lo, a);
        hi = std::max(hi, b);
        if (nparts[t] >= 2)  // write the partial; the last part (modelled: the final split) merges
          extra += part_cost * (1.0 + (sp == (uhi[t] - 1) / p.tiles_per_split ? nparts[t] : 0));
      }
      if (hi > lo) cost[(size_t)qb * splits + sp] = (hi - lo) + kItemOverhead + extra;
    }
  }
  const long long n_items = (long long)p.n_qblk * pr.B * pr.H * splits;
  std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
  for (int i = 0; i < sms; ++i) free_at.push(0.0);
  double makespan = 0.0;
  for (long long idx = 0; idx < n_items; ++idx) {
    int bh, sp, qb;
    item_coords(p, (int)idx, bh, sp, qb);
    const double c = cost[(size_t)qb * splits + sp];
    if (c <= 0.0) continue;
    const double t = free_at.top() + c;
    free_at.pop();
    free_at.push(t);
    makespan = std::max(makespan, t);
  }
  return makespan;
}

// Key-range split count of the tensor-core kernel.  Long unmasked key ranges over many items
// use the uniform rule.  Otherwise (causal or windowed masks, or few items per SM) the launch
// is modelled for no split and for splits of 128 down to 8 key tiles, and the count with the
// shortest modelled launch is taken (a split must save 3 %): with few (batch, head) units per
// GPU — e.g. one GPU's share of a call split across GPUs — the heaviest causal query blocks or
// the last wave of window items would otherwise run on alone at the end of the launch.
// Decisions are cached per shape and SM count.
int choose_splits(const Problem& pr, int sms) {
  const long long n_qblk = (pr.Sq + kBM2 - 1) / kBM2;
  const long long units = pr.B * pr.H;
  const int kv_tiles = (int)((pr.Skv + kBN - 1) / kBN);
  const bool masked = pr.causal || pr.wl >= 0 || pr.wr >= 0;
  const int uniform = masked ? 1 : uniform_splits(pr, sms);
  const long long items = n_qblk * units;
  // many items per SM and short items: the dispatch order already balances the launch
  if (items <= 0 || kv_tiles < 4 || items >= 16LL * sms || items * 64 > (1LL << 24))
    return uniform;
  struct Key {
    long long units, Sq, Skv, wl, wr, qoff, kvoff;
    int causal, D, sms;
    bool operator==(const Key& o) const {
      return units == o.units && Sq == o.Sq && Skv == o.Skv && wl == o.wl && wr == o.wr &&
             qoff == o.qoff && kvoff == o.kvoff && causal == o.causal && D == o.D && sms == o.sms;
    }
  };
  static std::mutex mu;
  static std::vector<std::pair<Key, int>> cache;
  const Key key{units, pr.Sq, pr.Skv, pr.wl, pr.wr, pr.qoff, pr.kvoff, pr.causal, (int)pr.D, sms};
  {
    std::lock_guard<std::mutex> g(mu);
    for (const auto& e : cache)
      if (e.first == key) return e.second;
  }
  int best = uniform;
  double best_t = model_launch_steps(pr, uniform, sms);
  const double base_t = best_t;
  for (int T : {128, 96, 64, 48, 32, 24, 16, 12, 8}) {
    if (T >= kv_tiles) continue;
    const int sp = std::min(32, (kv_tiles + T - 1) / T);
    if (sp == best || sp <= 1) continue;
    const double t = model_launch_steps(pr, sp, sms);
    if (t < best_t && t < 0.97 * base_t) {
      best_t = t;
      best = sp;
    }
  }
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() >= 256) cache.erase(cache.begin());
  cache.emplace_back(key, best);
  return best;
}

// Key splits of the fp32 kernel (two resident CTAs of 64 query rows per SM): split only while
// the query blocks alone would not fill one wave of resident CTAs, keeping at least 4 key tiles
// per split and at most 8 splits.  With the causal blocks ordered heaviest first, extra splits
// cost more (partials written, merged by the last split) than the tail they remove (config 1,
// 384 query blocks: 1 / 2 / 3 / 4 splits 23.5 / 23.1 / 22.0 / 21.4 TFLOPS).
int choose_splits_f32(const Problem& pr, int sms) {
  const int bm = 64, bn = pr.D >= 128 ? 32 : 64;
  const long long base = (pr.Sq + bm - 1) / bm * pr.B * pr.H;
  const long long kv_tiles = (pr.Skv + bn - 1) / bn;
  int s = 1;
  while (s < 8 && base * s < 2LL * sms && kv_tiles / (2 * s) >= 4) s *= 2;
  return s;
}

// Workspace of the fp32 kernel's key splits: fp32 partials [split][B][H][Sq][D], then their
// LSEs [split][B][H][Sq], then one counter per 64-row query block (the split that completes a
// block's count merges its partials inside the kernel).
size_t f32_lse_offset(const Problem& pr, int splits) {
  const size_t rows = (size_t)splits * pr.B * pr.H * pr.Sq;
  return ((rows * pr.D * 4) + 255) / 256 * 256;
}
size_t f32_cnt_offset(const Problem& pr, int splits) {
  const size_t rows = (size_t)splits * pr.B * pr.H * pr.Sq;
  return (f32_lse_offset(pr, splits) + rows * 4 + 255) / 256 * 256;
}
size_t f32_blocks(const Problem& pr) { return (size_t)((pr.Sq + 63) / 64) * pr.B * pr.H; }
size_t split_workspace_f32(const Problem& pr, int splits) {
  if (splits <= 1) return 0;
  return f32_cnt_offset(pr, splits) + f32_blocks(pr) * 4;
}

// Workspace of the tensor-core kernel's key splits (merged inside the kernel): one counter per
// query tile of 128 rows, then per (query tile, split) the partial's 128 LSEs and its 128 x D
// normalised fp32 outputs (FwdParams::part_o / part_lse / tile_cnt).
struct TcSplitLayout {
  size_t tiles, cnt_bytes, lse_bytes, o_bytes;
  size_t total() const { return cnt_bytes + lse_bytes + o_bytes; }
};
TcSplitLayout tc_split_layout(const Problem& pr, int splits) {
  TcSplitLayout l{0, 0, 0, 0};
  if (splits <= 1) return l;
  // query tiles as the kernel numbers them: two per 256-row query block (FwdParams::n_qtile)
  const size_t tiles = (size_t)pr.B * pr.H * 2 * ((pr.Sq + kBM2 - 1) / kBM2);
  l.tiles = tiles;
  l.cnt_bytes = (tiles * 4 + 255) / 256 * 256;
  l.lse_bytes = tiles * splits * 128 * 4;
  l.o_bytes = tiles * splits * 128 * pr.D * 4;
  return l;
}
size_t split_workspace(const Problem& pr, int splits) {
  return pr.dtype == MLXP_DTYPE_FP32 ? split_workspace_f32(pr, splits)
                                     : tc_split_layout(pr, splits).total();
}

// Scratch of mlxp_attn_fwd_split_noalloc: a fixed array in the library's device image, so the
// entry point needs no allocation.  Every GPU that loads the library holds it until exit.
// Its device address is looked up once per device (the first call on that device).
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
void* g_noalloc_ptr[kMaxDevices] = {};

int noalloc_scratch(void** out) {
  int dev;
  if (int rc = current_device(dev)) return rc;
  std::lock_guard<std::mutex> g(g_dev_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-allocation scratch)");
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return MLXP_OK;
}

template <int D, bool BF16, bool BIAS, bool ROPE>
struct TcKernel {
  static constexpr int NS = (D == 128) ? 2 : 3;  // K/V ring stages
  using Cfg = Sm100Cfg<D, NS>;
  // attribute-cache bits 32..43: (head_dim, element type) x (plain, bias, RoPE)
  static constexpr unsigned long long kBit =
      1ull << (32 + (D == 128 ? 0 : 1) + (BF16 ? 0 : 2) + 4 * (BIAS ? 1 : ROPE ? 2 : 0));
  static int launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                    const CUtensorMap& mo, const FwdParams& p, cudaStream_t stream) {
    auto kern = attn_fwd_sm100_kernel<D, BF16, NS, BIAS, ROPE>;
    if (int rc = ensure_smem_attr(kern, Cfg::SMEM_ALLOC, kBit)) return rc;
    const long long items = (long long)p.n_qblk * p.B * p.H * p.splits;
    if (items <= 0) return MLXP_OK;
    int sms = 0;
    if (int rc = device_info(nullptr, &sms)) return rc;
    const long long grid = std::min<long long>(items, sms);  // persistent: one CTA per SM
    kern<<<(unsigned)grid, Cfg::THREADS, Cfg::SMEM_ALLOC, stream>>>(mq, mk, mv, mo, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      cudaFuncAttributes fa{};
      cudaFuncGetAttributes(&fa, kern);
      return fail(MLXP_ERR_CUDA,
                  "attn_fwd_sm100 launch: %s (regs/thread %d, max threads/block %d, dynamic smem "
                  "%d of max %d, threads %d, grid %lld)",
                  cudaGetErrorString(e), fa.numRegs, fa.maxThreadsPerBlock, Cfg::SMEM_ALLOC,
                  fa.maxDynamicSharedSizeBytes, Cfg::THREADS, grid);
    }
    return MLXP_OK;
  }
};

template <bool BIAS, bool ROPE>
int launch_tc_t(int D, bool bf16, const CUtensorMap& mq, const CUtensorMap& mk,
                const CUtensorMap& mv, const CUtensorMap& mo, const FwdParams& p, cudaStream_t s) {
  if (D == 128) return bf16 ? TcKernel<128, true, BIAS, ROPE>::launch(mq, mk, mv, mo, p, s)
                            : TcKernel<128, false, BIAS, ROPE>::launch(mq, mk, mv, mo, p, s);
  return bf16 ? TcKernel<64, true, BIAS, ROPE>::launch(mq, mk, mv, mo, p, s)
              : TcKernel<64, false, BIAS, ROPE>::launch(mq, mk, mv, mo, p, s);
}
// The bias (custom mask) and RoPE variants are separate instantiations: the default kernel
// carries no trace of either.
int launch_tc(int D, bool bf16, const CUtensorMap& mq, const CUtensorMap& mk,
              const CUtensorMap& mv, const CUtensorMap& mo, const FwdParams& p, cudaStream_t s) {
  if (p.bias != nullptr) return launch_tc_t<true, false>(D, bf16, mq, mk, mv, mo, p, s);
  if (p.rope_items > 0) return launch_tc_t<false, true>(D, bf16, mq, mk, mv, mo, p, s);
  return launch_tc_t<false, false>(D, bf16, mq, mk, mv, mo, p, s);
}

template <int D>
int launch_f32_t(const FwdParamsF32& p, cudaStream_t s) {
  using C = F32Cfg<D>;
  auto kern = attn_fwd_fp32_kernel<D>;
  if (int rc = ensure_smem_attr(kern, C::SMEM_BYTES, 1u << (8 + (D / 32)))) return rc;
  const long long grid = (long long)((p.Sq + C::BM - 1) / C::BM) * p.B * p.H * p.splits;
  if (grid <= 0) return MLXP_OK;
  kern<<<(unsigned)grid, 256, C::SMEM_BYTES, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attn_fwd_fp32 launch");
  return MLXP_OK;
}

int check_out_strides(const void* o, const int64_t st[4], int align_elems, const char* name) {
  if (o == nullptr) return fail(MLXP_ERR_INVALID, "%s is null", name);
  if (st[3] != 1) return fail(MLXP_ERR_INVALID, "%s: head_dim stride must be 1", name);
  if (reinterpret_cast<uintptr_t>(o) % 16)
    return fail(MLXP_ERR_INVALID, "%s: base address must be 16-byte aligned", name);
  for (int i = 0; i < 3; ++i)
    if (st[i] % align_elems)
      return fail(MLXP_ERR_INVALID, "%s: strides must be multiples of 16 bytes", name);
  return MLXP_OK;
}

int fill_empty(const Problem& pr, void* o, float* lse, const int64_t ost[4], cudaStream_t s) {
  const long long rows = pr.B * pr.H * pr.Sq;
  if (rows == 0) return MLXP_OK;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  if (pr.dtype == MLXP_DTYPE_FP32)
    fill_empty_kernel<float><<<grid, 256, 0, s>>>((float*)o, lse, rows, pr.H, pr.Sq, pr.D, ost[0], ost[1], ost[2]);
  else if (pr.dtype == MLXP_DTYPE_BF16)
    fill_empty_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((__nv_bfloat16*)o, lse, rows, pr.H, pr.Sq, pr.D, ost[0], ost[1], ost[2]);
  else
    fill_empty_kernel<__half><<<grid, 256, 0, s>>>((__half*)o, lse, rows, pr.H, pr.Sq, pr.D, ost[0], ost[1], ost[2]);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "fill_empty launch");
}

template <typename OutT>
int launch_merge(const float* o_parts, const float* lse_parts, int n, void* o, float* lse_out,
                 const Problem& pr, const int64_t ost[4], cudaStream_t s) {
  const long long rows = pr.B * pr.H * pr.Sq;
  if (rows == 0) return MLXP_OK;
  lse_merge_kernel<OutT><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(
      o_parts, lse_parts, n, (OutT*)o, lse_out, (int)pr.B, (int)pr.H, (int)pr.Sq, (int)pr.D,
      ost[0], ost[1], ost[2]);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "lse_merge launch");
}

int merge_dispatch(const float* o_parts, const float* lse_parts, int n, void* o, float* lse_out,
                   const Problem& pr, const int64_t ost[4], cudaStream_t s) {
  if (pr.dtype == MLXP_DTYPE_FP32) return launch_merge<float>(o_parts, lse_parts, n, o, lse_out, pr, ost, s);
  if (pr.dtype == MLXP_DTYPE_BF16)
    return launch_merge<__nv_bfloat16>(o_parts, lse_parts, n, o, lse_out, pr, ost, s);
  return launch_merge<__half>(o_parts, lse_parts, n, o, lse_out, pr, ost, s);
}

// Shared implementation of mlxp_attn_fwd (out_f32 = 0) and mlxp_attn_fwd_partial (out_f32 = 1).
// RoPE applied inside the attention launch (mlxp_rope_attn_fwd): fp32 cos/sin tables
// [n_pos][D/2] and the position of row 0 of q and of k.
struct RopeArgs {
  const float* cosc;
  const float* sinc;
  int64_t n_pos, q_pos, k_pos;
};

// Workspace of RoPE inside the attention launch: one counter per (batch, head) unit (an upper
// bound on the scheduling groups), then the rotated Q and K copies (contiguous BHSD); the
// key-split workspace, when splits are used, follows.
struct RopeLayout {
  size_t cnt_bytes, q_bytes, k_bytes;
  size_t total() const { return cnt_bytes + q_bytes + k_bytes; }
};
RopeLayout rope_layout(const Problem& pr) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  RopeLayout l;
  l.cnt_bytes = up((size_t)pr.B * pr.H * 4 + 4);  // per-group counters + the item counter
  l.q_bytes = up((size_t)pr.B * pr.H * pr.Sq * pr.D * 2);
  l.k_bytes = up((size_t)pr.B * pr.H * pr.Skv * pr.D * 2);
  return l;
}

// Output modes of attn_fwd_impl: the input dtype (mlxp_attn_fwd), normalised fp32 + LSE
// (mlxp_attn_fwd_partial), or merged into a running fp32 result (mlxp_attn_fwd_accumulate).
enum FwdMode { kOutNormal = 0, kOutPartial = 1, kOutAccumulate = 2 };

int attn_fwd_impl(const void* q, const void* k, const void* v, void* o, float* lse,
                  const Problem& pr, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                  const int64_t* os, float scale, int64_t kv_splits, void* ws, size_t ws_bytes,
                  int mode, cudaStream_t stream, const RopeArgs* rope = nullptr,
                  const float* bias = nullptr, const int64_t* bias_st = nullptr) {
  const bool out_f32 = mode != kOutNormal;
  const bool accumulate = mode == kOutAccumulate;
  if (int rc = validate(pr)) return rc;
  if (!(scale > 0.f) || !std::isfinite(scale))
    return fail(MLXP_ERR_INVALID, "scale must be positive and finite");
  // Empty tensors may have null data pointers: q only matters when Sq > 0, k/v when Skv > 0.
  if ((pr.Sq > 0 && !q) || (pr.Skv > 0 && (!k || !v)))
    return fail(MLXP_ERR_INVALID, "q, k and v must be non-null");
  if (!qs || !ks || !vs || !os) return fail(MLXP_ERR_INVALID, "stride arrays must be non-null");
  if (out_f32 && lse == nullptr) return fail(MLXP_ERR_INVALID, "partial output needs lse");
  const bool fp32 = pr.dtype == MLXP_DTYPE_FP32;
  if (out_f32 && fp32)
    return fail(MLXP_ERR_UNSUPPORTED, "partial and accumulating outputs take bf16/fp16 inputs");
  if (bias != nullptr) {
    // fp32, unit key stride, 16-byte aligned rows (the kernels read 4 keys at a time)
    if (!bias_st || bias_st[3] != 1)
      return fail(MLXP_ERR_INVALID, "mask: the key (last) stride must be 1");
    if (reinterpret_cast<uintptr_t>(bias) % 16 || (bias_st[0] % 4) || (bias_st[1] % 4) ||
        (bias_st[2] % 4) || bias_st[0] < 0 || bias_st[1] < 0 || bias_st[2] < 0)
      return fail(MLXP_ERR_INVALID, "mask: base and (batch, head, row) strides must be 16-byte "
                                    "aligned and non-negative");
    if (out_f32 || rope) return fail(MLXP_ERR_UNSUPPORTED, "mask with this entry point");
  }
  if (int rc = check_out_strides(o, os, (fp32 || out_f32) ? 4 : 8, "o")) return rc;
  if (reinterpret_cast<uintptr_t>(lse) % 4) return fail(MLXP_ERR_INVALID, "lse misaligned");
  if (pr.Sq == 0) return MLXP_OK;
  int* status = nullptr;
  int sms = 0;
  if (int rc = device_info(&status, &sms)) return rc;

  Problem pe = pr;
  if (out_f32) pe.dtype = MLXP_DTYPE_FP32;  // output element type for the empty fill
  if (pr.Skv == 0) return accumulate ? MLXP_OK : fill_empty(pe, o, lse, os, stream);

  const float scale_log2 = scale * 1.4426950408889634f;
  if (fp32) {
    for (const int64_t* st : {qs, ks, vs})
      if (st[3] != 1 || (st[0] % 4) || (st[1] % 4) || (st[2] % 4))
        return fail(MLXP_ERR_INVALID, "fp32 q/k/v need unit head_dim stride and 16-byte aligned rows");
    for (const void* ptr : {q, k, v})
      if (reinterpret_cast<uintptr_t>(ptr) % 16)
        return fail(MLXP_ERR_INVALID, "fp32 q/k/v base addresses must be 16-byte aligned");
    FwdParamsF32 p{};
    p.B = (int)pr.B;
    p.H = (int)pr.H;
    p.kv_group = (int)(pr.H / pr.kv_heads());
    p.Sq = (int)pr.Sq;
    p.Skv = (int)pr.Skv;
    p.q = (const float*)q;
    p.k = (const float*)k;
    p.v = (const float*)v;
    p.q_sb = qs[0]; p.q_sh = qs[1]; p.q_ss = qs[2];
    p.k_sb = ks[0]; p.k_sh = ks[1]; p.k_ss = ks[2];
    p.v_sb = vs[0]; p.v_sh = vs[1]; p.v_ss = vs[2];
    p.o = (float*)o;
    p.o_sb = os[0]; p.o_sh = os[1]; p.o_ss = os[2];
    p.lse = lse;
    p.scale_log2 = scale_log2;
    p.mask = mask_of(pr);
    if (bias) {
      p.bias = bias;
      p.bias_sb = bias_st[0];
      p.bias_sh = bias_st[1];
      p.bias_sq = bias_st[2];
    }
    int splits = 1;
    if (!out_f32) {
      if (kv_splits == 0) splits = choose_splits_f32(pr, sms);
      else if (kv_splits > 1) splits = (int)std::min<int64_t>(kv_splits, (pr.Skv + 31) / 32);
    }
    p.splits = splits;
    if (splits > 1) {  // partials in the workspace, merged inside the kernel into o
      const size_t need = split_workspace(pr, splits);
      if (ws == nullptr || ws_bytes < need)
        return fail(MLXP_ERR_WORKSPACE, "split-KV needs %zu bytes of workspace, got %zu", need,
                    ws_bytes);
      if (reinterpret_cast<uintptr_t>(ws) % 256)
        return fail(MLXP_ERR_INVALID, "workspace must be 256-byte aligned");
      const long long rows = pr.B * pr.H * pr.Sq;
      float* o_parts = static_cast<float*>(ws);
      float* lse_parts =
          reinterpret_cast<float*>(static_cast<char*>(ws) + f32_lse_offset(pr, splits));
      p.blk_cnt = reinterpret_cast<unsigned*>(static_cast<char*>(ws) + f32_cnt_offset(pr, splits));
      cudaError_t e = cudaMemsetAsync(p.blk_cnt, 0, f32_blocks(pr) * 4, stream);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(split counters)");
      p.o_final = (float*)o;
      p.of_sb = os[0];
      p.of_sh = os[1];
      p.of_ss = os[2];
      p.lse_final = lse;
      p.o = o_parts;
      p.o_sh = pr.Sq * pr.D;
      p.o_sb = pr.H * p.o_sh;
      p.o_ss = pr.D;
      p.o_split = rows * pr.D;
      p.lse = lse_parts;
      p.lse_split = rows;
    }
    int rc;
    switch (pr.D) {
      case 32: rc = launch_f32_t<32>(p, stream); break;
      case 64: rc = launch_f32_t<64>(p, stream); break;
      default: rc = launch_f32_t<128>(p, stream); break;
    }
    return rc;
  }

  const bool bf16 = pr.dtype == MLXP_DTYPE_BF16;
  CUtensorMap mq, mk, mv;
  FwdParams p{};
  const CUtensorMapDataType dt16 =
      bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // With RoPE the kernel's rotation items write rotated Q and K into the workspace, and the
  // Q/K tensor maps read those contiguous copies instead of q and k.
  const void* q_map = q;
  const void* k_map = k;
  const int64_t* qs_map = qs;
  const int64_t* ks_map = ks;
  int64_t rq_st[4], rk_st[4];
  RopeLayout rlay{0, 0, 0};
  if (rope) {
    if (pr.kv_heads() != pr.H)
      return fail(MLXP_ERR_UNSUPPORTED, "RoPE inside the attention launch needs as many K/V "
                                        "heads as query heads");
    if (!rope->cosc || !rope->sinc) return fail(MLXP_ERR_INVALID, "cos/sin tables must be non-null");
    if ((reinterpret_cast<uintptr_t>(rope->cosc) | reinterpret_cast<uintptr_t>(rope->sinc)) % 16)
      return fail(MLXP_ERR_INVALID, "cos/sin tables must be 16-byte aligned");
    if (rope->q_pos < 0 || rope->k_pos < 0 || rope->q_pos + pr.Sq > rope->n_pos ||
        rope->k_pos + pr.Skv > rope->n_pos)
      return fail(MLXP_ERR_INVALID,
                  "positions [%lld, %lld) / [%lld, %lld) exceed the cos/sin table of %lld positions",
                  (long long)rope->q_pos, (long long)(rope->q_pos + pr.Sq), (long long)rope->k_pos,
                  (long long)(rope->k_pos + pr.Skv), (long long)rope->n_pos);
    if (int rc = check_out_strides(q, qs, 8, "q")) return rc;  // 16-byte row accesses
    if (int rc = check_out_strides(k, ks, 8, "k")) return rc;
    rlay = rope_layout(pr);
    if (ws == nullptr || ws_bytes < rlay.total())
      return fail(MLXP_ERR_WORKSPACE, "RoPE in the attention launch needs %zu bytes of workspace, "
                  "got %zu", rlay.total(), ws_bytes);
    if (reinterpret_cast<uintptr_t>(ws) % 256)
      return fail(MLXP_ERR_INVALID, "workspace must be 256-byte aligned");
    char* base = static_cast<char*>(ws);
    p.rot_done = reinterpret_cast<unsigned*>(base);
    p.rot_counter = p.rot_done + pr.B * pr.H;  // one past the per-group counters
    p.rq_dst = base + rlay.cnt_bytes;
    p.rk_dst = base + rlay.cnt_bytes + rlay.q_bytes;
    p.rq_src = q;
    p.rk_src = k;
    for (int i = 0; i < 3; ++i) {
      p.rq_s[i] = qs[i];
      p.rk_s[i] = ks[i];
    }
    p.rope_cos = rope->cosc;
    p.rope_sin = rope->sinc;
    p.rope_q_pos = rope->q_pos;
    p.rope_k_pos = rope->k_pos;
    p.rope_q_items = (int)((pr.Sq + kRopeRows - 1) / kRopeRows);
    p.rope_items = p.rope_q_items + (int)((pr.Skv + kRopeRows - 1) / kRopeRows);
    const int64_t qc[4] = {pr.H * pr.Sq * pr.D, pr.Sq * pr.D, pr.D, 1};
    const int64_t kc[4] = {pr.H * pr.Skv * pr.D, pr.Skv * pr.D, pr.D, 1};
    std::memcpy(rq_st, qc, sizeof(qc));
    std::memcpy(rk_st, kc, sizeof(kc));
    q_map = p.rq_dst;
    k_map = p.rk_dst;
    qs_map = rq_st;
    ks_map = rk_st;
    // what follows (key splits) uses the rest of the workspace
    ws = base + rlay.total();
    ws_bytes -= rlay.total();
  }
  if (int rc = make_tmap(q_map, dt16, 2, pr.B, pr.H, pr.Sq, pr.D, qs_map, 128, 64, "q", &mq,
                         &p.cq))
    return rc;
  if (int rc = make_tmap(k_map, dt16, 2, pr.B, pr.kv_heads(), pr.Skv, pr.D, ks_map, kBN, 64, "k",
                         &mk, &p.ck))
    return rc;
  if (int rc = make_tmap(v, dt16, 2, pr.B, pr.kv_heads(), pr.Skv, pr.D, vs, kBN, 64, "v", &mv,
                         &p.cv))
    return rc;
  p.kv_group = (int)(pr.H / pr.kv_heads());

  int splits = 1;
  if (!out_f32) {
    if (kv_splits == 0) splits = choose_splits(pr, sms);
    else if (kv_splits > 1) splits = (int)std::min<int64_t>(kv_splits, (pr.Skv + kBN - 1) / kBN);
  }
  p.B = (int)pr.B;
  p.H = (int)pr.H;
  p.Sq = (int)pr.Sq;
  p.Skv = (int)pr.Skv;
  p.n_qblk = (int)((pr.Sq + kBM2 - 1) / kBM2);
  p.n_qtile = 2 * p.n_qblk;
  p.splits = splits;
  const int kv_tiles = (int)((pr.Skv + kBN - 1) / kBN);
  p.tiles_per_split = (kv_tiles + splits - 1) / splits;
  p.heavy_first = pr.causal ? 1 : 0;
  p.n_groups = sched_groups(pr.B * pr.H, (long long)p.n_qblk * splits, sms);
  p.scale_log2 = scale_log2;
  p.mask = mask_of(pr);
  if (bias) {
    p.bias = bias;
    p.bias_sb = bias_st[0];
    p.bias_sh = bias_st[1];
    p.bias_sq = bias_st[2];
    p.inv_scale = 1.0f / scale;
  }
  p.status = status;
  p.timeout_ns = g_timeout_ns.load();
  {
    int dev;
    if (int rc = current_device(dev)) return rc;
    const unsigned slot = g_counter_seq[dev].fetch_add(1) % kCounterSlots;
    p.work_counter = g_counter_ptr[dev] + 2 * slot;
  }

  // O is written through a tensor map: 128-row boxes of 128 bytes (64 bf16/fp16 or 32 fp32
  // columns).  The output was validated above (16-byte aligned base, 16-byte strides).
  CUtensorMap mo;
  p.out_f32 = out_f32 ? 1 : 0;
  p.lse = lse;
  if (accumulate) {
    p.accumulate = 1;
    p.acc_o = static_cast<const float*>(o);
    p.acc_sb = os[0];
    p.acc_sh = os[1];
    p.acc_ss = os[2];
  }
  if (int rc = out_f32 ? make_tmap(o, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, pr.B, pr.H, pr.Sq, pr.D,
                                   os, 128, 32, "o", &mo, &p.co)
                       : make_tmap(o, dt16, 2, pr.B, pr.H, pr.Sq, pr.D, os, 128, 64, "o", &mo,
                                   &p.co))
    return rc;
  if (splits > 1) {
    // key splits are merged inside the kernel; the workspace holds the partials and the
    // per-query-tile counters, which must start at zero
    const TcSplitLayout lay = tc_split_layout(pr, splits);
    if (ws == nullptr || ws_bytes < lay.total())
      return fail(MLXP_ERR_WORKSPACE, "workspace of %zu bytes needed for %d key splits, got %zu",
                  lay.total(), splits, ws_bytes);
    if (reinterpret_cast<uintptr_t>(ws) % 256)
      return fail(MLXP_ERR_INVALID, "workspace must be 256-byte aligned");
    char* base = static_cast<char*>(ws);
    p.tile_cnt = reinterpret_cast<unsigned*>(base);
    p.part_lse = reinterpret_cast<float*>(base + lay.cnt_bytes);
    p.part_o = reinterpret_cast<float*>(base + lay.cnt_bytes + lay.lse_bytes);
    p.part_tiles = (long long)lay.tiles;
    cudaError_t e = cudaMemsetAsync(base, 0, lay.cnt_bytes, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(split counters)");
  }
  if (rope) {
    cudaError_t e = cudaMemsetAsync(p.rot_done, 0, rlay.cnt_bytes, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(rotation counters)");
  }
  return launch_tc((int)pr.D, bf16, mq, mk, mv, mo, p, stream);
}

// RoPE of one or two tensors ([B][H][S][D] in element strides) in one launch.
int rope_launch(int dtype, int64_t D, RopeParams& rp, const int64_t* const xs[2],
                const int64_t* const ys[2], cudaStream_t stream) {
  if (D < 2 || (D % 2)) return fail(MLXP_ERR_INVALID, "head_dim must be even for RoPE, got %lld", (long long)D);
  if (!rp.cosc || !rp.sinc) return fail(MLXP_ERR_INVALID, "cos/sin caches must be non-null");
  if (dtype < 0 || dtype > 2) return fail(MLXP_ERR_INVALID, "unknown dtype %d", dtype);
  const int es = dtype == MLXP_DTYPE_FP32 ? 4 : 2;
  const int vec = 16 / es;
  rp.half = (int)(D / 2);
  bool vec_ok = (rp.half % vec) == 0 && ((rp.half * es) % 16) == 0;
  long long total = 0;
  for (int i = 0; i < rp.n; ++i) {
    RopeTensor& t = rp.t[i];
    if (!t.x || !t.y || !xs[i] || !ys[i]) return fail(MLXP_ERR_INVALID, "rope tensors must be non-null");
    if (xs[i][3] != 1 || ys[i][3] != 1) return fail(MLXP_ERR_INVALID, "head_dim stride must be 1");
    if (t.pos_offset < 0 || t.pos_offset + t.S > rp.n_pos)
      return fail(MLXP_ERR_INVALID,
                  "positions [%lld, %lld) exceed the cos/sin cache of %lld positions",
                  (long long)t.pos_offset, (long long)(t.pos_offset + t.S), (long long)rp.n_pos);
    for (int d = 0; d < 3; ++d) {
      t.xs[d] = xs[i][d];
      t.ys[d] = ys[i][d];
      if ((xs[i][d] * es) % 16 || (ys[i][d] * es) % 16) vec_ok = false;
    }
    if (reinterpret_cast<uintptr_t>(t.x) % 16 || reinterpret_cast<uintptr_t>(t.y) % 16) vec_ok = false;
    total += t.rows;
  }
  if (total == 0) return MLXP_OK;
  int sms = 148;
  if (int rc = device_info(nullptr, &sms)) return rc;
  long long tokens = 0;  // one block per token (batch, position) at a time
  for (int i = 0; i < rp.n; ++i) tokens += rp.t[i].H > 0 ? rp.t[i].rows / rp.t[i].H : 0;
  const unsigned grid = (unsigned)std::max<long long>(1, std::min<long long>(tokens, 16LL * sms));
  if (dtype == MLXP_DTYPE_BF16) {
    if (vec_ok) rope_kernel<__nv_bfloat16, 8><<<grid, 256, 0, stream>>>(rp);
    else rope_kernel<__nv_bfloat16, 1><<<grid, 256, 0, stream>>>(rp);
  } else if (dtype == MLXP_DTYPE_FP16) {
    if (vec_ok) rope_kernel<__half, 8><<<grid, 256, 0, stream>>>(rp);
    else rope_kernel<__half, 1><<<grid, 256, 0, stream>>>(rp);
  } else {
    if (vec_ok) rope_kernel<float, 4><<<grid, 256, 0, stream>>>(rp);
    else rope_kernel<float, 1><<<grid, 256, 0, stream>>>(rp);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "rope launch");
}


// ---- paged attention (cache/paged_attention.py) ----

struct PagedProblem {
  int dtype;
  int64_t B, H, Sq, D, Hkv, num_blocks, block_size, max_blocks;
};

int paged_validate(const PagedProblem& pp) {
  if (pp.B < 0 || pp.H <= 0 || pp.Sq < 0 || pp.Hkv <= 0 || pp.num_blocks < 0 ||
      pp.block_size <= 0 || pp.max_blocks < 0)
    return fail(MLXP_ERR_INVALID,
                "invalid paged shape B=%lld H=%lld Sq=%lld kv_heads=%lld num_blocks=%lld "
                "block_size=%lld max_blocks=%lld",
                (long long)pp.B, (long long)pp.H, (long long)pp.Sq, (long long)pp.Hkv,
                (long long)pp.num_blocks, (long long)pp.block_size, (long long)pp.max_blocks);
  if (pp.H % pp.Hkv)
    return fail(MLXP_ERR_INVALID, "num_heads (%lld) must be divisible by the pool's heads (%lld)",
                (long long)pp.H, (long long)pp.Hkv);
  if (pp.dtype < 0 || pp.dtype > 2) return fail(MLXP_ERR_INVALID, "unknown dtype %d", pp.dtype);
  if (pp.D != 32 && pp.D != 64 && pp.D != 128)
    return fail(MLXP_ERR_UNSUPPORTED, "paged attention supports head_dim 32, 64 and 128, got %lld",
                (long long)pp.D);
  if (pp.B * pp.Sq > INT32_MAX || pp.max_blocks * pp.block_size > INT32_MAX ||
      pp.num_blocks > INT32_MAX || pp.H > INT32_MAX)
    return fail(MLXP_ERR_INVALID, "paged shape too large");
  return MLXP_OK;
}

// Grid of the stream-K decomposition (paged_attn.cuh).  kv_splits: 1 = one CTA per (row, head)
// pair (no partials), n > 1 = n CTAs per pair, 0 = automatic: the resident CTA count (3 per SM
// for 16-bit types, 1 for fp32, set by shared memory), or fewer so that every CTA gets at least
// 4 blocks.
// The TMA kernel (paged_attn_tma_kernel) serves bf16/fp16 pools whose block size is a multiple
// of its 16-row chunk; everything else runs the cp.async kernel.
bool paged_tma_shape(const PagedProblem& pp) {
  return pp.dtype != MLXP_DTYPE_FP32 && pp.block_size % kTmaRows == 0 && pp.num_blocks >= 1;
}

long long paged_grid(const PagedProblem& pp, int64_t kv_splits, int sms) {
  const long long pairs = pp.B * pp.Sq * pp.H;
  const long long total = pairs * pp.max_blocks;
  if (total <= 0) return 0;
  const int per_sm = paged_tma_shape(pp) ? 1 : (pp.dtype == MLXP_DTYPE_FP32 ? 1 : 3);
  long long g;
  if (kv_splits == 1) g = pairs;
  else if (kv_splits > 1) g = pairs * std::min<long long>(kv_splits, pp.max_blocks);
  else g = std::min<long long>((long long)sms * per_sm, std::max<long long>(1, total / 4));
  return std::max<long long>(1, std::min<long long>(g, total));
}

// Tensor map of a pool as {D, kv_heads, block_size, num_blocks} with a {D, 1, 16, 1} box.
// Returns false when the pool's address or strides do not suit TMA.
bool make_pool_tmap(const void* ptr, int dtype, const PagedProblem& pp, const int64_t ps[4],
                    CUtensorMap* map) {
  if (get_encode_fn() != MLXP_OK) return false;
  const int es = 2;
  if (reinterpret_cast<uintptr_t>(ptr) % 16) return false;
  int64_t sh = ps[2], st = ps[1], sb = ps[0];
  if (pp.Hkv == 1) sh = (pp.D * es + 15) / 16 * 16 / es;  // unused dimension: any legal stride
  if (pp.num_blocks == 1 && sb <= 0) sb = st * pp.block_size;
  for (int64_t x : {sh, st, sb})
    if (x <= 0 || (x * es) % 16) return false;
  cuuint64_t gdim[4] = {(cuuint64_t)pp.D, (cuuint64_t)pp.Hkv, (cuuint64_t)pp.block_size,
                        (cuuint64_t)pp.num_blocks};
  cuuint64_t gstride[3] = {(cuuint64_t)(sh * es), (cuuint64_t)(st * es), (cuuint64_t)(sb * es)};
  cuuint32_t box[4] = {(cuuint32_t)pp.D, 1, (cuuint32_t)kTmaRows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == MLXP_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = g_encode(map, dt, 4, const_cast<void*>(ptr), gdim, gstride, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int LPR>
int paged_tma_launch_d(const CUtensorMap& mk, const CUtensorMap& mv, const PagedParams& p,
                       unsigned grid, cudaStream_t s) {
  constexpr int smem = paged_tma_smem<T, LPR * 4>();
  static std::atomic<unsigned long long> attr_done{0};  // one bit per device
  int dev;
  if (int rc = current_device(dev)) return rc;
  cudaError_t e;
  if (!(attr_done.load() >> dev & 1ull)) {
    e = cudaFuncSetAttribute(paged_attn_tma_kernel<T, LPR>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(paged attention, TMA)");
    attr_done.fetch_or(1ull << dev);
  }
  paged_attn_tma_kernel<T, LPR><<<grid, 32 * kTmaWarps, smem, s>>>(mk, mv, p);
  e = cudaGetLastError();
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "paged attention launch (TMA)");
}

template <typename T>
int paged_tma_launch_t(const CUtensorMap& mk, const CUtensorMap& mv, const PagedParams& p,
                       int LPR, unsigned grid, cudaStream_t s) {
  if (LPR == 32) return paged_tma_launch_d<T, 32>(mk, mv, p, grid, s);
  if (LPR == 16) return paged_tma_launch_d<T, 16>(mk, mv, p, grid, s);
  return paged_tma_launch_d<T, 8>(mk, mv, p, grid, s);
}

// Partial slots per pair: a pair of max_blocks slots meets at most this many CTA ranges.
long long paged_max_parts(const PagedProblem& pp, long long grid) {
  const long long total = pp.B * pp.Sq * pp.H * pp.max_blocks;
  const long long per = total / grid;  // >= 1: grid <= total
  return (pp.max_blocks + per - 1) / per + 1;
}

// Workspace: fp32 partials and log2-sum-exps per (pair, slot), then the pair counters.  None
// when every CTA owns whole pairs.
size_t paged_workspace(const PagedProblem& pp, long long grid) {
  const long long pairs = pp.B * pp.Sq * pp.H;
  if (grid <= 0 || grid == pairs) return 0;
  const size_t rows = (size_t)pairs * paged_max_parts(pp, grid);
  const size_t o_bytes = (rows * pp.D * 4 + 255) / 256 * 256;
  const size_t l_bytes = (rows * 4 + 255) / 256 * 256;
  return o_bytes + l_bytes + (size_t)pairs * 4;
}

template <typename T, int LPR>
int paged_launch_d(const PagedParams& p, unsigned grid, cudaStream_t s) {
  constexpr int smem = paged_smem_bytes<T>(LPR * 4);
  static std::atomic<unsigned long long> attr_done{0};  // one bit per device
  int dev;
  if (int rc = current_device(dev)) return rc;
  cudaError_t e;
  if (!(attr_done.load() >> dev & 1ull)) {
    e = cudaFuncSetAttribute(paged_attn_kernel<T, LPR>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(paged attention)");
    attr_done.fetch_or(1ull << dev);
  }
  paged_attn_kernel<T, LPR><<<grid, 32 * kPagedWarps, smem, s>>>(p);
  e = cudaGetLastError();
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "paged attention launch");
}

template <typename T>
int paged_launch_t(const PagedParams& p, int LPR, unsigned grid, cudaStream_t s) {
  if (LPR == 32) return paged_launch_d<T, 32>(p, grid, s);
  if (LPR == 16) return paged_launch_d<T, 16>(p, grid, s);
  return paged_launch_d<T, 8>(p, grid, s);
}


// ---- backward (dQ, dK, dV) ----

// The tensor-core backward serves bf16/fp16 with head_dim 64 or 128; it needs the padded L2 and
// Delta rows and the fp32 dQ accumulator.  Everything else runs the CUDA-core backward (Delta).
bool bwd_tc_shape(const Problem& pr) {
  return (pr.dtype == MLXP_DTYPE_BF16 || pr.dtype == MLXP_DTYPE_FP16) &&
         (pr.D == 64 || pr.D == 128) && pr.Sq > 0 && pr.Skv > 0;
}
size_t bwd_tc_rows_bytes(const Problem& pr) {
  const size_t sq_pad = (size_t)(pr.Sq + 63) / 64 * 64;
  return ((size_t)pr.B * pr.H * sq_pad * 4 + 255) / 256 * 256;
}
size_t bwd_workspace(const Problem& pr) {
  const size_t base = ((size_t)pr.B * pr.H * pr.Sq * 4 + 255) / 256 * 256;
  if (!bwd_tc_shape(pr)) return base;
  const size_t acc = ((size_t)pr.B * pr.H * pr.Sq * pr.D * 4 + 255) / 256 * 256;
  return std::max(base, 2 * bwd_tc_rows_bytes(pr) + acc);
}

template <bool kBF16, int D>
int bwd_tc_kernel_launch(const CUtensorMap* m, const BwdTcParams& tp, unsigned grid,
                         cudaStream_t s) {
  using C = BwdTcCfg<D>;
  static std::atomic<unsigned long long> attr_done{0};  // one bit per device
  int dev;
  if (int rc = current_device(dev)) return rc;
  if (!(attr_done.load() >> dev & 1ull)) {
    cudaError_t e = cudaFuncSetAttribute(attn_bwd_sm100_kernel<kBF16, D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_ALLOC);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(backward)");
    attr_done.fetch_or(1ull << dev);
  }
  attn_bwd_sm100_kernel<kBF16, D><<<grid, C::THREADS, C::SMEM_ALLOC, s>>>(m[0], m[1], m[2], m[3],
                                                                         m[4], tp);
  return MLXP_OK;
}

template <typename T, int D>
void bwd_tc_aux_launch(const BwdParams& bp, int Sq_pad, float* lse2, float* delta,
                       const float* acc, bool post, int sms, cudaStream_t s) {
  if (!post) {
    const long long prow = (long long)bp.B * bp.H * Sq_pad;
    bwd_tc_prep_kernel<T, D><<<(unsigned)((prow + 7) / 8), 256, 0, s>>>(bp, Sq_pad, lse2, delta);
    return;
  }
  const long long n8 = (long long)bp.B * bp.H * bp.Sq * (D / 8);
  const unsigned pg = (unsigned)std::min<long long>((n8 + 255) / 256, (long long)sms * 32);
  const bool vec = reinterpret_cast<uintptr_t>(bp.dq) % 16 == 0 && bp.dq_sb % 8 == 0 &&
                   bp.dq_sh % 8 == 0 && bp.dq_ss % 8 == 0;
  if (vec) bwd_tc_post_kernel<T, D, true><<<pg, 256, 0, s>>>(bp, acc);
  else bwd_tc_post_kernel<T, D, false><<<pg, 256, 0, s>>>(bp, acc);
}

// Tensor-core backward; returns MLXP_ERR_UNSUPPORTED (nothing launched) when an operand does
// not suit TMA, so that the caller can take the CUDA-core path.
int bwd_tc_launch(const BwdParams& bp, const Problem& pr, const int64_t* const st[8],
                  void* workspace, cudaStream_t s) {
  const int es = 2;
  const int64_t D = pr.D;
  const CUtensorMapDataType dt = pr.dtype == MLXP_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // dK / dV rows are written with 16-byte stores
  for (const void* ptr : {bp.dk, bp.dv})
    if (reinterpret_cast<uintptr_t>(ptr) % 16) return MLXP_ERR_UNSUPPORTED;
  for (int t : {6, 7})
    for (int d = 0; d < 3; ++d)
      if (st[t][d] % 8) return MLXP_ERR_UNSUPPORTED;
  const int64_t Hkv = pr.kv_heads();
  CUtensorMap maps[5];  // q, k, v, dout, dq accumulator
  BwdTcParams tp{};
  const std::string saved = t_last_error;
  if (make_tmap(bp.q, dt, es, pr.B, pr.H, pr.Sq, D, st[0], 64, 64, "q", &maps[0], &tp.cq) ||
      make_tmap(bp.k, dt, es, pr.B, Hkv, pr.Skv, D, st[1], 128, 64, "k", &maps[1], &tp.ck) ||
      make_tmap(bp.v, dt, es, pr.B, Hkv, pr.Skv, D, st[2], 128, 64, "v", &maps[2], &tp.cv) ||
      make_tmap(bp.dout, dt, es, pr.B, pr.H, pr.Sq, D, st[4], 64, 64, "dout", &maps[3], &tp.cdo)) {
    t_last_error = saved;
    return MLXP_ERR_UNSUPPORTED;
  }
  char* w = static_cast<char*>(workspace);
  const size_t rows = bwd_tc_rows_bytes(pr);
  float* lse2 = reinterpret_cast<float*>(w);
  float* delta = reinterpret_cast<float*>(w + rows);
  float* acc = reinterpret_cast<float*>(w + 2 * rows);
  const int64_t acc_st[4] = {pr.H * pr.Sq * D, pr.Sq * D, D, 1};
  if (int rc = make_tmap(acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, pr.B, pr.H, pr.Sq, D, acc_st,
                         32, 32, "dq accumulator", &maps[4], &tp.cdq))
    return rc;
  int* status = nullptr;
  int sms = 148;
  if (int rc = device_info(&status, &sms)) return rc;
  const int Sq_pad = (int)((pr.Sq + 63) / 64 * 64);
  tp.B = (int)pr.B;
  tp.H = (int)pr.H;
  tp.Sq = (int)pr.Sq;
  tp.Skv = (int)pr.Skv;
  tp.kv_group = bp.kv_group;
  tp.n_kt = (int)((pr.Skv + 127) / 128);
  tp.Sq_pad = Sq_pad;
  tp.lse2 = lse2;
  tp.delta = delta;
  tp.dk = bp.dk;
  tp.dv = bp.dv;
  tp.dk_sb = bp.dk_sb;
  tp.dk_sh = bp.dk_sh;
  tp.dk_ss = bp.dk_ss;
  tp.dv_sb = bp.dv_sb;
  tp.dv_sh = bp.dv_sh;
  tp.dv_ss = bp.dv_ss;
  tp.scale = bp.scale;
  tp.scale_log2 = bp.scale_log2;
  tp.mask = bp.mask;
  tp.status = status;
  tp.timeout_ns = g_timeout_ns.load();
  cudaError_t e = cudaMemsetAsync(acc, 0, (size_t)pr.B * pr.H * pr.Sq * D * 4, s);
  if (e != cudaSuccess) return cuda_fail(e, "dq accumulator reset");
  const bool bf16 = pr.dtype == MLXP_DTYPE_BF16;
  const unsigned grid = (unsigned)(tp.n_kt * pr.B * Hkv);
  int rc;
  if (D == 128) {
    if (bf16) bwd_tc_aux_launch<__nv_bfloat16, 128>(bp, Sq_pad, lse2, delta, acc, false, sms, s);
    else bwd_tc_aux_launch<__half, 128>(bp, Sq_pad, lse2, delta, acc, false, sms, s);
    rc = bf16 ? bwd_tc_kernel_launch<true, 128>(maps, tp, grid, s)
              : bwd_tc_kernel_launch<false, 128>(maps, tp, grid, s);
    if (rc) return rc;
    if (bf16) bwd_tc_aux_launch<__nv_bfloat16, 128>(bp, Sq_pad, lse2, delta, acc, true, sms, s);
    else bwd_tc_aux_launch<__half, 128>(bp, Sq_pad, lse2, delta, acc, true, sms, s);
  } else {
    if (bf16) bwd_tc_aux_launch<__nv_bfloat16, 64>(bp, Sq_pad, lse2, delta, acc, false, sms, s);
    else bwd_tc_aux_launch<__half, 64>(bp, Sq_pad, lse2, delta, acc, false, sms, s);
    rc = bf16 ? bwd_tc_kernel_launch<true, 64>(maps, tp, grid, s)
              : bwd_tc_kernel_launch<false, 64>(maps, tp, grid, s);
    if (rc) return rc;
    if (bf16) bwd_tc_aux_launch<__nv_bfloat16, 64>(bp, Sq_pad, lse2, delta, acc, true, sms, s);
    else bwd_tc_aux_launch<__half, 64>(bp, Sq_pad, lse2, delta, acc, true, sms, s);
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "attention backward launch (tensor cores)");
}

template <typename T, int D>
int bwd_launch_t(const BwdParams& bp, cudaStream_t s) {
  constexpr int smem_kv = bwd_dkdv_smem<D>();
  constexpr int smem_q = bwd_dq_smem<D>();
  // attribute-cache bits 13..30: two per (element type, head_dim) pair
  constexpr int ti = sizeof(T) == 4 ? 0 : (std::is_same<T, __nv_bfloat16>::value ? 1 : 2);
  constexpr int slot = 13 + 2 * (ti * 3 + (D == 32 ? 0 : D == 64 ? 1 : 2));
  if (int rc = ensure_smem_attr(bwd_dkdv_kernel<T, D>, smem_kv, 1u << slot)) return rc;
  if (int rc = ensure_smem_attr(bwd_dq_kernel<T, D>, smem_q, 1u << (slot + 1))) return rc;
  const long long rows = (long long)bp.B * bp.H * bp.Sq;
  bwd_delta_kernel<T><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(bp, D);
  const long long n_kt = (bp.Skv + 63) / 64, n_qt = (bp.Sq + 63) / 64;
  const long long g_kv = n_kt * bp.B * (bp.H / bp.kv_group), g_q = n_qt * bp.B * bp.H;
  if (g_kv > 0) bwd_dkdv_kernel<T, D><<<(unsigned)g_kv, 256, smem_kv, s>>>(bp);
  if (g_q > 0) bwd_dq_kernel<T, D><<<(unsigned)g_q, 256, smem_q, s>>>(bp);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "attention backward launch");
}

template <typename T>
int bwd_dispatch_d(const BwdParams& bp, int D, cudaStream_t s) {
  if (D == 32) return bwd_launch_t<T, 32>(bp, s);
  if (D == 64) return bwd_launch_t<T, 64>(bp, s);
  return bwd_launch_t<T, 128>(bp, s);
}

}  // namespace
}  // namespace mlxp

using namespace mlxp;

extern "C" {

int mlxp_version(void) { return 100; }

const char* mlxp_last_error(void) { return t_last_error.c_str(); }

int mlxp_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int dtype,
                  int64_t B, int64_t H, int64_t Sq, int64_t Skv, int64_t D,
                  const int64_t q_strides[4], const int64_t k_strides[4],
                  const int64_t v_strides[4], const int64_t o_strides[4], float scale,
                  int causal, int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                  int64_t kv_pos_offset, int64_t kv_splits, void* workspace, size_t ws_bytes,
                  void* cuda_stream) {
  Problem pr{dtype, B, H, Sq, Skv, D, causal ? 1 : 0, window_left, window_right, q_pos_offset,
             kv_pos_offset};
  return attn_fwd_impl(q, k, v, o, lse, pr, q_strides, k_strides, v_strides, o_strides, scale,
                       kv_splits, workspace, ws_bytes, kOutNormal,
                       static_cast<cudaStream_t>(cuda_stream));
}

int mlxp_attn_fwd_gqa(const void* q, const void* k, const void* v, void* o, float* lse,
                      int dtype, int64_t B, int64_t H, int64_t H_kv, int64_t Sq, int64_t Skv,
                      int64_t D, const int64_t q_strides[4], const int64_t k_strides[4],
                      const int64_t v_strides[4], const int64_t o_strides[4], float scale,
                      int causal, int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                      int64_t kv_pos_offset, int64_t kv_splits, void* workspace, size_t ws_bytes,
                      void* cuda_stream) {
  Problem pr{dtype, B, H, Sq, Skv, D, causal ? 1 : 0, window_left, window_right, q_pos_offset,
             kv_pos_offset, H_kv};
  if (H_kv < 1) return fail(MLXP_ERR_INVALID, "num_kv_heads must be >= 1");
  return attn_fwd_impl(q, k, v, o, lse, pr, q_strides, k_strides, v_strides, o_strides, scale,
                       kv_splits, workspace, ws_bytes, kOutNormal,
                       static_cast<cudaStream_t>(cuda_stream));
}

size_t mlxp_attn_workspace_size(int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Skv,
                                int64_t D, int causal, int64_t window_left,
                                int64_t window_right, int64_t q_pos_offset,
                                int64_t kv_pos_offset, int64_t kv_splits) {
  Problem pr{dtype, B, H, Sq, Skv, D, causal ? 1 : 0, window_left, window_right, q_pos_offset,
             kv_pos_offset};
  if (validate(pr) != MLXP_OK || Sq == 0 || Skv == 0) return 0;
  const bool fp32 = dtype == MLXP_DTYPE_FP32;
  int splits = 1;
  if (kv_splits == 0) {
    int sms = 148;
    if (device_info(nullptr, &sms) != MLXP_OK) sms = 148;
    splits = fp32 ? choose_splits_f32(pr, sms) : choose_splits(pr, sms);
  } else if (kv_splits > 1) {
    splits = (int)std::min<int64_t>(kv_splits, (Skv + (fp32 ? 31 : kBN - 1)) / (fp32 ? 32 : kBN));
  }
  return split_workspace(pr, splits);
}

// Split-KV attention whose scratch (the per-split fp32 partial outputs and LSEs and the
// per-query-tile counters) lives in the library's static device array instead of a
// caller-provided workspace; see mlxp_attn.h.  Only the counters must start at zero, and the
// split path clears them on the call's stream before the kernel; every partial the kernel
// merges was written by the same launch, so the contents left by an earlier call are never
// read.
int mlxp_attn_fwd_split_noalloc(const void* q, const void* k, const void* v, void* o,
                                float* lse, int dtype, int64_t B, int64_t H, int64_t Sq,
                                int64_t Skv, int64_t D, const int64_t q_strides[4],
                                const int64_t k_strides[4], const int64_t v_strides[4],
                                const int64_t o_strides[4], float scale, int causal,
                                int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                                int64_t kv_pos_offset, int64_t kv_splits, void* cuda_stream) {
  Problem pr{dtype, B, H, Sq, Skv, D, causal ? 1 : 0, window_left, window_right, q_pos_offset,
             kv_pos_offset};
  if (int rc = validate(pr)) return rc;
  if (dtype == MLXP_DTYPE_FP32)
    return fail(MLXP_ERR_UNSUPPORTED,
                "mlxp_attn_fwd_split_noalloc runs the bf16/fp16 split-KV kernel");
  if (kv_splits < 2)
    return fail(MLXP_ERR_INVALID, "mlxp_attn_fwd_split_noalloc needs kv_splits >= 2, got %lld",
                (long long)kv_splits);
  const int splits = (int)std::min<int64_t>(kv_splits, std::max<int64_t>(1, (Skv + kBN - 1) / kBN));
  const size_t need = split_workspace(pr, splits);
  if (need > kNoAllocScratchBytes)
    return fail(MLXP_ERR_WORKSPACE,
                "mlxp_attn_fwd_split_noalloc: %d key splits of B*H*Sq = %lld rows x head_dim "
                "%lld need %zu bytes of scratch; the static scratch holds %zu bytes (use fewer "
                "splits, a smaller batch, or mlxp_attn_fwd with a workspace)",
                splits, (long long)(B * H * Sq), (long long)D, need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  return attn_fwd_impl(q, k, v, o, lse, pr, q_strides, k_strides, v_strides, o_strides, scale,
                       splits, scratch, kNoAllocScratchBytes, kOutNormal,
                       static_cast<cudaStream_t>(cuda_stream));
}

int mlxp_attn_fwd_partial(const void* q, const void* k, const void* v, float* o_part,
                          float* lse_part, int dtype, int64_t B, int64_t H, int64_t Sq,
                          int64_t Skv, int64_t D, const int64_t q_strides[4],
                          const int64_t k_strides[4], const int64_t v_strides[4],
                          const int64_t o_strides[4], float scale, int causal,
                          int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                          int64_t kv_pos_offset, void* cuda_stream) {
  if (dtype == MLXP_DTYPE_FP32)
    return fail(MLXP_ERR_UNSUPPORTED, "mlxp_attn_fwd_partial takes bf16/fp16 inputs");
  Problem pr{dtype, B, H, Sq, Skv, D, causal ? 1 : 0, window_left, window_right, q_pos_offset,
             kv_pos_offset};
  return attn_fwd_impl(q, k, v, o_part, lse_part, pr, q_strides, k_strides, v_strides,
                       o_strides, scale, 1, nullptr, 0, kOutPartial,
                       static_cast<cudaStream_t>(cuda_stream));
}

int mlxp_attn_fwd_masked(const void* q, const void* k, const void* v, void* o, float* lse,
                         int dtype, int64_t B, int64_t H, int64_t H_kv, int64_t Sq, int64_t Skv,
                         int64_t D, const int64_t q_strides[4], const int64_t k_strides[4],
                         const int64_t v_strides[4], const int64_t o_strides[4],
                         const float* mask, const int64_t mask_strides[4], float scale,
                         int causal, int64_t window_left, int64_t window_right,
                         int64_t q_pos_offset, int64_t kv_pos_offset, int64_t kv_splits,
                         void* workspace, size_t ws_bytes, void* cuda_stream) {
  Problem pr{dtype, B, H, Sq, Skv, D, causal ? 1 : 0, window_left, window_right, q_pos_offset,
             kv_pos_offset, H_kv};
  if (H_kv < 1) return fail(MLXP_ERR_INVALID, "num_kv_heads must be >= 1");
  if (mask == nullptr && Sq > 0 && Skv > 0) return fail(MLXP_ERR_INVALID, "mask is null");
  return attn_fwd_impl(q, k, v, o, lse, pr, q_strides, k_strides, v_strides, o_strides, scale,
                       kv_splits, workspace, ws_bytes, kOutNormal,
                       static_cast<cudaStream_t>(cuda_stream), nullptr, mask, mask_strides);
}

int mlxp_attn_fwd_accumulate(const void* q, const void* k, const void* v, float* o_acc,
                             float* lse_acc, int dtype, int64_t B, int64_t H, int64_t Sq,
                             int64_t Skv, int64_t D, const int64_t q_strides[4],
                             const int64_t k_strides[4], const int64_t v_strides[4],
                             const int64_t acc_strides[4], float scale, int causal,
                             int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                             int64_t kv_pos_offset, void* cuda_stream) {
  Problem pr{dtype, B, H, Sq, Skv, D, causal ? 1 : 0, window_left, window_right, q_pos_offset,
             kv_pos_offset};
  return attn_fwd_impl(q, k, v, o_acc, lse_acc, pr, q_strides, k_strides, v_strides,
                       acc_strides, scale, 1, nullptr, 0, kOutAccumulate,
                       static_cast<cudaStream_t>(cuda_stream));
}

size_t mlxp_rope_attn_workspace_size(int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Skv,
                                     int64_t D, int causal, int64_t window_left,
                                     int64_t window_right, int64_t q_pos_offset,
                                     int64_t kv_pos_offset, int64_t kv_splits) {
  Problem pr{dtype, B, H, Sq, Skv, D, causal ? 1 : 0, window_left, window_right, q_pos_offset,
             kv_pos_offset};
  if (validate(pr) != MLXP_OK || dtype == MLXP_DTYPE_FP32 || Sq == 0 || Skv == 0) return 0;
  return rope_layout(pr).total() +
         mlxp_attn_workspace_size(dtype, B, H, Sq, Skv, D, causal, window_left, window_right,
                                  q_pos_offset, kv_pos_offset, kv_splits);
}

int mlxp_rope_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                       int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Skv, int64_t D,
                       const int64_t q_strides[4], const int64_t k_strides[4],
                       const int64_t v_strides[4], const int64_t o_strides[4],
                       const float* cos_cache, const float* sin_cache, int64_t n_pos,
                       int64_t q_rope_offset, int64_t k_rope_offset, float scale, int causal,
                       int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                       int64_t kv_pos_offset, int64_t kv_splits, void* workspace,
                       size_t ws_bytes, void* cuda_stream) {
  Problem pr{dtype, B, H, Sq, Skv, D, causal ? 1 : 0, window_left, window_right, q_pos_offset,
             kv_pos_offset};
  if (dtype == MLXP_DTYPE_FP32)
    return fail(MLXP_ERR_UNSUPPORTED, "RoPE inside the attention launch takes bf16/fp16 inputs");
  const RopeArgs ra{cos_cache, sin_cache, n_pos, q_rope_offset, k_rope_offset};
  return attn_fwd_impl(q, k, v, o, lse, pr, q_strides, k_strides, v_strides, o_strides, scale,
                       kv_splits, workspace, ws_bytes, kOutNormal,
                       static_cast<cudaStream_t>(cuda_stream), &ra);
}

int mlxp_lse_merge(const float* o_parts, const float* lse_parts, int64_t n_parts, void* o,
                   float* lse_out, int dtype, int64_t B, int64_t H, int64_t S, int64_t D,
                   const int64_t o_strides[4], void* cuda_stream) {
  if (!o_parts || !lse_parts || n_parts < 1 || B < 1 || H < 1 || S < 0 || D < 1)
    return fail(MLXP_ERR_INVALID, "invalid lse_merge arguments");
  if (dtype < 0 || dtype > 2) return fail(MLXP_ERR_INVALID, "unknown dtype %d", dtype);
  if (!o_strides || o == nullptr || o_strides[3] != 1)
    return fail(MLXP_ERR_INVALID, "o must be non-null with unit head_dim stride");
  Problem pr{dtype, B, H, S, 0, D, 0, -1, -1, 0, 0};
  return merge_dispatch(o_parts, lse_parts, (int)n_parts, o, lse_out, pr, o_strides,
                        static_cast<cudaStream_t>(cuda_stream));
}

int mlxp_lse_merge_accumulate(float* o_acc, float* lse_acc, const float* o_new,
                              const float* lse_new, int64_t B, int64_t H, int64_t S, int64_t D,
                              void* cuda_stream) {
  if (!o_acc || !lse_acc || !o_new || !lse_new || B < 1 || H < 1 || S < 0 || D < 1)
    return fail(MLXP_ERR_INVALID, "invalid lse_merge_accumulate arguments");
  const long long rows = B * H * S;
  if (rows == 0) return MLXP_OK;
  lse_merge_acc_kernel<<<(unsigned)((rows + 7) / 8), 256, 0,
                         static_cast<cudaStream_t>(cuda_stream)>>>(o_acc, lse_acc, o_new,
                                                                   lse_new, rows, (int)D);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "lse_merge_accumulate launch");
}

int mlxp_cast_output(const float* o_acc, void* o, int dtype, int64_t B, int64_t H, int64_t S,
                     int64_t D, const int64_t o_strides[4], void* cuda_stream) {
  if (!o_acc || !o || !o_strides || o_strides[3] != 1 || B < 1 || H < 1 || S < 0 || D < 1)
    return fail(MLXP_ERR_INVALID, "invalid cast_output arguments");
  const long long rows = B * H * S;
  if (rows == 0) return MLXP_OK;
  cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
  const unsigned grid = (unsigned)((rows + 7) / 8);
  if (dtype == MLXP_DTYPE_FP32)
    cast_rows_kernel<float><<<grid, 256, 0, s>>>(o_acc, (float*)o, rows, (int)H, (int)S, (int)D, o_strides[0], o_strides[1], o_strides[2]);
  else if (dtype == MLXP_DTYPE_BF16)
    cast_rows_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(o_acc, (__nv_bfloat16*)o, rows, (int)H, (int)S, (int)D, o_strides[0], o_strides[1], o_strides[2]);
  else if (dtype == MLXP_DTYPE_FP16)
    cast_rows_kernel<__half><<<grid, 256, 0, s>>>(o_acc, (__half*)o, rows, (int)H, (int)S, (int)D, o_strides[0], o_strides[1], o_strides[2]);
  else
    return fail(MLXP_ERR_INVALID, "unknown dtype %d", dtype);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "cast_output launch");
}

int mlxp_rope(const void* x, void* y, int dtype, int64_t B, int64_t H, int64_t S, int64_t D,
              const int64_t x_strides[4], const int64_t y_strides[4], const float* cos_cache,
              const float* sin_cache, int64_t n_pos, int64_t pos_offset, void* cuda_stream) {
  if (B < 0 || H < 0 || S < 0) return fail(MLXP_ERR_INVALID, "invalid rope shape");
  RopeParams rp{};
  rp.n = 1;
  rp.cosc = cos_cache;
  rp.sinc = sin_cache;
  rp.n_pos = n_pos;
  rp.t[0] = RopeTensor{x, y, {0, 0, 0}, {0, 0, 0}, (int)H, (int)S, (long long)B * H * S,
                       (long long)pos_offset};
  const int64_t* xs[2] = {x_strides, nullptr};
  const int64_t* ys[2] = {y_strides, nullptr};
  return rope_launch(dtype, D, rp, xs, ys, static_cast<cudaStream_t>(cuda_stream));
}

int mlxp_rope_qk(const void* q, const void* k, void* q_out, void* k_out, int dtype, int64_t B,
                 int64_t Hq, int64_t Hk, int64_t Sq, int64_t Sk, int64_t D,
                 const int64_t q_strides[4], const int64_t k_strides[4],
                 const int64_t qo_strides[4], const int64_t ko_strides[4],
                 const float* cos_cache, const float* sin_cache, int64_t n_pos,
                 int64_t q_pos_offset, int64_t k_pos_offset, void* cuda_stream) {
  if (B < 0 || Hq < 0 || Hk < 0 || Sq < 0 || Sk < 0) return fail(MLXP_ERR_INVALID, "invalid rope shape");
  RopeParams rp{};
  rp.n = 2;
  rp.cosc = cos_cache;
  rp.sinc = sin_cache;
  rp.n_pos = n_pos;
  rp.t[0] = RopeTensor{q, q_out, {0, 0, 0}, {0, 0, 0}, (int)Hq, (int)Sq, (long long)B * Hq * Sq,
                       (long long)q_pos_offset};
  rp.t[1] = RopeTensor{k, k_out, {0, 0, 0}, {0, 0, 0}, (int)Hk, (int)Sk, (long long)B * Hk * Sk,
                       (long long)k_pos_offset};
  const int64_t* xs[2] = {q_strides, k_strides};
  const int64_t* ys[2] = {qo_strides, ko_strides};
  return rope_launch(dtype, D, rp, xs, ys, static_cast<cudaStream_t>(cuda_stream));
}

size_t mlxp_paged_attn_workspace_size(int dtype, int64_t B, int64_t H, int64_t Sq, int64_t D,
                                      int64_t kv_heads, int64_t num_blocks, int64_t block_size,
                                      int64_t max_blocks, int64_t kv_splits) {
  PagedProblem pp{dtype, B, H, Sq, D, kv_heads, num_blocks, block_size, max_blocks};
  if (paged_validate(pp) != MLXP_OK) return 0;
  int sms = 148;
  if (kv_splits == 0 && device_info(nullptr, &sms) != MLXP_OK) sms = 148;
  return paged_workspace(pp, paged_grid(pp, kv_splits, sms));
}

int mlxp_paged_attn(const void* q, const void* k_pool, const void* v_pool,
                    const int32_t* block_tables, const int32_t* context_lens,
                    const float* alibi_slopes, void* o, int dtype, int64_t B, int64_t H,
                    int64_t Sq, int64_t D, int64_t kv_heads, int64_t num_blocks,
                    int64_t block_size, int64_t max_blocks, const int64_t q_strides[4],
                    const int64_t pool_strides[4], int64_t bt_stride,
                    const int64_t o_strides[4], float scale, int causal, int64_t kv_splits,
                    void* workspace, size_t ws_bytes, void* cuda_stream) {
  PagedProblem pp{dtype, B, H, Sq, D, kv_heads, num_blocks, block_size, max_blocks};
  if (int rc = paged_validate(pp)) return rc;
  if (!(scale > 0.f) || !std::isfinite(scale))
    return fail(MLXP_ERR_INVALID, "scale must be positive and finite");
  if (kv_splits < 0) return fail(MLXP_ERR_INVALID, "kv_splits must be >= 0");
  if (B == 0 || Sq == 0) return MLXP_OK;
  if (!q || !o || !context_lens || !q_strides || !o_strides || !pool_strides)
    return fail(MLXP_ERR_INVALID, "q, o, context_lens and the stride arrays must be non-null");
  if (max_blocks > 0 && (!k_pool || !v_pool || !block_tables))
    return fail(MLXP_ERR_INVALID, "k_pool, v_pool and block_tables must be non-null");
  if (max_blocks > 0 && B > 1 && bt_stride < max_blocks)
    return fail(MLXP_ERR_INVALID, "block-table row stride (%lld) is below max_blocks (%lld)",
                (long long)bt_stride, (long long)max_blocks);
  if (q_strides[3] != 1 || o_strides[3] != 1 || pool_strides[3] != 1)
    return fail(MLXP_ERR_INVALID, "head_dim stride must be 1");
  // every lane reads 4 consecutive elements as one vector
  const int es = dtype == MLXP_DTYPE_FP32 ? 4 : 2;
  const uintptr_t qa = 4u * es;
  const void* ptrs[3] = {q, k_pool, v_pool};
  for (const void* ptr : ptrs)
    if (ptr && reinterpret_cast<uintptr_t>(ptr) % qa)
      return fail(MLXP_ERR_INVALID, "q, k_pool and v_pool must be %d-byte aligned", (int)qa);
  for (int d = 0; d < 3; ++d)
    if (q_strides[d] % 4 || pool_strides[d] % 4 || q_strides[d] < 0 || pool_strides[d] < 0)
      return fail(MLXP_ERR_INVALID, "q and pool strides must be non-negative multiples of 4 elements");
  int sms = 148;
  if (int rc = device_info(nullptr, &sms)) return rc;
  const long long grid = paged_grid(pp, kv_splits, sms);
  const size_t need = paged_workspace(pp, grid);
  if (need > 0 && (workspace == nullptr || ws_bytes < need))
    return fail(MLXP_ERR_WORKSPACE, "paged attention needs %zu bytes of workspace, got %zu", need,
                ws_bytes);
  if (need > 0 && reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(MLXP_ERR_INVALID, "workspace must be 256-byte aligned");
  PagedParams p{};
  p.q = q;
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.block_tables = block_tables;
  p.context_lens = context_lens;
  p.alibi = alibi_slopes;
  p.o = o;
  p.q_sb = q_strides[0];
  p.q_sh = q_strides[1];
  p.q_ss = q_strides[2];
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.o_ss = o_strides[2];
  p.p_sb = pool_strides[0];
  p.p_st = pool_strides[1];
  p.p_sh = pool_strides[2];
  p.bt_stride = bt_stride;
  p.B = (int)B;
  p.H = (int)H;
  p.Sq = (int)Sq;
  p.D = (int)D;
  p.kv_group = (int)(H / kv_heads);
  p.num_blocks = (int)num_blocks;
  p.block_size = (int)block_size;
  p.max_blocks = (int)max_blocks;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
  if (grid == 0) {  // no block-table slots: every row has no admissible key
    Problem pr{dtype, B, H, Sq, 0, D, 0, -1, -1, 0, 0};
    return fill_empty(pr, o, nullptr, o_strides, s);
  }
  if (grid > INT32_MAX) return fail(MLXP_ERR_INVALID, "paged shape too large");
  p.grid = (int)grid;
  p.total = B * Sq * H * max_blocks;
  if (need > 0) {
    const long long pairs = B * Sq * H;
    p.max_parts = (int)paged_max_parts(pp, grid);
    const size_t rows = (size_t)pairs * p.max_parts;
    char* w = static_cast<char*>(workspace);
    const size_t o_bytes = (rows * D * 4 + 255) / 256 * 256;
    const size_t l_bytes = (rows * 4 + 255) / 256 * 256;
    p.o_part = reinterpret_cast<float*>(w);
    p.lse_part = reinterpret_cast<float*>(w + o_bytes);
    p.counters = reinterpret_cast<unsigned*>(w + o_bytes + l_bytes);
    cudaError_t e = cudaMemsetAsync(p.counters, 0, (size_t)pairs * 4, s);
    if (e != cudaSuccess) return cuda_fail(e, "paged attention counter reset");
  }
  const int LPR = (int)(D / 4);
  if (paged_tma_shape(pp)) {
    CUtensorMap mk, mv;
    if (make_pool_tmap(k_pool, dtype, pp, pool_strides, &mk) &&
        make_pool_tmap(v_pool, dtype, pp, pool_strides, &mv)) {
      int* status = nullptr;
      if (int rc = device_info(&status, nullptr)) return rc;
      p.status = status;
      p.timeout_ns = g_timeout_ns.load();
      if (dtype == MLXP_DTYPE_BF16)
        return paged_tma_launch_t<__nv_bfloat16>(mk, mv, p, LPR, (unsigned)grid, s);
      return paged_tma_launch_t<__half>(mk, mv, p, LPR, (unsigned)grid, s);
    }
  }
  if (dtype == MLXP_DTYPE_BF16) return paged_launch_t<__nv_bfloat16>(p, LPR, (unsigned)grid, s);
  if (dtype == MLXP_DTYPE_FP16) return paged_launch_t<__half>(p, LPR, (unsigned)grid, s);
  return paged_launch_t<float>(p, LPR, (unsigned)grid, s);
}

size_t mlxp_attn_bwd_workspace_size(int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Skv,
                                    int64_t D) {
  Problem pr{dtype, B, H, Sq, Skv, D, 0, -1, -1, 0, 0};
  if (B < 0 || H <= 0 || Sq < 0 || Skv < 0) return 0;
  return bwd_workspace(pr);
}

int mlxp_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                  const float* lse, void* dq, void* dk, void* dv, int dtype, int64_t B,
                  int64_t H, int64_t H_kv, int64_t Sq, int64_t Skv, int64_t D,
                  const int64_t q_strides[4], const int64_t k_strides[4],
                  const int64_t v_strides[4], const int64_t o_strides[4],
                  const int64_t do_strides[4], const int64_t dq_strides[4],
                  const int64_t dk_strides[4], const int64_t dv_strides[4], float scale,
                  int causal, int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                  int64_t kv_pos_offset, void* workspace, size_t ws_bytes, void* cuda_stream) {
  if (B < 0 || H <= 0 || H_kv <= 0 || Sq < 0 || Skv < 0)
    return fail(MLXP_ERR_INVALID, "invalid backward shape B=%lld H=%lld H_kv=%lld Sq=%lld Skv=%lld",
                (long long)B, (long long)H, (long long)H_kv, (long long)Sq, (long long)Skv);
  if (H % H_kv) return fail(MLXP_ERR_INVALID, "num_heads must be divisible by num_kv_heads");
  if (dtype < 0 || dtype > 2) return fail(MLXP_ERR_INVALID, "unknown dtype %d", dtype);
  if (D != 32 && D != 64 && D != 128)
    return fail(MLXP_ERR_UNSUPPORTED, "attention backward supports head_dim 32, 64 and 128, got %lld",
                (long long)D);
  if (!(scale > 0.f) || !std::isfinite(scale))
    return fail(MLXP_ERR_INVALID, "scale must be positive and finite");
  if (window_left < -1 || window_right < -1)
    return fail(MLXP_ERR_INVALID, "window must be >= 0 or -1");
  if (B * H * std::max(Sq, Skv) > INT32_MAX || Sq > INT32_MAX / 2 || Skv > INT32_MAX / 2)
    return fail(MLXP_ERR_INVALID, "shape too large");
  if (B == 0 || Sq == 0) return MLXP_OK;
  const int64_t* st[8] = {q_strides, k_strides, v_strides, o_strides, do_strides, dq_strides,
                          dk_strides, dv_strides};
  for (const int64_t* a : st) {
    if (!a) return fail(MLXP_ERR_INVALID, "stride arrays must be non-null");
    if (a[3] != 1) return fail(MLXP_ERR_INVALID, "head_dim stride must be 1");
  }
  if (!q || !o || !dout || !lse || !dq || (Skv > 0 && (!k || !v || !dk || !dv)))
    return fail(MLXP_ERR_INVALID, "tensor pointers must be non-null");
  Problem pr{dtype, B, H, Sq, Skv, D, causal ? 1 : 0, window_left, window_right, q_pos_offset,
             kv_pos_offset, H_kv};
  const size_t need = bwd_workspace(pr);
  if (workspace == nullptr || ws_bytes < need)
    return fail(MLXP_ERR_WORKSPACE, "attention backward needs %zu bytes of workspace, got %zu",
                need, ws_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(MLXP_ERR_INVALID, "workspace must be 256-byte aligned");
  BwdParams bp{};
  bp.B = (int)B;
  bp.H = (int)H;
  bp.Sq = (int)Sq;
  bp.Skv = (int)Skv;
  bp.kv_group = (int)(H / H_kv);
  bp.q = q;
  bp.k = k;
  bp.v = v;
  bp.o = o;
  bp.dout = dout;
  bp.lse = lse;
  bp.delta = static_cast<float*>(workspace);
  bp.dq = dq;
  bp.dk = dk;
  bp.dv = dv;
  long long* dst[8][3] = {{&bp.q_sb, &bp.q_sh, &bp.q_ss},    {&bp.k_sb, &bp.k_sh, &bp.k_ss},
                          {&bp.v_sb, &bp.v_sh, &bp.v_ss},    {&bp.o_sb, &bp.o_sh, &bp.o_ss},
                          {&bp.do_sb, &bp.do_sh, &bp.do_ss}, {&bp.dq_sb, &bp.dq_sh, &bp.dq_ss},
                          {&bp.dk_sb, &bp.dk_sh, &bp.dk_ss}, {&bp.dv_sb, &bp.dv_sh, &bp.dv_ss}};
  for (int t = 0; t < 8; ++t)
    for (int d = 0; d < 3; ++d) *dst[t][d] = st[t][d];
  bp.scale = scale;
  bp.scale_log2 = scale * 1.4426950408889634f;
  bp.mask = mask_of(pr);
  cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
  if (bwd_tc_shape(pr) && !g_bwd_force_cuda_cores.load()) {
    const int rc = bwd_tc_launch(bp, pr, st, workspace, s);
    if (rc != MLXP_ERR_UNSUPPORTED) return rc;
  }
  if (dtype == MLXP_DTYPE_BF16) return bwd_dispatch_d<__nv_bfloat16>(bp, (int)D, s);
  if (dtype == MLXP_DTYPE_FP16) return bwd_dispatch_d<__half>(bp, (int)D, s);
  return bwd_dispatch_d<float>(bp, (int)D, s);
}

int mlxp_device_status(int* status_out, int reset) {
  int* status = nullptr;
  if (int rc = device_info(&status, nullptr)) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpy(&v, status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read device status");
  if (status_out) *status_out = v;
  if (reset) {
    const int zero = 0;
    e = cudaMemcpy(status, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "reset device status");
  }
  return MLXP_OK;
}

int mlxp_set_backward_path(int cuda_cores_only) {
  g_bwd_force_cuda_cores.store(cuda_cores_only ? 1 : 0);
  return MLXP_OK;
}


int mlxp_set_wait_timeout_ns(uint64_t ns) {
  if (ns == 0) return fail(MLXP_ERR_INVALID, "timeout must be positive");
  g_timeout_ns.store(ns);
  return MLXP_OK;
}

#if MLXP_TRACE
// Trace builds only: copies the cycle stamps of CTA 0 (see attn_fwd_sm100.cuh) to dst.
int mlxp_trace_read(long long* dst, int n) {
  const int cap = 4 * 64 * 8;
  cudaError_t e = cudaMemcpyFromSymbol(dst, g_mlxp_trace, sizeof(long long) * (n < cap ? n : cap));
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "trace read");
}
// Trace builds only: the split model's launch estimate (key-tile steps) for a shape.
double mlxp_model_steps(int64_t B, int64_t H, int64_t Sq, int64_t Skv, int64_t D, int causal,
                        int64_t wl, int64_t wr, int64_t qoff, int splits, int sms) {
  Problem pr{MLXP_DTYPE_BF16, B, H, Sq, Skv, D, causal, wl, wr, qoff, 0};
  return model_launch_steps(pr, splits, sms);
}
int mlxp_cta_life_read(long long* dst, int n) {
  const int cap = 1024 * 3;
  cudaError_t e = cudaMemcpyFromSymbol(dst, g_mlxp_cta_life, sizeof(long long) * (n < cap ? n : cap));
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "cta life read");
}
int mlxp_rot_trace_read(long long* dst, int n) {
  const int cap = 2048 * 3;
  cudaError_t e = cudaMemcpyFromSymbol(dst, g_mlxp_rot_trace, sizeof(long long) * (n < cap ? n : cap));
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "rot trace read");
}
int mlxp_cta_trace_read(long long* dst, int n) {
  const int cap = 8192 * 4;
  cudaError_t e = cudaMemcpyFromSymbol(dst, g_mlxp_cta_trace, sizeof(long long) * (n < cap ? n : cap));
  return e == cudaSuccess ? MLXP_OK : cuda_fail(e, "cta trace read");
}
#endif

int mlxp_selftest_wait_timeout(uint64_t timeout_ns, void* cuda_stream) {
  int* status = nullptr;
  if (int rc = device_info(&status, nullptr)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
  const int zero = 0;
  cudaError_t e0 = cudaMemcpy(status, &zero, sizeof(int), cudaMemcpyHostToDevice);
  if (e0 != cudaSuccess) return cuda_fail(e0, "selftest reset status");
  // The self-test reports through the status word, the wait's own error channel.
  wait_selftest_kernel<<<1, 64, 0, s>>>(status, (unsigned long long)timeout_ns);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "selftest sync");
  int v = 0;
  e = cudaMemcpy(&v, status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "selftest read status");
  if ((v & 0xff) == kDevTimeout) return fail(MLXP_ERR_TIMEOUT, "bounded wait gave up at site %d", v >> 8);
  return MLXP_OK;
}

}  // extern "C"

// The NCCL ring (mlxp_ring_*): drives the entry points above.
#include "ring_nccl.cuh"
