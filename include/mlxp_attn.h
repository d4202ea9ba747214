/*
 * mlxp_attn.h — C ABI of libmlxp_attn.so, the B200 (sm_100a) attention forward library.
 *
 * This is the drop-in boundary that replaces the reference's kernel dispatch for the
 * mlx_primitives.attention forward path.  Every pointer is a device pointer unless stated
 * otherwise, every stride is in ELEMENTS and given in (batch, head, seq, dim) order, so the
 * BSHD and BHSD layouts are both just stride vectors (no transpose kernel anywhere).  The
 * dim stride must be 1.  Calls are asynchronous on the given CUDA stream (NULL = legacy
 * default stream) and never allocate device memory: scratch space is passed in by the caller
 * (see mlxp_attn_workspace_size).  Every function returns an mlxp_status; the message of the
 * last failure on the calling thread is available from mlxp_last_error().
 *
 * Reference interfaces replaced (paths inside zakkeown/mlx-primitives):
 *   mlx_primitives/attention/flash.py:178-183, 220-235   mx.fast.scaled_dot_product_attention calls
 *   mlx_primitives/attention/flash.py:319-476            flash_attention Metal kernel + launch
 *   mlx_primitives/attention/sliding_window.py:46-133,316-360   sliding-window Metal kernel + launch
 *   mlx_primitives/attention/chunked.py:258-407          chunked cross-attention Metal kernel + launch
 *   mlx_primitives/attention/_online_softmax.py:42-106   online_softmax_merge (LSE merge)
 *   mlx_primitives/kernels/_registry.py:122-156          get_kernel (kernel cache)
 */
#ifndef MLXP_ATTN_H
#define MLXP_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference raises ValueError for bad shapes/dtypes/layouts
 * (flash.py:123-169) and RuntimeError for kernel failures (flash.py:236-251); the Python shim
 * maps MLXP_ERR_INVALID to ValueError and everything else to RuntimeError. */
typedef enum mlxp_status {
  MLXP_OK = 0,
  MLXP_ERR_INVALID = 1,     /* bad argument: shape, stride, alignment, null pointer */
  MLXP_ERR_UNSUPPORTED = 2, /* valid but not built: head_dim / dtype combination      */
  MLXP_ERR_CUDA = 3,        /* a CUDA runtime or driver call failed                    */
  MLXP_ERR_NCCL = 4,        /* an NCCL call failed or NCCL could not be loaded         */
  MLXP_ERR_TIMEOUT = 5,     /* a bounded device-side wait ran out (see mlxp_device_status) */
  MLXP_ERR_WORKSPACE = 6    /* workspace missing or smaller than mlxp_attn_workspace_size */
} mlxp_status;

/* Element types. */
typedef enum mlxp_dtype {
  MLXP_DTYPE_FP32 = 0,
  MLXP_DTYPE_BF16 = 1,
  MLXP_DTYPE_FP16 = 2
} mlxp_dtype;

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int mlxp_version(void);

/* Message of the last failure on the calling thread ("" if none).  Thread-local. */
const char* mlxp_last_error(void);

/*
 * Attention forward:  O = softmax(scale * Q K^T + mask) V, per (batch, head).
 *
 * Replaces the SDPA call / Metal kernel launch of flash_attention (flash.py:178-183, 220-235,
 * 463-474), sliding_window_attention (sliding_window.py:217, 351-358) and
 * chunked_cross_attention (chunked.py:394-405).
 *
 * Shapes: q [B,H,Sq,D], k/v [B,H,Skv,D], o [B,H,Sq,D] (logical, in the given strides).
 * Masking uses absolute positions qpos = i + q_pos_offset, kpos = j + kv_pos_offset:
 *   causal != 0          requires kpos <= qpos
 *   window_left  >= 0    requires qpos - kpos <= window_left   (-1 = unbounded)
 *   window_right >= 0    requires kpos - qpos <= window_right  (-1 = unbounded)
 * The reference's conventions map onto these as:
 *   flash_attention causal (bottom-right aligned, utils/masking.py:14-66):  q_pos_offset = Skv - Sq
 *   sliding window |i-j| <= W (+ causal)  (sliding_window.py:136-161):     window_left = W [, window_right = W]
 *   chunked causal, top-left absolute positions (_online_softmax.py:149-161): offsets 0
 * A query row with no admissible key yields O = 0 and LSE = -inf.
 *
 * lse (nullable): fp32 [B,H,Sq] contiguous, natural-log sum-exp of the scaled, masked scores.
 * dtype: element type of q, k, v and o.  BF16/FP16 run the tcgen05 tensor-core kernel
 * (head_dim 64 or 128); FP32 runs the CUDA-core kernel (head_dim 32, 64 or 128).
 * kv_splits: 1 = no split, 0 = automatic, >1 = split the key range into that many parts that
 * run as separate CTAs; the part that finishes a query block last merges the parts' results
 * (LSE weights) inside the same launch.  Needs workspace (mlxp_attn_workspace_size): the parts'
 * fp32 partials and per-block counters; the counters are cleared on the call's stream.
 */
int mlxp_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                  int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Skv, int64_t D,
                  const int64_t q_strides[4], const int64_t k_strides[4],
                  const int64_t v_strides[4], const int64_t o_strides[4],
                  float scale, int causal, int64_t window_left, int64_t window_right,
                  int64_t q_pos_offset, int64_t kv_pos_offset,
                  int64_t kv_splits, void* workspace, size_t ws_bytes, void* cuda_stream);

/*
 * Grouped-query / multi-query attention: as mlxp_attn_fwd, with H_kv K/V heads shared by the H
 * query heads (H % H_kv == 0; query head h reads K/V head h / (H / H_kv), the head repetition of
 * the reference's gqa_attention and mqa_attention).  k and v are [B][H_kv][Skv][D] through their
 * strides.  The workspace is the same as mlxp_attn_fwd's for the query shape.
 * Replaces: mlx_primitives/attention/grouped_query.py:195-261 (gqa_attention),
 *           mlx_primitives/attention/multi_query.py:161-225 (mqa_attention).
 */
int mlxp_attn_fwd_gqa(const void* q, const void* k, const void* v, void* o, float* lse,
                      int dtype, int64_t B, int64_t H, int64_t H_kv, int64_t Sq, int64_t Skv,
                      int64_t D, const int64_t q_strides[4], const int64_t k_strides[4],
                      const int64_t v_strides[4], const int64_t o_strides[4], float scale,
                      int causal, int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                      int64_t kv_pos_offset, int64_t kv_splits, void* workspace, size_t ws_bytes,
                      void* cuda_stream);

/*
 * Attention with an additive mask: as mlxp_attn_fwd_gqa, with
 *   scores = scale * Q K^T + mask[b][h][i][j]   (before causal / window masking and softmax)
 * the custom `mask` of the reference's gqa_attention and mqa_attention, added to the scores
 * after the causal mask (mlx_primitives/attention/grouped_query.py:253-254,
 * multi_query.py:218-219).  mask: fp32, element strides (batch, head, query row, key) in
 * mask_strides — 0 for broadcast dims, key stride 1, the others multiples of 4 with a 16-byte
 * aligned base; -inf entries exclude keys.  A row left with no admissible key gives O = 0,
 * LSE = -inf.  bf16/fp16 run a separate instantiation of the tensor-core kernel that adds the
 * mask row by row to the scores (the unmasked kernel is unchanged); fp32 the CUDA-core kernel.
 * The workspace is mlxp_attn_fwd's (mlxp_attn_workspace_size).
 */
int mlxp_attn_fwd_masked(const void* q, const void* k, const void* v, void* o, float* lse,
                         int dtype, int64_t B, int64_t H, int64_t H_kv, int64_t Sq, int64_t Skv,
                         int64_t D, const int64_t q_strides[4], const int64_t k_strides[4],
                         const int64_t v_strides[4], const int64_t o_strides[4],
                         const float* mask, const int64_t mask_strides[4], float scale,
                         int causal, int64_t window_left, int64_t window_right,
                         int64_t q_pos_offset, int64_t kv_pos_offset, int64_t kv_splits,
                         void* workspace, size_t ws_bytes, void* cuda_stream);

/*
 * Bytes of workspace mlxp_attn_fwd needs for these arguments (0 when no split is used).
 * kv_splits as for mlxp_attn_fwd (0 = the automatic choice mlxp_attn_fwd would make).
 * Replaces the reference's implicit MLX allocation of intermediate arrays (chunked.py:142-166).
 */
size_t mlxp_attn_workspace_size(int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Skv,
                                int64_t D, int causal, int64_t window_left,
                                int64_t window_right, int64_t q_pos_offset,
                                int64_t kv_pos_offset, int64_t kv_splits);

/*
 * Split-KV attention forward that allocates nothing.  No counterpart in the reference (MLX
 * allocates every intermediate itself); this entry point exists for callers that cannot call
 * cudaMalloc or hand out a workspace: code that is given only the input and output device
 * pointers by a host framework it plugs into, and latency-critical loops that must not take a
 * device allocation (cudaMalloc may synchronise the device and its caching allocators may
 * block on a lock).
 *
 * Same arguments and results as mlxp_attn_fwd with kv_splits >= 2 (bf16/fp16 only), except that
 * the per-split partial outputs and the per-query-tile counters live in a static device array
 * of 32 MiB inside the library (held by every GPU that loads the library until process exit)
 * instead of a workspace.  The split count is kv_splits clamped to the number of 128-key tiles,
 * ceil(Skv / 128); a key range of one tile therefore runs unsplit and leaves the array unused.
 * Sizes whose scratch needs more than 32 MiB (about splits * B*H*Sq rows * (head_dim + 1)
 * floats, see mlxp_attn_workspace_size) are rejected with MLXP_ERR_WORKSPACE and a message;
 * the caller can use fewer splits.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) and caches it for the life of the process; make that first
 * call before any stream capture, and do not keep using the library on a device after
 * cudaDeviceReset (the cached address may no longer be the array's).  Every call shares the
 * array and clears the counters it needs (cudaMemsetAsync on the call's stream) before its
 * kernel: calls that overlap on the GPU (other streams, other threads) race on the array and
 * must be serialised by the caller.
 */
int mlxp_attn_fwd_split_noalloc(const void* q, const void* k, const void* v, void* o,
                                float* lse, int dtype, int64_t B, int64_t H, int64_t Sq,
                                int64_t Skv, int64_t D, const int64_t q_strides[4],
                                const int64_t k_strides[4], const int64_t v_strides[4],
                                const int64_t o_strides[4], float scale, int causal,
                                int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                                int64_t kv_pos_offset, int64_t kv_splits, void* cuda_stream);

/*
 * Partial attention forward: as mlxp_attn_fwd, but writes the NORMALISED output in fp32
 * (o_part, [B,H,Sq,D] with o_strides) and the natural-log LSE (lse_part, [B,H,Sq]
 * contiguous, required).  This is the (O, m, l) triple of compute_chunk_attention
 * (_online_softmax.py:109-176) in LSE form, used by the ring pass and by callers that merge
 * several key ranges themselves.  bf16/fp16 inputs only; no split.
 */
int mlxp_attn_fwd_partial(const void* q, const void* k, const void* v, float* o_part,
                          float* lse_part, int dtype, int64_t B, int64_t H, int64_t Sq,
                          int64_t Skv, int64_t D, const int64_t q_strides[4],
                          const int64_t k_strides[4], const int64_t v_strides[4],
                          const int64_t o_strides[4], float scale, int causal,
                          int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                          int64_t kv_pos_offset, void* cuda_stream);

/*
 * Accumulating attention forward: as mlxp_attn_fwd_partial, but instead of writing this key
 * range's result it merges it into a running one — the per-key-range fold of the reference's
 * chunk loop (compute_chunk_attention + online_softmax_merge, _online_softmax.py:42-176), in
 * LSE form, done in the attention kernel's epilogue:
 *   (o_acc, lse_acc) <- merge((o_acc, lse_acc), (O, LSE) of q against this k/v range).
 * o_acc: fp32 [B,H,Sq,D] with acc_strides (normalised running output); lse_acc: fp32 [B,H,Sq]
 * contiguous, natural log, required.  Rows whose lse_acc is -inf take the new result alone
 * (their o_acc is not read, so it need not be initialised; it gets O = 0 when this range has
 * no admissible key for the row either); other rows this range gives no admissible key keep
 * their values.  Start with lse_acc = -inf and cast o_acc at the end (mlxp_cast_output).
 * bf16/fp16 inputs, head_dim 64 or 128; no split.  Used by the ring pass.
 */
int mlxp_attn_fwd_accumulate(const void* q, const void* k, const void* v, float* o_acc,
                             float* lse_acc, int dtype, int64_t B, int64_t H, int64_t Sq,
                             int64_t Skv, int64_t D, const int64_t q_strides[4],
                             const int64_t k_strides[4], const int64_t v_strides[4],
                             const int64_t acc_strides[4], float scale, int causal,
                             int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                             int64_t kv_pos_offset, void* cuda_stream);

/*
 * LSE merge of n_parts partial results (online_softmax_merge, _online_softmax.py:42-106, in
 * LSE form):  w_i = exp(lse_i - max_j lse_j);  O = sum_i w_i O_i / sum_i w_i;
 * lse = max_j lse_j + log(sum_i w_i).
 * o_parts: fp32 [n_parts,B,H,S,D] contiguous; lse_parts: fp32 [n_parts,B,H,S] contiguous.
 * o: output in dtype with o_strides; lse_out (nullable): fp32 [B,H,S] contiguous.
 */
int mlxp_lse_merge(const float* o_parts, const float* lse_parts, int64_t n_parts, void* o,
                   float* lse_out, int dtype, int64_t B, int64_t H, int64_t S, int64_t D,
                   const int64_t o_strides[4], void* cuda_stream);

/*
 * In-place running merge for the ring pass: (o_acc, lse_acc) <- merge((o_acc, lse_acc),
 * (o_new, lse_new)).  All fp32; o_acc/o_new [B,H,S,D] contiguous, lse [B,H,S] contiguous.
 * An accumulator row with lse_acc = -inf is simply replaced.
 */
int mlxp_lse_merge_accumulate(float* o_acc, float* lse_acc, const float* o_new,
                              const float* lse_new, int64_t B, int64_t H, int64_t S,
                              int64_t D, void* cuda_stream);

/*
 * Final conversion of a ring accumulator: o = o_acc cast to dtype (o_strides).
 */
int mlxp_cast_output(const float* o_acc, void* o, int dtype, int64_t B, int64_t H, int64_t S,
                     int64_t D, const int64_t o_strides[4], void* cuda_stream);

/*
 * Rotary position embedding, the half-split rotation of the reference's rope
 * (mlx_primitives/kernels/rope.py:451-496, fast_rope :350-381): with h = D/2 and the row's
 * position p = pos_offset + s,  y[:h] = x[:h]*cos[p] - x[h:]*sin[p],
 * y[h:] = x[:h]*sin[p] + x[h:]*cos[p].  cos_cache/sin_cache: fp32 [n_pos][D/2] contiguous
 * (precompute_rope_cache, rope.py:223-255); positions past n_pos are rejected.  x and y are
 * [B][H][S][D] through their strides (y may alias x); fp32/bf16/fp16, computed in fp32.
 */
int mlxp_rope(const void* x, void* y, int dtype, int64_t B, int64_t H, int64_t S, int64_t D,
              const int64_t x_strides[4], const int64_t y_strides[4], const float* cos_cache,
              const float* sin_cache, int64_t n_pos, int64_t pos_offset, void* cuda_stream);

/*
 * RoPE of Q and K in one launch (rope.py:384-448, fast_rope_qk), with their own head counts,
 * lengths and position offsets (grouped K/V heads, a KV cache longer than the queries).
 * The rotation step of fused_rope_attention (kernels/fused_rope_attention.py:939-985) where
 * mlxp_rope_attn_fwd does not apply (grouped K/V heads, head_dims other than 64 and 128),
 * followed by mlxp_attn_fwd on the rotated tensors.
 */
int mlxp_rope_qk(const void* q, const void* k, void* q_out, void* k_out, int dtype, int64_t B,
                 int64_t Hq, int64_t Hk, int64_t Sq, int64_t Sk, int64_t D,
                 const int64_t q_strides[4], const int64_t k_strides[4],
                 const int64_t qo_strides[4], const int64_t ko_strides[4],
                 const float* cos_cache, const float* sin_cache, int64_t n_pos,
                 int64_t q_pos_offset, int64_t k_pos_offset, void* cuda_stream);

/*
 * RoPE and attention in one launch: O = softmax(scale * rope(Q) rope(K)^T + mask) V, the
 * rotation of mlxp_rope (half-split, fp32 cos/sin tables [n_pos][D/2], rounded once to the
 * element type) applied to Q at positions q_rope_offset + i and to K at k_rope_offset + j.
 * Replaces the reference's fused kernel, which rotates Q and K as it loads them
 * (mlx_primitives/kernels/fused_rope_attention.py:52-198, called by fused_rope_attention
 * :939-985).  Here the persistent attention kernel also runs rotation work items: chunks of
 * 256 rows of Q and K are rotated into the workspace (rotation for the next scheduling group of
 * (batch, head) units is handed out before attention of the current one, so the rotated rows
 * are read back from L2), and the attention items read them through TMA.  The result is bit
 * for bit that of mlxp_rope_qk followed by mlxp_attn_fwd.  Masks (causal, windows, offsets) as
 * mlxp_attn_fwd — independent of the RoPE positions.  bf16/fp16, head_dim 64 or 128, as many
 * K/V heads as query heads; q and k rows 16-byte aligned.  workspace: >=
 * mlxp_rope_attn_workspace_size bytes, 256-byte aligned (the rotated copies of Q and K, counters,
 * and any key-split scratch).
 */
int mlxp_rope_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                       int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Skv, int64_t D,
                       const int64_t q_strides[4], const int64_t k_strides[4],
                       const int64_t v_strides[4], const int64_t o_strides[4],
                       const float* cos_cache, const float* sin_cache, int64_t n_pos,
                       int64_t q_rope_offset, int64_t k_rope_offset, float scale, int causal,
                       int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                       int64_t kv_pos_offset, int64_t kv_splits, void* workspace,
                       size_t ws_bytes, void* cuda_stream);

/* Bytes of workspace mlxp_rope_attn_fwd needs for these arguments (0 for an invalid shape). */
size_t mlxp_rope_attn_workspace_size(int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Skv,
                                     int64_t D, int causal, int64_t window_left,
                                     int64_t window_right, int64_t q_pos_offset,
                                     int64_t kv_pos_offset, int64_t kv_splits);

/*
 * Backward pass of attention: dQ, dK, dV of O = softmax(scale * Q K^T + mask) V, the gradient
 * the reference obtains by MLX autodiff through its forward (mlx_primitives/attention/
 * flash.py:52-316; checked by tests/gradients/test_numerical_gradients.py:20-270).
 * Inputs: q, k, v and the forward's o and lse (fp32 [B][H][Sq], natural log, as returned by
 * mlxp_attn_fwd), and dout = dL/dO.  Outputs dq, dk, dv in the input dtype (dk/dv per K/V
 * head: grouped heads sum their query heads' contributions).  Every tensor through its own
 * strides ((batch, head, seq, dim) order, dim stride 1); masks and offsets as mlxp_attn_fwd.
 * head_dim 32, 64 or 128; computed in fp32.  workspace: >= mlxp_attn_bwd_workspace_size bytes,
 * 256-byte aligned.  bf16/fp16 with head_dim 64 or 128 run on the tensor cores (P and dS rounded to
 * the input type for the matmuls, as flash-attention backward passes do; dQ accumulated in
 * fp32 by TMA reduce-add, so its last bits depend on the order of the additions); the rest on
 * CUDA cores in fp32, deterministic.
 */
int mlxp_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                  const float* lse, void* dq, void* dk, void* dv, int dtype, int64_t B,
                  int64_t H, int64_t H_kv, int64_t Sq, int64_t Skv, int64_t D,
                  const int64_t q_strides[4], const int64_t k_strides[4],
                  const int64_t v_strides[4], const int64_t o_strides[4],
                  const int64_t do_strides[4], const int64_t dq_strides[4],
                  const int64_t dk_strides[4], const int64_t dv_strides[4], float scale,
                  int causal, int64_t window_left, int64_t window_right, int64_t q_pos_offset,
                  int64_t kv_pos_offset, void* workspace, size_t ws_bytes, void* cuda_stream);

/*
 * Which backward runs: 0 (default) = the tensor-core kernel where it applies (bf16/fp16,
 * head_dim 64 or 128, TMA-compatible operands), the CUDA-core kernels otherwise; 1 = always the
 * CUDA-core kernels (for cross-checking the two).  Process-wide.
 */
int mlxp_set_backward_path(int cuda_cores_only);

/* Bytes of workspace mlxp_attn_bwd needs (the per-row dO . O terms; for the tensor-core path
 * also the padded log-sum-exp rows and the fp32 dQ accumulator). */
size_t mlxp_attn_bwd_workspace_size(int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Skv,
                                    int64_t D);

/*
 * Attention over a paged K/V pool: replaces paged_attention and paged_attention_with_bias
 * (mlx_primitives/cache/paged_attention.py:44-105 and 323-384), whose decode and prefill
 * bodies (paged_attention.py:108-208, 211-320) gather the pool blocks into dense K/V first.
 * Here the kernel reads the blocks in place through the block table.
 *   q, o:        [B][H][Sq][D] through q_strides / o_strides ((batch, head, seq, dim) order).
 *   k_pool, v_pool: (num_blocks, block_size, kv_heads, D) through pool_strides ((block,
 *                token, head, dim) order, shared by both pools); query head h reads pool head
 *                h / (H / kv_heads) (kv_heads = H in the reference).
 *   block_tables: int32 [B][max_blocks], row stride bt_stride; -1 marks a missing block.
 *   context_lens: int32 [B].
 *   alibi_slopes: fp32 [H] or NULL (get_alibi_slopes, paged_attention.py:17-41).
 * Key position t = slot * block_size + offset is admissible when t < context_lens[b], the
 * slot's id is in [0, num_blocks), and, if causal and Sq > 1, t <= query index.  ALiBi adds
 * slope[h] * (t - q_pos), q_pos = context_lens[b] when Sq == 1 and the query index otherwise.
 * A query row with no admissible key gets zeros (the reference's softmax gives NaN).
 * head_dim 32, 64 or 128; fp32/bf16/fp16, computed in fp32.  q and the pools 4*elem-size
 * aligned with strides that are multiples of 4 elements.  kv_splits: 0 = automatic, 1 = none,
 * n = n shares of the block table per query row (combined by an LSE merge into o).
 * workspace: >= mlxp_paged_attn_workspace_size bytes, 256-byte aligned (0 bytes when no split).
 */
int mlxp_paged_attn(const void* q, const void* k_pool, const void* v_pool,
                    const int32_t* block_tables, const int32_t* context_lens,
                    const float* alibi_slopes, void* o, int dtype, int64_t B, int64_t H,
                    int64_t Sq, int64_t D, int64_t kv_heads, int64_t num_blocks,
                    int64_t block_size, int64_t max_blocks, const int64_t q_strides[4],
                    const int64_t pool_strides[4], int64_t bt_stride,
                    const int64_t o_strides[4], float scale, int causal, int64_t kv_splits,
                    void* workspace, size_t ws_bytes, void* cuda_stream);

/* Bytes of workspace mlxp_paged_attn needs for these arguments (0 = none, or invalid shape). */
size_t mlxp_paged_attn_workspace_size(int dtype, int64_t B, int64_t H, int64_t Sq, int64_t D,
                                      int64_t kv_heads, int64_t num_blocks, int64_t block_size,
                                      int64_t max_blocks, int64_t kv_splits);

/*
 * Device-side status word of the current device: 0 when every bounded wait completed,
 * otherwise MLXP_ERR_TIMEOUT | (site << 8), or MLXP_ERR_WORKSPACE | (site << 8) when a kernel
 * found its workspace smaller than its work (it then wrote nothing there).  Synchronises the
 * device.  reset != 0 clears it.
 */
int mlxp_device_status(int* status_out, int reset);

/* Limit for every bounded device-side wait, in nanoseconds (default 2 s). */
int mlxp_set_wait_timeout_ns(uint64_t ns);

/*
 * Self-test of the bounded-wait machinery: launches one CTA whose threads wait on an
 * mbarrier that nothing ever arrives on, with the given limit.  Returns MLXP_ERR_TIMEOUT
 * (and leaves the device status set) when the wait correctly gave up; MLXP_OK would mean the
 * wait completed, which cannot happen.  Synchronises the stream.
 */
int mlxp_selftest_wait_timeout(uint64_t timeout_ns, void* cuda_stream);

/*
 * Sequence-parallel causal attention over NCCL (one process per GPU), for callers that are not
 * Python; the reference is single-device, so these have no counterpart there: they are the
 * ring entry points the long-context configuration needs (the Python API runs the same schedule
 * over torch.distributed in mlx_primitives/attention/ring.py).
 *
 * The full sequence of S = nranks * S_local tokens is cut into 2 * nranks chunks of
 * C = S_local / 2; rank r holds chunks r and 2*nranks-1-r of Q, K and V back to back (zig-zag)
 * and receives the same chunks of O.  NCCL is loaded at run time (libnccl.so.2); when it cannot
 * be, these return MLXP_ERR_NCCL.  Each rank calls them on its own device (the current device at
 * mlxp_ring_init).  A rank that never joins leaves the others blocked inside NCCL, as with any
 * NCCL collective: a process-level watchdog is the caller's.
 */

/* A new 128-byte NCCL unique id: created on one rank and shared with the others out of band. */
int mlxp_ring_unique_id(void* id_out);

/* Joins the ring of nranks ranks as `rank`; *comm receives the handle. */
int mlxp_ring_init(const void* nccl_unique_id, int nranks, int rank, void** comm);

/* Bytes of device workspace mlxp_ring_attn_fwd needs (0 for an invalid shape). */
size_t mlxp_ring_workspace_size(int dtype, int64_t B, int64_t H, int64_t S_local, int64_t D);

/*
 * o = causal softmax(scale * q k^T) v of this rank's zig-zag shard, against the whole
 * sequence.  q, k, v, o: [B][H][S_local][D] with element strides (BHSD or BSHD), bf16/fp16,
 * D in {64, 128}, S_local even.  Collective: every rank calls it with the same shapes, in the
 * same order.  workspace: >= mlxp_ring_workspace_size bytes, 256-byte aligned.
 */
int mlxp_ring_attn_fwd(void* comm, const void* q, const void* k, const void* v, void* o,
                       int dtype, int64_t B, int64_t H, int64_t S_local, int64_t D,
                       const int64_t q_strides[4], const int64_t k_strides[4],
                       const int64_t v_strides[4], const int64_t o_strides[4], float scale,
                       void* workspace, size_t ws_bytes, void* cuda_stream);

/* Leaves the ring and frees the handle (NULL is a no-op). */
int mlxp_ring_destroy(void* comm);

#ifdef __cplusplus
}
#endif

#endif /* MLXP_ATTN_H */
