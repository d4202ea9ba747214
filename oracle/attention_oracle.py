"""CPU oracle for the attention forward path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithms of the reference's attention path
(zakkeown/mlx-primitives, mlx_primitives/attention/*.py).  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline / reference arm may import it, and only as the checker or the timed
CPU baseline.  The product (mlx_primitives + libmlxp_attn.so) never calls it.

Parity is pinned: tests/golden/*.npz hold outputs of the reference's own Python code paths
(flash.py:257-316 tiled loop, flash.py:479-525 dense path, sliding_window.py:363-511 tiled
loop, chunked.py:129-203 chunk loop and dense path, _online_softmax.py:42-176 merge/chunk
helpers) executed over a numpy stand-in for the mlx.core array functions they call
(tests/golden/make_golden.py); tests/test_oracle_golden.py checks this restatement against them.

Conventions (file:line in the reference):
  mask value -1e38                                   constants.py:100
  softmax-denominator epsilon 1e-6 (tiled paths)     constants.py:110, flash.py:312
  causal, equal lengths: j <= i                      flash.py:286, _online_softmax.py:149-161
  causal mask Sq != Skv: bottom-right aligned        utils/masking.py:14-66 (triu k=Skv-Sq+1)
  sliding window: |i - j| <= W (and j <= i)          sliding_window.py:136-161
  chunked causal: top-left absolute positions        chunked.py:192-197
"""

from __future__ import annotations

import math

import numpy as np

MASK_VALUE = -1e38     # constants.py:100 ATTENTION_MASK_VALUE
SOFTMAX_EPS = 1e-6     # constants.py:110 METAL_SOFTMAX_EPSILON


# ----------------------------------------------------------------------------------------
# Masks
# ----------------------------------------------------------------------------------------
def admissible(sq: int, skv: int, causal: bool, window_left: int = -1, window_right: int = -1,
               q_offset: int = 0, kv_offset: int = 0) -> np.ndarray:
    """Boolean (sq, skv): key j admissible for query i, positions qpos = i + q_offset,
    kpos = j + kv_offset (the C-ABI's convention)."""
    qpos = np.arange(sq, dtype=np.int64)[:, None] + q_offset
    kpos = np.arange(skv, dtype=np.int64)[None, :] + kv_offset
    ok = np.ones((sq, skv), dtype=bool)
    if causal:
        ok &= kpos <= qpos
    if window_left >= 0:
        ok &= (qpos - kpos) <= window_left
    if window_right >= 0:
        ok &= (kpos - qpos) <= window_right
    return ok


def create_causal_mask(seq_q: int, seq_kv: int, dtype=np.float32) -> np.ndarray:
    """utils/masking.py:14-66: additive -1e38 above diagonal offset seq_kv - seq_q + 1."""
    return np.triu(np.full((seq_q, seq_kv), MASK_VALUE, dtype=dtype), k=seq_kv - seq_q + 1)


def create_sliding_window_mask(seq_len: int, window_size: int, causal: bool = True) -> np.ndarray:
    """sliding_window.py:628-656: True where |i - j| <= W (and j <= i if causal)."""
    pos = np.arange(seq_len)
    mask = np.abs(pos[:, None] - pos[None, :]) <= window_size
    if causal:
        mask &= pos[None, :] <= pos[:, None]
    return mask


# ----------------------------------------------------------------------------------------
# Dense attention: the semantic definition every kernel is checked against
# ----------------------------------------------------------------------------------------
def attention_bhsd(q, k, v, scale: float, causal: bool = False, window_left: int = -1,
                   window_right: int = -1, q_offset: int = 0, kv_offset: int = 0,
                   dtype=np.float64, empty_rows: str = "zero", return_lse: bool = False,
                   bias=None):
    """softmax(scale * Q K^T + mask) V per (b, h) for BHSD arrays, computed in `dtype`.

    This is the reference's dense path (flash.py:186-192 / 479-525, sliding_window.py:514-560,
    chunked.py:172-203) with the mask given in absolute positions.  Rows with no admissible key:
    empty_rows="zero" gives O = 0 / LSE = -inf (the B200 library's definition); "mean" gives the
    reference's finite-mask result mean(V) (every score replaced by -1e38).  `bias`: an additive
    score mask broadcastable to (B, H, Sq, Skv), added after scaling (grouped_query.py:253-254);
    rows it leaves without a finite score count as empty.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    B, H, Sq, D = q.shape
    Skv = k.shape[2]
    ok = admissible(Sq, Skv, causal, window_left, window_right, q_offset, kv_offset)
    empty = ~ok.any(axis=1)
    out = np.zeros((B, H, Sq, v.shape[3]), dtype=dtype)
    lse = np.full((B, H, Sq), -np.inf, dtype=np.float64)
    if bias is not None:
        bias = np.broadcast_to(np.asarray(bias, dtype=dtype), (B, H, Sq, Skv))
    for b in range(B):
        for h in range(H):
            s = (q[b, h] @ k[b, h].T) * scale
            if bias is not None:
                s = s + bias[b, h]
            s = np.where(ok, s, -np.inf)
            if bias is not None:
                empty = ~np.isfinite(s).any(axis=1)
            m = s.max(axis=1, keepdims=True)
            m = np.where(np.isfinite(m), m, 0.0)
            e = np.exp(s - m)
            den = e.sum(axis=1, keepdims=True)
            o = (e @ v[b, h]) / np.where(den > 0, den, 1.0)
            with np.errstate(divide="ignore"):
                lse[b, h] = np.where(den[:, 0] > 0, np.log(np.where(den[:, 0] > 0, den[:, 0], 1.0)) + m[:, 0], -np.inf)
            if empty.any():
                o[empty] = v[b, h].mean(axis=0) if empty_rows == "mean" else 0.0
            out[b, h] = o
    return (out, lse) if return_lse else out


def attention_rows_bhsd(q, k, v, rows, scale: float, causal: bool = True, window_left: int = -1,
                        window_right: int = -1, q_offset: int = 0, kv_offset: int = 0,
                        bh=None):
    """Exact fp64 outputs for selected query rows only: [len(bh), len(rows), D].

    Row-sampled oracle for shapes whose full score matrix is too large (e.g. 128K tokens):
    each sampled row against its full admissible key range.  `bh` lists (b, h) pairs
    (default: all)."""
    q = np.asarray(q)
    B, H = q.shape[:2]
    pairs = bh if bh is not None else [(b, h) for b in range(B) for h in range(H)]
    rows = np.asarray(rows, dtype=np.int64)
    out = np.zeros((len(pairs), len(rows), v.shape[3]), dtype=np.float64)
    Skv = k.shape[2]
    for n, (b, h) in enumerate(pairs):
        qs = np.asarray(q[b, h, rows], dtype=np.float64)
        kk = np.asarray(k[b, h], dtype=np.float64)
        vv = np.asarray(v[b, h], dtype=np.float64)
        s = (qs @ kk.T) * scale
        qpos = rows[:, None] + q_offset
        kpos = np.arange(Skv)[None, :] + kv_offset
        ok = np.ones_like(s, dtype=bool)
        if causal:
            ok &= kpos <= qpos
        if window_left >= 0:
            ok &= (qpos - kpos) <= window_left
        if window_right >= 0:
            ok &= (kpos - qpos) <= window_right
        s = np.where(ok, s, -np.inf)
        m = s.max(axis=1, keepdims=True)
        e = np.exp(s - m)
        out[n] = (e @ vv) / e.sum(axis=1, keepdims=True)
    return out


def to_bhsd(x, layout: str):
    return x if layout == "BHSD" else np.swapaxes(x, 1, 2)


def from_bhsd(x, layout: str):
    return x if layout == "BHSD" else np.swapaxes(x, 1, 2)


# ----------------------------------------------------------------------------------------
# Public-API semantics of the reference (what each entry point computes)
# ----------------------------------------------------------------------------------------
def flash_attention(q, k, v, scale=None, causal=True, layout="BSHD", dtype=np.float64):
    """flash.py:52-254 semantics: causal aligned bottom-right (SDPA mask="causal",
    utils/masking.py:14-66), default scale 1/sqrt(head_dim), output in `layout`."""
    qb, kb, vb = (to_bhsd(np.asarray(t), layout) for t in (q, k, v))
    if scale is None:
        scale = 1.0 / math.sqrt(qb.shape[-1])
    sq, skv = qb.shape[2], kb.shape[2]
    o = attention_bhsd(qb, kb, vb, scale, causal=causal, q_offset=(skv - sq) if causal else 0,
                       dtype=dtype)
    return from_bhsd(o, layout)


def sliding_window_attention(q, k, v, window_size, scale=None, causal=True, dtype=np.float64):
    """sliding_window.py:227-312 semantics (BSHD): |i - j| <= W, and j <= i if causal."""
    qb, kb, vb = (to_bhsd(np.asarray(t), "BSHD") for t in (q, k, v))
    if scale is None:
        scale = 1.0 / math.sqrt(qb.shape[-1])
    o = attention_bhsd(qb, kb, vb, scale, causal=causal, window_left=window_size,
                       window_right=-1 if causal else window_size, dtype=dtype)
    return from_bhsd(o, "BSHD")


def chunked_cross_attention(q, k, v, chunk_size=1024, scale=None, causal=False, dtype=np.float64):
    """chunked.py:43-126 semantics (BSHD): full attention over Skv, causal top-left."""
    qb, kb, vb = (to_bhsd(np.asarray(t), "BSHD") for t in (q, k, v))
    if scale is None:
        scale = 1.0 / math.sqrt(qb.shape[-1])
    o = attention_bhsd(qb, kb, vb, scale, causal=causal, dtype=dtype)
    return from_bhsd(o, "BSHD")


def gqa_attention(q, k, v, num_kv_groups, scale=None, mask=None, causal=False, dtype=np.float64):
    """grouped_query.py:195-261 semantics (BSHD): K/V head j serves query heads
    j*num_kv_groups .. (j+1)*num_kv_groups-1 (broadcast + reshape in the reference); causal
    aligned bottom-right (triu(k = seq_kv - seq_q + 1)).  Rows with no admissible key give 0
    (the library's convention; the reference's -inf mask would give NaN there)."""
    q, k, v = (np.asarray(t) for t in (q, k, v))
    if q.shape[2] != k.shape[2] * num_kv_groups:
        raise ValueError("num_heads must equal num_kv_heads * num_kv_groups")
    k = np.repeat(k, num_kv_groups, axis=2)
    v = np.repeat(v, num_kv_groups, axis=2)
    if mask is None:
        return flash_attention(q, k, v, scale=scale, causal=causal, layout="BSHD", dtype=dtype)
    # custom additive mask (grouped_query.py:253-254): scores + causal mask + mask, softmax
    Sq, Skv = q.shape[1], k.shape[1]
    if scale is None:
        scale = 1.0 / np.sqrt(q.shape[-1])
    o = attention_bhsd(to_bhsd(q, "BSHD"), to_bhsd(k, "BSHD"), to_bhsd(v, "BSHD"), scale,
                       causal=causal, q_offset=(Skv - Sq) if causal else 0, dtype=dtype,
                       bias=mask)
    return from_bhsd(o, "BSHD")


def mqa_attention(q, k, v, scale=None, mask=None, causal=False, dtype=np.float64):
    """multi_query.py:161-225 semantics: one K/V head ((B, Skv, D) or (B, Skv, 1, D)) for all
    query heads."""
    k, v = np.asarray(k), np.asarray(v)
    if k.ndim == 3:
        k, v = k[:, :, None, :], v[:, :, None, :]
    return gqa_attention(q, k, v, np.asarray(q).shape[2], scale=scale, mask=mask, causal=causal,
                         dtype=dtype)


def precompute_rope_cache(seq_len, head_dim, base=10000.0):
    """kernels/rope.py:223-255: theta_i = base^(-i/(head_dim/2)) and position angles in fp32,
    cos/sin (seq_len, head_dim // 2) in fp32."""
    half = head_dim // 2
    inv_freq = np.float32(base) ** (-np.arange(0, half, dtype=np.float32) / np.float32(half))
    freqs = np.outer(np.arange(seq_len, dtype=np.float32), inv_freq.astype(np.float32))
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


def rope(x, cos, sin, offset=0, dtype=np.float64):
    """kernels/rope.py:477-496 (BSHD): half-split rotation at positions offset + s."""
    x = np.asarray(x, dtype=dtype)
    s = x.shape[1]
    h = x.shape[-1] // 2
    c = np.asarray(cos, dtype=dtype)[offset:offset + s][None, :, None, :]
    sn = np.asarray(sin, dtype=dtype)[offset:offset + s][None, :, None, :]
    x1, x2 = x[..., :h], x[..., h:]
    return np.concatenate([x1 * c - x2 * sn, x1 * sn + x2 * c], axis=-1)


def fused_rope_attention(q, k, v, scale=None, cos_cache=None, sin_cache=None, rope_base=10000.0,
                         q_offset=0, kv_offset=0, causal=False, dtype=np.float64):
    """kernels/fused_rope_attention.py:766-800 semantics: RoPE on Q (positions from q_offset)
    and K (from kv_offset), then flash_attention (BSHD, causal bottom-right)."""
    q, k, v = (np.asarray(t) for t in (q, k, v))
    if cos_cache is None or sin_cache is None:
        max_pos = max(q.shape[1] + q_offset, k.shape[1] + kv_offset)
        cos_cache, sin_cache = precompute_rope_cache(max_pos, q.shape[-1], rope_base)
    qr = rope(q, cos_cache, sin_cache, q_offset, dtype)
    kr = rope(k, cos_cache, sin_cache, kv_offset, dtype)
    return flash_attention(qr, kr, v, scale=scale, causal=causal, layout="BSHD", dtype=dtype)


# ----------------------------------------------------------------------------------------
# The reference's own blockwise algorithms (fp32, as MLX computes them)
# ----------------------------------------------------------------------------------------
def compute_chunk_attention(q, k_chunk, v_chunk, scale, causal=False, q_offset=0, kv_offset=0):
    """_online_softmax.py:109-176 — BSHD block scores, -1e38 causal mask in absolute
    positions, row max m, row sum l of exp(s - m), unnormalised O = sum exp(s - m) V."""
    s = np.einsum("bqhd,bkhd->bqhk", q, k_chunk).astype(np.float32) * np.float32(scale)
    if causal:
        qpos = np.arange(q.shape[1]) + q_offset
        kpos = np.arange(k_chunk.shape[1]) + kv_offset
        ok = kpos[None, :] <= qpos[:, None]
        s = np.where(ok[None, :, None, :], s, np.float32(MASK_VALUE))
    m = s.max(axis=-1)
    e = np.exp(s - m[..., None])
    l = e.sum(axis=-1)
    o = np.einsum("bqhk,bkhd->bqhd", e, v_chunk)
    return o.astype(np.float32), m.astype(np.float32), l.astype(np.float32)


def online_softmax_merge(acc_o, acc_m, acc_l, new_o, new_m, new_l):
    """_online_softmax.py:42-106 — m' = max(m1, m2); l' = l1 e^(m1-m') + l2 e^(m2-m');
    O' = O1 e^(m1-m') + O2 e^(m2-m')."""
    gm = np.maximum(acc_m, new_m)
    ca = np.exp(acc_m - gm)
    cn = np.exp(new_m - gm)
    return acc_o * ca[..., None] + new_o * cn[..., None], gm, acc_l * ca + new_l * cn


def tiled_flash_attention(q, k, v, scale, causal, block_q=32, block_kv=32):
    """flash.py:257-316 — query blocks x key blocks (causal: keys < q_end), merged with
    online_softmax_merge, normalised by (l + 1e-6)."""
    q, k, v = (np.asarray(t, dtype=np.float32) for t in (q, k, v))
    B, S, H, D = q.shape
    outs = []
    for q0 in range(0, S, block_q):
        q1 = min(q0 + block_q, S)
        n = q1 - q0
        m = np.full((B, n, H), MASK_VALUE, dtype=np.float32)
        l = np.zeros((B, n, H), dtype=np.float32)
        o = np.zeros((B, n, H, D), dtype=np.float32)
        limit = q1 if causal else S
        for k0 in range(0, limit, block_kv):
            k1 = min(k0 + block_kv, limit)
            co, cm, cl = compute_chunk_attention(q[:, q0:q1], k[:, k0:k1], v[:, k0:k1], scale,
                                                 causal=causal, q_offset=q0, kv_offset=k0)
            o, m, l = online_softmax_merge(o, m, l, co, cm, cl)
        outs.append(o / (l[..., None] + np.float32(SOFTMAX_EPS)))
    return np.concatenate(outs, axis=1)


def tiled_sliding_window_attention(q, k, v, window_size, scale, causal, block_q=32):
    """sliding_window.py:363-511 — key range [max(0, q0 - W), q_end) (causal) or
    [max(0, q0 - W), min(S, q_end + W)), exact |i - j| <= W (+ causal) mask per element."""
    q, k, v = (np.asarray(t, dtype=np.float32) for t in (q, k, v))
    B, S, H, D = q.shape
    outs = []
    for q0 in range(0, S, block_q):
        q1 = min(q0 + block_q, S)
        n = q1 - q0
        m = np.full((B, n, H), MASK_VALUE, dtype=np.float32)
        l = np.zeros((B, n, H), dtype=np.float32)
        o = np.zeros((B, n, H, D), dtype=np.float32)
        k_lo = max(0, q0 - window_size)
        k_hi = q1 if causal else min(S, q1 + window_size)
        for k0 in range(k_lo, k_hi, block_q):
            k1 = min(k0 + block_q, k_hi)
            s = np.einsum("bqhd,bkhd->bqhk", q[:, q0:q1], k[:, k0:k1]) * np.float32(scale)
            qpos = np.arange(q0, q1)[:, None]
            kpos = np.arange(k0, k1)[None, :]
            ok = np.abs(qpos - kpos) <= window_size
            if causal:
                ok &= kpos <= qpos
            s = np.where(ok[None, :, None, :], s, np.float32(MASK_VALUE))
            cm = s.max(axis=-1)
            e = np.exp(s - cm[..., None])
            cl = e.sum(axis=-1)
            co = np.einsum("bqhk,bkhd->bqhd", e, v[:, k0:k1])
            o, m, l = online_softmax_merge(o, m, l, co, cm, cl)
        outs.append(o / (l[..., None] + np.float32(SOFTMAX_EPS)))
    return np.concatenate(outs, axis=1)


def chunked_cross_attention_loop(q, k, v, chunk_size, scale, causal=False):
    """chunked.py:129-169 — for each key chunk: compute_chunk_attention (q_offset 0,
    kv_offset = chunk start), online_softmax_merge; finally / (l + 1e-6)."""
    q, k, v = (np.asarray(t, dtype=np.float32) for t in (q, k, v))
    B, Sq, H, D = q.shape
    o = np.zeros((B, Sq, H, D), dtype=np.float32)
    m = np.full((B, Sq, H), MASK_VALUE, dtype=np.float32)
    l = np.zeros((B, Sq, H), dtype=np.float32)
    for c0 in range(0, k.shape[1], chunk_size):
        c1 = min(c0 + chunk_size, k.shape[1])
        co, cm, cl = compute_chunk_attention(q, k[:, c0:c1], v[:, c0:c1], scale, causal=causal,
                                             q_offset=0, kv_offset=c0)
        o, m, l = online_softmax_merge(o, m, l, co, cm, cl)
    return o / (l[..., None] + np.float32(SOFTMAX_EPS))


# ----------------------------------------------------------------------------------------
# LSE form of the merge (what the split-KV and ring kernels compute)
# ----------------------------------------------------------------------------------------
def lse_merge(o_parts, lse_parts):
    """Merge normalised partials: w_i = exp(lse_i - max lse); O = sum w_i O_i / sum w_i."""
    o_parts = np.asarray(o_parts, dtype=np.float64)
    lse_parts = np.asarray(lse_parts, dtype=np.float64)
    mx = lse_parts.max(axis=0)
    safe = np.where(np.isfinite(mx), mx, 0.0)
    w = np.exp(lse_parts - safe)
    den = w.sum(axis=0)
    o = (w[..., None] * o_parts).sum(axis=0) / np.where(den > 0, den, 1.0)[..., None]
    with np.errstate(divide="ignore"):
        lse = np.where(den > 0, safe + np.log(np.where(den > 0, den, 1.0)), -np.inf)
    return o, lse


# ----------------------------------------------------------------------------------------
# Backward: the gradient the reference takes by MLX autodiff through its forward
# ----------------------------------------------------------------------------------------
def attention_bwd_bhsd(q, k, v, dout, scale: float, causal: bool = False, window_left: int = -1,
                       window_right: int = -1, q_offset: int = 0, kv_offset: int = 0):
    """dQ, dK, dV (fp64, BHSD) of O = softmax(scale * Q K^T + mask) V for the loss
    sum(dout * O), by the chain rule written out: P = softmax(S), dV = P^T dO, dP = dO V^T,
    dS = P * (dP - rowsum(dO * O)), dQ = scale dS K, dK = scale dS^T Q.  K/V may have fewer
    heads than Q (grouped heads: query head h reads K/V head h // (H / H_kv)); their gradients
    sum over the query heads that read them.  Rows with no admissible key contribute nothing.
    This is what autodiff of the reference's forward (flash.py:52-316 under mx.grad) computes;
    tests/test_oracle_backward.py checks it against torch autograd of the dense definition."""
    q, k, v, dout = (np.asarray(t, dtype=np.float64) for t in (q, k, v, dout))
    B, H, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    g = H // Hkv
    ok = admissible(Sq, Skv, causal, window_left, window_right, q_offset, kv_offset)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for b in range(B):
        for h in range(H):
            kh, vh = k[b, h // g], v[b, h // g]
            s = np.where(ok, (q[b, h] @ kh.T) * scale, -np.inf)
            m = s.max(axis=1, keepdims=True)
            m = np.where(np.isfinite(m), m, 0.0)
            e = np.exp(s - m)
            den = e.sum(axis=1, keepdims=True)
            p = e / np.where(den > 0, den, 1.0)
            o = p @ vh
            dv[b, h // g] += p.T @ dout[b, h]
            dp = dout[b, h] @ vh.T
            ds = p * (dp - (dout[b, h] * o).sum(axis=1, keepdims=True))
            dq[b, h] = scale * ds @ kh
            dk[b, h // g] += scale * ds.T @ q[b, h]
    return dq, dk, dv


# ----------------------------------------------------------------------------------------
# Paged K/V attention (cache/paged_attention.py)
# ----------------------------------------------------------------------------------------
def get_alibi_slopes(num_heads: int) -> np.ndarray:
    """paged_attention.py:17-41: slope_h = (2^(-8/H))^(h+1), fp32."""
    ratio = 2 ** (-8 / num_heads)
    return np.array([ratio ** (i + 1) for i in range(num_heads)], dtype=np.float32)


def create_block_table_from_lengths(sequence_lengths, block_size: int, max_blocks=None):
    """paged_attention.py:387-440: sequence b owns blocks cum[b] .. cum[b] + n_b - 1
    (n_b = ceil(len_b / block_size), cum = exclusive prefix sum of n), -1 past n_b; int32."""
    lens = np.asarray(sequence_lengths, dtype=np.int64)
    n = (lens + block_size - 1) // block_size
    mb = int(n.max()) if max_blocks is None else int(max_blocks)
    cum = np.concatenate([[0], np.cumsum(n)[:-1]])
    pos = np.arange(mb)[None, :]
    return np.where(pos < n[:, None], cum[:, None] + pos, -1).astype(np.int32)


def paged_attention(q, k_pool, v_pool, block_tables, context_lens, scale=None, block_size=16,
                    causal=True, alibi_slopes=None, dtype=np.float64):
    """paged_attention.py:44-320 semantics.  q (B, Sq, H, D); pools (num_blocks, block_size,
    H, D); block_tables (B, max_blocks), -1 = missing block; context_lens (B,).

    The reference gathers pool blocks max(id, 0) into (B, max_blocks * block_size, H, D)
    (lines 137-147, 249-259) and masks key position t unless t < context_lens[b] and the
    slot's id >= 0 (lines 181-199, 288-303); with Sq > 1 and causal it also masks t > i
    (lines 306-313: top-left, query i at position i).  ALiBi adds slope[h] * (t - q_pos) to the
    scaled scores, q_pos = context_lens[b] for Sq == 1 (lines 161-179) and i otherwise
    (lines 271-286).  Softmax over the masked scores: a row with no admissible key is NaN, as
    the reference's softmax of all -inf gives.
    """
    q = np.asarray(q, dtype=dtype)
    k_pool = np.asarray(k_pool, dtype=dtype)
    v_pool = np.asarray(v_pool, dtype=dtype)
    bt = np.asarray(block_tables, dtype=np.int64)
    ctx = np.asarray(context_lens, dtype=np.int64)
    B, Sq, H, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    mb = bt.shape[1]
    T = mb * block_size
    safe = np.maximum(bt, 0)
    k = k_pool[safe].reshape(B, T, H, D)
    v = v_pool[safe].reshape(B, T, H, D)
    s = np.einsum("bqhd,bthd->bhqt", q, k) * scale                 # (B, H, Sq, T)
    t = np.arange(T)
    if alibi_slopes is not None:
        slopes = np.asarray(alibi_slopes, dtype=dtype)
        qpos = ctx[:, None] if Sq == 1 else np.broadcast_to(np.arange(Sq), (B, Sq))
        diff = (t[None, None, :] - qpos[:, :, None]).astype(dtype)  # (B, Sq, T)
        s = s + slopes[None, :, None, None] * diff[:, None]
    valid = (t[None, :] < ctx[:, None]) & (bt[:, t // block_size] >= 0)  # (B, T)
    valid = np.broadcast_to(valid[:, None, None, :], s.shape)
    if causal and Sq > 1:
        valid = valid & (t[None, :] <= np.arange(Sq)[:, None])[None, None]
    s = np.where(valid, s, -np.inf)
    with np.errstate(invalid="ignore"):
        m = s.max(axis=-1, keepdims=True)
        e = np.exp(s - m)
        p = e / e.sum(axis=-1, keepdims=True)
    o = np.einsum("bhqt,bthd->bqhd", p, v)
    return o


# ----------------------------------------------------------------------------------------
# Zig-zag ring schedule (the sequence-parallel split of the 128K-token causal config)
# ----------------------------------------------------------------------------------------
def zigzag_chunks(world: int, rank: int):
    """Global chunk ids held by `rank` when the sequence is cut into 2*world chunks."""
    return (rank, 2 * world - 1 - rank)


def ring_reference(q, k, v, world: int, scale: float):
    """Run the zig-zag ring schedule serially on CPU for BHSD q/k/v of the full sequence and
    return the full output: every rank's local queries against every K/V block that reaches it,
    each pair a partial (O, LSE) merged with lse_merge.  Must equal attention_bhsd(causal)."""
    q, k, v = (np.asarray(t, dtype=np.float64) for t in (q, k, v))
    B, H, S, D = q.shape
    C = S // (2 * world)
    out = np.zeros_like(q)
    for r in range(world):
        for qc in zigzag_chunks(world, r):
            qs = q[:, :, qc * C:(qc + 1) * C]
            parts_o, parts_l = [], []
            for step in range(world):
                src = (r - step) % world
                for kc in zigzag_chunks(world, src):
                    if kc > qc:
                        continue  # entirely above the diagonal
                    o, lse = attention_bhsd(qs, k[:, :, kc * C:(kc + 1) * C],
                                            v[:, :, kc * C:(kc + 1) * C], scale, causal=True,
                                            q_offset=qc * C, kv_offset=kc * C, return_lse=True)
                    parts_o.append(o)
                    parts_l.append(lse)
            o, _ = lse_merge(np.stack(parts_o), np.stack(parts_l))
            out[:, :, qc * C:(qc + 1) * C] = o
    return out


# ----------------------------------------------------------------------------------------
# Seeded inputs (identical arrays feed the oracle and the GPU)
# ----------------------------------------------------------------------------------------
def make_qkv(shape_q, shape_kv, seed: int = 42, std: float = 1.0, dtype=np.float32):
    """q, k, v ~ N(0, std^2) from numpy's legacy RandomState (stream frozen across numpy
    versions): q from seed, k from seed + 1, v from seed + 2."""
    q = np.random.RandomState(seed).standard_normal(shape_q).astype(np.float32) * np.float32(std)
    k = np.random.RandomState(seed + 1).standard_normal(shape_kv).astype(np.float32) * np.float32(std)
    v = np.random.RandomState(seed + 2).standard_normal(shape_kv).astype(np.float32) * np.float32(std)
    return q.astype(dtype), k.astype(dtype), v.astype(dtype)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 value (ties to even), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)
