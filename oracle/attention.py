"""ORACLE (test infrastructure): CPU restatement of the reference's attention path.

Used only by tests/, __graft_entry__.smoke() and bench.py's CPU baseline, as the checker.

* ``qkv_projection``      — the Ulysses attention graph, src/attention/builder.py:27-65
                            (q, k, v = x @ Wq, x @ Wk, x @ Wv reshaped per head).
* ``compute_attention``   — RootNode._compute_attention, src/orchestrator/root_node.py:250-314
                            (concat over nodes, [1, h, S, hd], RoPE, clip +-1000, optional
                            v-norm, GQA repeat, q k^T / sqrt(hd) with a causal -inf mask,
                            softmax, probs @ v, back to [1, S, h * hd]).
* ``attention_decode``    — RootNode._compute_attention_decode, root_node.py:1009-1031
                            (one query over the cache, padded prefill positions masked).
* ``decode_step``         — the decode attention block of root_node.py:900-933: RoPE of q and
                            k at start_pos = cache length, KV append, clip, attention_decode.

The kernels themselves (RoPE, softmax, RMSNorm) follow pyre_kernels.mojo through
oracle/kernels.py.
"""
from __future__ import annotations

import numpy as np

from . import kernels as K


def qkv_projection(x: np.ndarray, wq: np.ndarray, wk: np.ndarray, wv: np.ndarray, n_q: int, n_kv: int,
                   head_dim: int):
    """src/attention/builder.py:56-63. x [1, S, H] f32 -> q [1, S, n_q, hd], k/v [1, S, n_kv, hd]."""
    S = x.shape[1]
    x32 = x.astype(np.float32)
    q = (x32 @ wq.astype(np.float32)).astype(np.float32).reshape(1, S, n_q, head_dim)
    k = (x32 @ wk.astype(np.float32)).astype(np.float32).reshape(1, S, n_kv, head_dim)
    v = (x32 @ wv.astype(np.float32)).astype(np.float32).reshape(1, S, n_kv, head_dim)
    return q, k, v


def v_norm(v: np.ndarray) -> np.ndarray:
    """pyre_kernels.mojo apply_v_norm: f64 RMS over the last axis, eps 1e-6, no weight."""
    v64 = v.astype(np.float64)
    rstd = 1.0 / np.sqrt(np.sum(v64 * v64, axis=-1, keepdims=True) / v.shape[-1] + 1e-6)
    return (v64 * rstd).astype(np.float32)


def _gqa(x: np.ndarray, n_heads: int) -> np.ndarray:
    """root_node.py:295-297: repeat each KV head n_heads // n_kv times (head-major)."""
    _, n_kv, S, hd = x.shape
    rep = n_heads // n_kv
    return np.repeat(x[:, :, None, :, :], rep, axis=2).reshape(1, n_heads, S, hd)


def compute_attention(all_qkv, n_heads: int, n_kv: int, rope_fraction: float = 1.0, theta: float = 10000.0,
                      use_v_norm: bool = False, concat_by_head: bool = False) -> np.ndarray:
    """root_node.py:250-314 without the KV-sharing and cache bookkeeping.

    all_qkv: list over nodes (root first) of (q [1, S_i, h_i, hd], k, v). Returns [1, S, h*hd]."""
    axis = 2 if concat_by_head else 1
    q_full = np.concatenate([t[0] for t in all_qkv], axis=axis)
    k_full = np.concatenate([t[1] for t in all_qkv], axis=axis)
    v_full = np.concatenate([t[2] for t in all_qkv], axis=axis)
    S = q_full.shape[1]
    hd = q_full.shape[3]
    q = np.ascontiguousarray(q_full.transpose(0, 2, 1, 3)).astype(np.float32)
    k = np.ascontiguousarray(k_full.transpose(0, 2, 1, 3)).astype(np.float32)
    v = np.ascontiguousarray(v_full.transpose(0, 2, 1, 3)).astype(np.float32)
    if rope_fraction > 0:
        q = K.apply_rope(q, theta, 0, rope_fraction)
        k = K.apply_rope(k, theta, 0, rope_fraction)
    q = np.clip(q, -1000, 1000)
    k = np.clip(k, -1000, 1000)
    v = np.clip(v, -1000, 1000)
    if use_v_norm:
        v = v_norm(v)
    k_exp = _gqa(k, n_heads)
    v_exp = _gqa(v, n_heads)
    scale = np.float32(np.sqrt(hd))
    scores = (q @ k_exp.transpose(0, 1, 3, 2)).astype(np.float32) / scale
    mask = np.triu(np.full((S, S), -np.inf, dtype=np.float32), k=1)
    with np.errstate(invalid="ignore", over="ignore"):
        probs = K.softmax(scores + mask)
    attn = (probs @ v_exp).astype(np.float32)
    return attn.transpose(0, 2, 1, 3).reshape(1, S, n_heads * hd).astype(np.float32)


def attention_decode(q: np.ndarray, k: np.ndarray, v: np.ndarray, prefill_real: int = 0,
                     prefill_max_seq: int = 0) -> np.ndarray:
    """root_node.py:1009-1031. q [1, h, 1, hd]; k, v [1, n_kv, t, hd] -> [1, 1, h*hd]."""
    n_heads = q.shape[1]
    hd = q.shape[3]
    k_exp = _gqa(k.astype(np.float32), n_heads)
    v_exp = _gqa(v.astype(np.float32), n_heads)
    scale = np.float32(np.sqrt(hd))
    scores = (q.astype(np.float32) @ k_exp.transpose(0, 1, 3, 2)).astype(np.float32) / scale
    if prefill_max_seq > prefill_real:
        scores[:, :, :, prefill_real:prefill_max_seq] = -np.inf
    with np.errstate(invalid="ignore", over="ignore"):
        probs = K.softmax(scores)
    attn = (probs @ v_exp).astype(np.float32)
    return attn.transpose(0, 2, 1, 3).reshape(1, 1, n_heads * hd).astype(np.float32)


def decode_step(q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray, k_cache, v_cache, rope_fraction: float = 1.0,
                theta: float = 10000.0, prefill_real: int = 0, prefill_max_seq: int = 0):
    """root_node.py:900-933 for one token. q [1, h, 1, hd], k_new/v_new [1, n_kv, 1, hd];
    caches [1, n_kv, t, hd] or None. Returns (attn [1, 1, h*hd], k_cache', v_cache')."""
    cache_len = 0 if k_cache is None else k_cache.shape[2]
    q_r, k_r = q.astype(np.float32), k_new.astype(np.float32)
    if rope_fraction > 0:
        q_r = K.apply_rope(q_r, theta, cache_len, rope_fraction)
        k_r = K.apply_rope(k_r, theta, cache_len, rope_fraction)
    if k_cache is None:
        k_full, v_full = k_r, v_new.astype(np.float32)
    else:
        k_full = np.concatenate([k_cache, k_r], axis=2)
        v_full = np.concatenate([v_cache, v_new.astype(np.float32)], axis=2)
    out = attention_decode(np.clip(q_r, -1000, 1000), np.clip(k_full, -1000, 1000), np.clip(v_full, -1000, 1000),
                           prefill_real, prefill_max_seq)
    return out, k_full, v_full


def attention_rows_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, positions, heads, n_heads: int, n_kv: int,
                       theta: float, rope_fraction: float = 1.0) -> np.ndarray:
    """Row-wise f64 restatement of root_node.py:250-314 for chosen (query position, head) pairs
    of one causal sequence, for sequences whose full score matrix is too large to form (the
    32768-token long-context case): RoPE with the reference's f32 cos/sin tables
    (pyre_kernels.mojo:86-89) applied in f64, clip +-1000 (:288-290), the kv head of a query
    head (GQA, :295-297), q k^T / sqrt(hd) over positions 0..p (causal, :299-303), softmax and
    probs @ v, all in f64.

    q: [S, n_heads * hd], k, v: [S, n_kv * hd] (token-major projections, f32). positions,
    heads: equal-length integer sequences. Returns f64 [len(positions), hd]."""
    S = q.shape[0]
    hd = q.shape[1] // n_heads
    dims = int(float(hd) * float(rope_fraction))
    half = dims // 2 if dims >= 2 else 0
    c, s = K.rope_tables(theta, 0, S, max(dims, 2))
    c, s = c.astype(np.float64), s.astype(np.float64)

    rep = n_heads // n_kv
    out = np.empty((len(positions), hd), dtype=np.float64)
    kr_cache: dict = {}
    for i, (p, h) in enumerate(zip(positions, heads)):
        g = int(h) // rep
        if g not in kr_cache:
            kk = k[:, g * hd:(g + 1) * hd].astype(np.float64)
            vv = v[:, g * hd:(g + 1) * hd].astype(np.float64)
            if half:
                k1, k2 = kk[:, :half].copy(), kk[:, half:2 * half].copy()
                kk[:, :half] = k1 * c[:, :half] - k2 * s[:, :half]
                kk[:, half:2 * half] = k1 * s[:, :half] + k2 * c[:, :half]
            kr_cache[g] = (np.clip(kk, -1000, 1000), np.clip(vv, -1000, 1000))
        kk, vv = kr_cache[g]
        qq = q[int(p), int(h) * hd:(int(h) + 1) * hd].astype(np.float64)
        if half:
            q1, q2 = qq[:half].copy(), qq[half:2 * half].copy()
            qq[:half] = q1 * c[int(p), :half] - q2 * s[int(p), :half]
            qq[half:2 * half] = q1 * s[int(p), :half] + q2 * c[int(p), :half]
        qq = np.clip(qq, -1000, 1000)
        sc = kk[:int(p) + 1] @ qq / np.sqrt(float(hd))
        e = np.exp(sc - sc.max())
        out[i] = (e / e.sum()) @ vv[:int(p) + 1]
    return out
