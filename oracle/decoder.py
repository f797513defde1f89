"""ORACLE (test infrastructure): CPU restatement of the reference's whole-decoder greedy loop.

Used only by tests/ and __graft_entry__.smoke(), as the checker; pinned to the goldens that the
reference orchestrator itself produced (tests/golden/greedy_golden*.npz).

* ``layer``  — one decoder layer of RootNode with every head at the root (head-partitioned
               path): prefill, src/orchestrator/root_node.py:344-600 (RMSNorm, x @ Wq/Wk/Wv,
               compute_attention :250-314, x @ Wo, residual, RMSNorm, gated-SiLU FFN,
               residual); one decode token, root_node.py:739-1007 (the same with the decode
               attention block :900-933: RoPE at the cache length, KV append, clip, masked
               attention).
* ``greedy`` — Generator.generate at temperature 0 on token ids (generator.py:73-145):
               embedding rows of the f16 table as f32 (:38-39), the layers, final RMSNorm +
               logits against the f16 lm_head (:40-49), argmax (:51-53). The prompt is run
               unpadded; the reference pads it to seq_len and masks the padding, which gives
               the same numbers (causal attention, padding after the prompt).

The KV cache holds RoPE-rotated k and v unclipped, as the reference's concatenated arrays do;
clipping at use (elementwise, idempotent) gives the same attention either way.
"""
from __future__ import annotations

import numpy as np

from . import attention as OA
from . import kernels as K
from . import lmhead as OL


def layer(x: np.ndarray, lw: dict, cache: dict, n_heads: int, n_kv: int, head_dim: int, theta: float,
          eps: float = 1e-6, prefill: bool = False) -> np.ndarray:
    """x: f32 [S, H] (the prompt with prefill, else one token). lw: ln1, ln2, q, k, v, o, gate,
    up, down (f32, matrices [in, out]) and optionally q_bias, k_bias, v_bias (f32). cache: {"k": [1, n_kv, t, hd], "v": ...}, updated."""
    S = x.shape[0]
    xn = K.rms_norm(x, lw["ln1"], eps)
    q, k, v = (K.matmul_f32(xn, lw[n]) for n in ("q", "k", "v"))
    # optional f32 biases added right after the projections (root_node.py:443-451 prefill,
    # :786-799 head-partitioned decode)
    for t, n in ((q, "q_bias"), (k, "k_bias"), (v, "v_bias")):
        if lw.get(n) is not None:
            t += np.asarray(lw[n], np.float32).reshape(1, -1)
    q = q.reshape(1, S, n_heads, head_dim)
    k = k.reshape(1, S, n_kv, head_dim)
    v = v.reshape(1, S, n_kv, head_dim)
    if prefill:
        a = OA.compute_attention([(q, k, v)], n_heads, n_kv, 1.0, theta)[0]
        cache["k"] = K.apply_rope(np.ascontiguousarray(k.transpose(0, 2, 1, 3)), theta, 0, 1.0)
        cache["v"] = np.ascontiguousarray(v.transpose(0, 2, 1, 3))
    else:
        a, cache["k"], cache["v"] = OA.decode_step(np.ascontiguousarray(q.transpose(0, 2, 1, 3)),
                                                   np.ascontiguousarray(k.transpose(0, 2, 1, 3)),
                                                   np.ascontiguousarray(v.transpose(0, 2, 1, 3)),
                                                   cache["k"], cache["v"], 1.0, theta)
        a = a[0]
    h = x + K.matmul_f32(a, lw["o"])
    hn = K.rms_norm(h, lw["ln2"], eps)
    f = K.matmul_f32(K.silu_mul(K.matmul_f32(hn, lw["gate"]), K.matmul_f32(hn, lw["up"])), lw["down"])
    return (h + f).astype(np.float32)


def greedy(embedding_f16: np.ndarray, layers: list, final_norm: np.ndarray | None, prompt, n_tokens: int,
           n_heads: int, n_kv: int, head_dim: int, theta: float, eps: float = 1e-6, lm_head_f16=None,
           feed=None):
    """Greedy ids and the logits of every step, f32 [n_tokens, V]. The final norm is stored as
    f16 like the reference's (generator.py:34). feed: ids to run instead of the argmax from step
    1 on (teacher forcing, for comparing logits step by step); the returned ids stay the argmax."""
    table = embedding_f16 if lm_head_f16 is None else lm_head_f16
    fn = None if final_norm is None else np.asarray(final_norm).astype(np.float16)
    caches = [dict() for _ in layers]
    x = embedding_f16[np.asarray(prompt)].astype(np.float32)
    for lw, c in zip(layers, caches):
        x = layer(x, lw, c, n_heads, n_kv, head_dim, theta, eps, prefill=True)
    ids, logits = [], []
    for step in range(n_tokens):
        lg = OL.compute_logits(x[-1:], table, fn, eps)[0].astype(np.float32)
        logits.append(lg)
        ids.append(int(OL.greedy_token(lg[None])[0, 0]))
        if step + 1 == n_tokens:
            break
        nxt = ids[-1] if feed is None else int(feed[step])
        x = embedding_f16[[nxt]].astype(np.float32)
        for lw, c in zip(layers, caches):
            x = layer(x, lw, c, n_heads, n_kv, head_dim, theta, eps, prefill=False)
    return ids, np.stack(logits)
