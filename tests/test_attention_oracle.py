"""The attention oracle (oracle/attention.py) against the reference's own attention code run
in this container (tests/golden/attn_golden.npz, written by tests/golden/make_golden.py):
the Ulysses QKV projection graph, the prefill attention of RootNode._compute_attention
(sequence- and head-concatenated nodes, RoPE fractions, v-norm) and the decode attention with
a padded prefill. Bit-exact."""
import numpy as np

from conftest import GOLDEN
from oracle import attention as OA


def test_qkv_projection_golden():
    z = np.load(GOLDEN / "attn_golden.npz")
    H, nq, nkv, hd, S = (int(v) for v in z["proj__dims"])
    for i, (a, b) in enumerate(((0, 6), (6, 10))):
        q, k, v = OA.qkv_projection(z["proj__x"][:, a:b], z["proj__wq"], z["proj__wk"], z["proj__wv"], nq, nkv, hd)
        assert np.array_equal(q, z[f"proj{i}__q"])
        assert np.array_equal(k, z[f"proj{i}__k"])
        assert np.array_equal(v, z[f"proj{i}__v"])


def test_prefill_attention_golden():
    z = np.load(GOLDEN / "attn_golden.npz")
    _, nq, nkv, _, _ = (int(v) for v in z["proj__dims"])
    for name in ("seq_rope1", "seq_rope05_vnorm", "head_rope1"):
        by_head, vn = (bool(v) for v in z[f"{name}__cfg"])
        parts = [tuple(z[f"{name}__n{i}_{t}"] for t in "qkv") for i in range(2)]
        got = OA.compute_attention(parts, nq, nkv, float(z[f"{name}__frac"]), 10000.0, vn, by_head)
        assert np.array_equal(got, z[f"{name}__attn"]), name


def test_decode_attention_golden():
    z = np.load(GOLDEN / "attn_golden.npz")
    lo, hi = (int(v) for v in z["decode__mask"])
    got = OA.attention_decode(z["decode__q"], z["decode__k"], z["decode__v"], lo, hi)
    assert np.array_equal(got, z["decode__attn"])


def test_decode_step_matches_prefill_rows():
    """Decoding token by token over a growing cache equals the last rows of the causal
    prefill attention on the same q, k, v (RoPE at the token's position in both)."""
    rng = np.random.default_rng(5)
    nq, nkv, hd, S = 4, 2, 8, 7
    q = (rng.standard_normal((1, S, nq, hd)) * 2).astype(np.float32)
    k = (rng.standard_normal((1, S, nkv, hd)) * 2).astype(np.float32)
    v = (rng.standard_normal((1, S, nkv, hd)) * 2).astype(np.float32)
    full = OA.compute_attention([(q, k, v)], nq, nkv, 1.0, 10000.0)
    kc = vc = None
    for s in range(S):
        out, kc, vc = OA.decode_step(q[:, s:s + 1].transpose(0, 2, 1, 3), k[:, s:s + 1].transpose(0, 2, 1, 3),
                                     v[:, s:s + 1].transpose(0, 2, 1, 3), kc, vc)
        np.testing.assert_allclose(out[0, 0], full[0, s], rtol=1e-5, atol=1e-5)


def test_attention_rows_f64_equals_full_oracle():
    """The row-wise f64 restatement used for the 32768-token check equals the full-matrix
    oracle (compute_attention, itself pinned to the reference's goldens) on sampled rows."""
    import numpy as np
    from oracle import attention as OA
    rng = np.random.default_rng(1)
    S, nq, nkv, hd = 200, 8, 2, 64
    q, k, v = (rng.standard_normal((S, n * hd)).astype(np.float32) * 3 for n in (nq, nkv, nkv))
    ref = OA.compute_attention([(q.reshape(1, S, nq, hd), k.reshape(1, S, nkv, hd), v.reshape(1, S, nkv, hd))],
                               nq, nkv, 1.0, 5e5)[0]
    pos, hs = rng.integers(0, S, 64), rng.integers(0, nq, 64)
    rows = OA.attention_rows_f64(q, k, v, pos, hs, nq, nkv, 5e5)
    want = np.stack([ref[p, h * hd:(h + 1) * hd] for p, h in zip(pos, hs)])
    assert np.abs(rows - want).max() <= 1e-5 * np.abs(want).max()
