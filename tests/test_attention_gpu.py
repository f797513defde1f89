"""Attention-path kernels on the GPU against the attention oracle (oracle/attention.py,
oracle/kernels.py), which is pinned to the reference's own code by tests/test_attention_oracle.py.

Tolerances (max |out - ref| / max |ref|): RMSNorm and softmax 1e-6 (f32 / f64 arithmetic like
the reference); the Q8_0 projections 1e-4 (f32 path, T <= 4) and 1e-2 (f16 tensor-core path);
RoPE + clip 2e-3 (the rotated values are stored as f16); attention 5e-3 (f16 q/k/v and
probabilities, f32 accumulation). The path's budget is 2e-2.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import attention as OA
from oracle import kernels as OK
from oracle import q80 as oq80

pytestmark = pytest.mark.gpu

TOL_ATTN = 5e-3


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def test_rms_norm_and_softmax():
    from pyre_b200.attention import rms_norm, softmax
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((7, 4096)) * 3).astype(np.float32)
    w = rng.standard_normal(4096).astype(np.float32)
    got = rms_norm(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()).cpu().numpy()
    assert rel(got, OK.rms_norm(x, w)) < 1e-6
    s = (rng.standard_normal((5, 37, 129)) * 4).astype(np.float32)
    s[0, 0, 5:] = -np.inf
    got = softmax(torch.from_numpy(s).cuda()).cpu().numpy()
    assert rel(got, OK.softmax(s)) < 1e-6


@pytest.mark.parametrize("T", [1, 3, 37])
def test_q80_linear(T):
    from pyre_b200.attention import Q80Linear
    from pyre_b200.quantizer import Q80Weight
    rng = np.random.default_rng(T)
    w = (rng.standard_normal((576, 384)) * 0.05).astype(np.float32)
    q, s, sh = oq80.quantize_q80(w)
    s = s.astype(np.float16).astype(np.float32)
    wd = oq80.dequantize_q80(q, s, sh)
    lin = Q80Linear(Q80Weight.from_tuple(("q8", q, s, sh), scale_dtype=torch.float16), max_tokens=T)
    x = rng.standard_normal((T, 576)).astype(np.float32)
    out = lin(torch.from_numpy(x).cuda()).cpu().numpy()
    ref = x.astype(np.float64) @ wd.astype(np.float64)
    assert rel(out, ref) < (1e-4 if T <= 4 else 1e-2)


# Projection shapes of the decode step: SmolLM QKV (K 576, N 960), Qwen QKV (896, 1152, 4.5
# slabs), 7B QKV and O (4096, 6144 / 4096), a tensor-parallel QKV (4096, 1024), a K at the
# cluster kernel's limit (8192) and one beyond it (14336, streaming kernel); f32 and bf16
# activations, f16 and f32 scales, with and without the bias.
@pytest.mark.parametrize("K,N,T,xbf16,s32,bias", [
    (576, 960, 1, False, False, True), (896, 1152, 3, False, False, True), (4096, 6144, 1, False, False, False),
    (4096, 4096, 4, True, False, False), (4096, 1024, 2, False, True, True), (8192, 512, 1, False, False, True),
    (14336, 4096, 1, False, False, True), (64, 32, 4, False, False, True)])
def test_q80_linear_decode_shapes(K, N, T, xbf16, s32, bias):
    from pyre_b200.attention import Q80Linear
    from pyre_b200.quantizer import Q80Weight
    rng = np.random.default_rng(K + N + T)
    w = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    q, sc, sh = oq80.quantize_q80(w)
    if not s32:
        sc = sc.astype(np.float16).astype(np.float32)
    wd = oq80.dequantize_q80(q, sc, sh)
    b = (rng.standard_normal(N) * 0.5).astype(np.float32) if bias else None
    lin = Q80Linear(Q80Weight.from_tuple(("q8", q, sc, sh), scale_dtype=torch.float32 if s32 else torch.float16),
                    max_tokens=T, bias=b)
    x = rng.standard_normal((T, K)).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    if xbf16:
        xt = xt.to(torch.bfloat16)
        x = xt.float().cpu().numpy()
    ref = x.astype(np.float64) @ wd.astype(np.float64) + (b.astype(np.float64) if bias else 0.0)
    for _ in range(2):          # repeated calls reuse the scratch
        out = lin(xt).cpu().numpy()
        assert rel(out, ref) < 1e-4
    torch.cuda.synchronize()
    assert int(lin.workspace[8:12].view(torch.int32).item()) == 0


def _qkv(rng, T, nq, nkv, hd, scale=2.0):
    q = (rng.standard_normal((T, nq * hd)) * scale).astype(np.float32)
    k = (rng.standard_normal((T, nkv * hd)) * scale).astype(np.float32)
    v = (rng.standard_normal((T, nkv * hd)) * scale).astype(np.float32)
    return q, k, v


def _as4(x, T, n, hd):
    return x.reshape(1, T, n, hd)


@pytest.mark.parametrize("T,nq,nkv,hd,frac,theta", [(70, 8, 2, 64, 1.0, 1e4), (130, 4, 4, 128, 1.0, 1e6),
                                                     (200, 32, 8, 128, 1.0, 5e5), (65, 6, 2, 64, 0.5, 1e4),
                                                     (1000, 8, 2, 128, 1.0, 1e6), (2048, 4, 1, 64, 1.0, 5e5),
                                                     (1, 4, 2, 128, 1.0, 1e4), (129, 2, 2, 128, 1.0, 1e4)])
def test_prefill_attention_vs_oracle(T, nq, nkv, hd, frac, theta):
    from pyre_b200.attention import AttentionOp
    rng = np.random.default_rng(T + nq)
    q, k, v = _qkv(rng, T, nq, nkv, hd)
    op = AttentionOp(nq, nkv, hd, max_t=T + 8, rope_theta=theta, rope_fraction=frac)
    out = op.prefill(*(torch.from_numpy(a).cuda() for a in (q, k, v))).cpu().numpy()
    ref = OA.compute_attention([(_as4(q, T, nq, hd), _as4(k, T, nkv, hd), _as4(v, T, nkv, hd))], nq, nkv, frac, theta)
    assert rel(out, ref[0]) < TOL_ATTN
    # the cache holds the rotated, clipped keys (f16)
    kr = np.clip(OK.apply_rope(_as4(k, T, nkv, hd).transpose(0, 2, 1, 3), theta, 0, frac), -1000, 1000)[0]
    assert rel(op.cache.k[:, :T].float().cpu().numpy(), kr) < 2e-3
    from pyre_b200 import _native as N
    st = ctypes.c_int(-1)
    N.call("pyre_attn_status", ctypes.byref(st))
    assert st.value == 0      # no bounded pipeline wait of the tensor-core kernel ran out


def test_prefill_golden_cases():
    """The reference's own prefill attention cases (sequence- and head-concatenated nodes)."""
    from pyre_b200.attention import AttentionOp
    z = np.load(GOLDEN / "attn_golden.npz")
    _, nq, nkv, hd, _ = (int(v) for v in z["proj__dims"])
    for name in ("seq_rope1", "head_rope1"):
        by_head = bool(z[f"{name}__cfg"][0])
        axis = 2 if by_head else 1
        q, k, v = (np.concatenate([z[f"{name}__n{i}_{t}"] for i in range(2)], axis=axis) for t in "qkv")
        T = q.shape[1]
        # The golden heads have hd = 16; the kernels take 64 or 128. Zero-pad each head to 64:
        # rope_fraction 16/64 rotates exactly the pairs (i, i + 8), i < 8, with the golden's
        # freq_i = 1 / theta^(2i/16); padded dims add nothing to q.k or to the output, and q is
        # doubled so that 1/sqrt(64) scales the scores like the golden's 1/sqrt(16).
        pad = 64 - hd
        op = AttentionOp(nq, nkv, 64, max_t=T, rope_theta=10000.0, rope_fraction=float(hd) / 64.0)
        qp, kp, vp = (np.concatenate([a, np.zeros(a.shape[:-1] + (pad,), np.float32)], axis=-1) for a in (q, k, v))
        qp = qp * 2.0
        out = op.prefill(*(torch.from_numpy(np.ascontiguousarray(a.reshape(T, -1))).cuda() for a in (qp, kp, vp)))
        out = out.cpu().numpy()
        out = out.reshape(T, nq, 64)[:, :, :hd].reshape(T, nq * hd)
        assert rel(out, z[f"{name}__attn"][0]) < TOL_ATTN, name


@pytest.mark.parametrize("nq,nkv,hd,t0", [(8, 2, 64, 37), (32, 8, 128, 300), (4, 4, 128, 1)])
def test_decode_steps_vs_oracle(nq, nkv, hd, t0):
    """Prefill t0 tokens, then decode 4 tokens one by one; each step equals the oracle's
    decode step on the same cache."""
    from pyre_b200.attention import AttentionOp
    rng = np.random.default_rng(nq * hd + t0)
    op = AttentionOp(nq, nkv, hd, max_t=t0 + 8, rope_theta=1e6)
    q, k, v = _qkv(rng, t0, nq, nkv, hd)
    op.prefill(*(torch.from_numpy(a).cuda() for a in (q, k, v)))
    kc = np.clip(OK.apply_rope(_as4(k, t0, nkv, hd).transpose(0, 2, 1, 3), 1e6, 0, 1.0), -1000, 1000)
    vc = np.clip(_as4(v, t0, nkv, hd).transpose(0, 2, 1, 3), -1000, 1000)
    for step in range(4):
        qn, kn, vn = _qkv(rng, 1, nq, nkv, hd)
        out = op.decode(*(torch.from_numpy(a).cuda() for a in (qn, kn, vn))).cpu().numpy()
        ref, kc, vc = OA.decode_step(qn.reshape(1, nq, 1, hd), kn.reshape(1, nkv, 1, hd), vn.reshape(1, nkv, 1, hd),
                                     kc, vc, 1.0, 1e6)
        assert rel(out, ref[0]) < TOL_ATTN, step


def test_decode_padding_mask_golden():
    """The reference's decode case with a padded prefill (positions 5..7 masked)."""
    from pyre_b200 import _device as D, _native as N
    z = np.load(GOLDEN / "attn_golden.npz")
    q, k, v = z["decode__q"], z["decode__k"], z["decode__v"]
    lo, hi = (int(x) for x in z["decode__mask"])
    nq, nkv, t, hd = q.shape[1], k.shape[1], k.shape[2], q.shape[3]
    pad = 64 - hd   # dot products and weighted sums are unchanged by zero padding of hd
    qh = torch.from_numpy(np.pad(q[0, :, 0], ((0, 0), (0, pad)))).cuda().half().contiguous()
    kh = torch.from_numpy(np.pad(k[0], ((0, 0), (0, 0), (0, pad)))).cuda().half().contiguous()
    vh = torch.from_numpy(np.pad(v[0], ((0, 0), (0, 0), (0, pad)))).cuda().half().contiguous()
    b = ctypes.c_int64(0)
    N.call("pyre_attn_decode_workspace_bytes", nq, nkv, 64, t, ctypes.byref(b))
    ws = torch.zeros(b.value, dtype=torch.uint8, device="cuda")
    out = torch.empty(nq * 64, device="cuda")
    # the golden's scale is 1/sqrt(16): scale q by sqrt(64)/sqrt(16) so 1/sqrt(64) gives the same
    qh = (qh.float() * 2.0).half()
    N.call("pyre_attn_decode", D.ptr(qh), D.ptr(kh), D.ptr(vh), t, nq, nkv, 64, t, lo, hi, D.ptr(out), D.ptr(ws),
           ws.numel(), D.stream_ptr())
    got = out.reshape(nq, 64)[:, :hd].reshape(-1).cpu().numpy()
    assert rel(got, z["decode__attn"][0, 0]) < TOL_ATTN


@pytest.mark.parametrize("nq,nkv,hd,t", [(32, 8, 128, 2175), (16, 2, 128, 9000), (8, 8, 64, 5000), (14, 2, 64, 700), (8, 1, 128, 40000)])
def test_decode_long_cache(nq, nkv, hd, t):
    """Split decode over long caches (cluster and cross-cluster partial combines, GQA groups
    of 1..8 heads) against the oracle's attention_decode on the same f16 cache."""
    from pyre_b200 import _device as D, _native as N
    rng = np.random.default_rng(t + nq)
    q = (rng.standard_normal((nq, hd)) * 2).astype(np.float16)
    k = (rng.standard_normal((nkv, t, hd)) * 2).astype(np.float16)
    v = (rng.standard_normal((nkv, t, hd)) * 2).astype(np.float16)
    b = ctypes.c_int64(0)
    N.call("pyre_attn_decode_workspace_bytes", nq, nkv, hd, t, ctypes.byref(b))
    ws = torch.zeros(b.value, dtype=torch.uint8, device="cuda")
    qh, kh, vh = (torch.from_numpy(a).cuda() for a in (q, k, v))
    out = torch.empty(nq * hd, device="cuda")
    ref = OA.attention_decode(q.astype(np.float32).reshape(1, nq, 1, hd), k.astype(np.float32)[None],
                              v.astype(np.float32)[None])[0, 0]
    for _ in range(2):     # the workspace's arrival counters are left at zero for the next call
        N.call("pyre_attn_decode", D.ptr(qh), D.ptr(kh), D.ptr(vh), t, nq, nkv, hd, t, 0, 0, D.ptr(out), D.ptr(ws),
               ws.numel(), D.stream_ptr())
        assert rel(out.cpu().numpy(), ref) < TOL_ATTN


@pytest.mark.parametrize("hd,frac,t0", [(128, 1.0, 3000), (64, 0.5, 40), (128, 0.0, 7000)])
def test_decode_step_fused_equals_rope_then_attention(hd, frac, t0):
    """pyre_attn_decode_step (RoPE + clip + append + attention in one launch) against
    pyre_rope_kv_append followed by pyre_attn_decode on a copy of the same cache, with a
    masked range."""
    from pyre_b200 import _device as D, _native as N
    from pyre_b200.attention.ops import rope_table
    nq, nkv, max_t = 16, 4, t0 + 4
    rng = np.random.default_rng(hd + t0)
    kc = torch.from_numpy((rng.standard_normal((nkv, max_t, hd)) * 2).astype(np.float16)).cuda()
    vc = torch.from_numpy((rng.standard_normal((nkv, max_t, hd)) * 2).astype(np.float16)).cuda()
    kc2, vc2 = kc.clone(), vc.clone()
    q, k, v = (torch.from_numpy((rng.standard_normal((1, n * hd)) * 3).astype(np.float32)).cuda()
               for n in (nq, nkv, nkv))
    tab = rope_table(1e6, frac, hd, max_t, kc.device)
    b = ctypes.c_int64(0)
    N.call("pyre_attn_decode_workspace_bytes", nq, nkv, hd, max_t, ctypes.byref(b))
    ws = torch.zeros(b.value, dtype=torch.uint8, device="cuda")
    out = torch.empty(nq * hd, device="cuda")
    N.call("pyre_attn_decode_step", D.ptr(q), D.ptr(k), D.ptr(v), t0, D.ptr(tab), frac, nq, nkv, hd, D.ptr(kc),
           D.ptr(vc), max_t, 5, 9, D.ptr(out), D.ptr(ws), ws.numel(), D.stream_ptr())
    q_out = torch.empty((nq, 1, hd), dtype=torch.float16, device="cuda")
    N.call("pyre_rope_kv_append", D.ptr(q), D.ptr(k), D.ptr(v), q.stride(0), k.stride(0), 1, nq, nkv, hd, t0,
           D.ptr(tab), frac, D.ptr(q_out), D.ptr(kc2), D.ptr(vc2), max_t, D.stream_ptr())
    out2 = torch.empty(nq * hd, device="cuda")
    N.call("pyre_attn_decode", D.ptr(q_out), D.ptr(kc2), D.ptr(vc2), t0 + 1, nq, nkv, hd, max_t, 5, 9, D.ptr(out2),
           D.ptr(ws), ws.numel(), D.stream_ptr())
    assert torch.equal(kc[:, :t0 + 1], kc2[:, :t0 + 1]) and torch.equal(vc[:, :t0 + 1], vc2[:, :t0 + 1])
    assert torch.equal(out, out2)


def test_ulysses_builder_projection():
    """build_ulysses_attention_graph through the session, on the reference's golden shards."""
    from pyre_b200.attention import ShardSpec, build_ulysses_attention_graph
    from pyre_b200.engine import DeviceRef, InferenceSession
    z = np.load(GOLDEN / "attn_golden.npz")
    H, nq, nkv, hd, S = (int(v) for v in z["proj__dims"])
    for i, (a, b) in enumerate(((0, 6), (6, 10))):
        g = build_ulysses_attention_graph(ShardSpec(0, nq * hd, a, b, nq, nkv, 0, 0), H, nq, nkv, hd,
                                          DeviceRef.GPU(0), full_q_weights=True)
        q, k, v = InferenceSession().load(g).execute(np.ascontiguousarray(z["proj__x"][:, a:b]), z["proj__wq"],
                                                     z["proj__wk"], z["proj__wv"])
        for t, got in zip("qkv", (q, k, v)):
            ref = z[f"proj{i}__{t}"]
            assert got.shape == ref.shape
            # weights go through Q8_0 (as on a reference worker): budget 2e-2
            assert rel(got.to_numpy(), ref) < 2e-2
