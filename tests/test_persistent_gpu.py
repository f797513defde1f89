"""The persistent decode step (every layer of a token in one launch, pyre_decoder_step_persistent)
against the launch-per-op decode step (pyre_decoder_step) on the same weights and the same
teacher-forced tokens.

Both run the reference's decode layer (RootNode._decode_single_layer, src/orchestrator/
root_node.py:739-1007) with the same Q8_0 weights, f16 KV cache and f32 activations; they differ
only in summation order (split-K partials, attention splits, f32 instead of f16 attention
probabilities in the weighted sum of values), so their logits agree to ~1e-4 of the logit scale
and the greedy tokens agree wherever the top-2 margin is not a near tie. Shapes cover head_dim
64 and 128, 1 to 4 query heads per kv head, QKV bias, prompts whose caches span many attention
splits with one and with several 32-position tiles per split, and more layers than the ring
holds stages for. Greedy-token parity with the reference's goldens on the persistent path is in
tests/test_greedy_gpu.py.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# name: (H, nq, nkv, hd, W, layers, vocab, bias, prompt, theta)
SHAPES = {
    "hd64_rep4_bias": (512, 8, 2, 64, 1024, 3, 1000, True, 100, 1e4),
    "hd128_rep4_long": (1024, 8, 2, 128, 2048, 2, 2000, False, 700, 1e6),
    "hd128_nkv8_multitile": (1024, 32, 8, 128, 1536, 2, 1500, False, 1000, 5e5),
    "hd64_rep7_qwenlike": (896, 14, 2, 64, 1152, 4, 3000, True, 300, 1e6),
}
N_STEPS = 24


def _weights(shape, dev):
    from pyre_b200.quantizer import Q80Weight
    H, nq, nkv, hd, W, n_layers, V, bias, _, _ = shape
    g = torch.Generator(device=dev).manual_seed(11)

    def w(k, n, std=0.05):
        return Q80Weight.from_float((torch.randn((k, n), generator=g, device=dev) * std).to(torch.bfloat16).float(),
                                    torch.float16)

    def norm():
        return 1.0 + 0.1 * torch.randn(H, generator=g, device=dev)

    layers = []
    for _ in range(n_layers):
        attn = {"q": w(H, nq * hd), "k": w(H, nkv * hd), "v": w(H, nkv * hd), "o": w(nq * hd, H)}
        if bias:
            attn["q_bias"] = 0.05 * torch.randn(nq * hd, generator=g, device=dev)
            attn["k_bias"] = 0.05 * torch.randn(nkv * hd, generator=g, device=dev)
            attn["v_bias"] = 0.05 * torch.randn(nkv * hd, generator=g, device=dev)
        layers.append({"input_layernorm": norm(), "post_attention_layernorm": norm(), "attn": attn,
                       "ffn": {"gate": w(H, W), "up": w(H, W), "down": w(W, H)}})
    emb = (torch.randn((V, H), generator=g, device=dev) * 0.5).half()
    return layers, emb, norm()


def _gen(shape, w, persistent, dev):
    from pyre_b200.generator import Generator
    H, nq, nkv, hd, W, n_layers, V, bias, prompt, theta = shape
    layers, emb, fn = w
    return Generator(layers, emb, fn, n_heads=nq, n_kv_heads=nkv, head_dim=hd, rope_theta=theta, eps=1e-6,
                     max_seq=prompt + N_STEPS + 8, max_prompt=prompt, device=dev, persistent=persistent)


@pytest.mark.parametrize("name", list(SHAPES))
def test_persistent_equals_per_op_decode(name):
    dev = torch.device("cuda", 0)
    shape = SHAPES[name]
    w = _weights(shape, dev)
    a, b = _gen(shape, w, False, dev), _gen(shape, w, True, dev)
    assert b.persistent and not a.persistent
    V, prompt = shape[6], shape[8]
    rng = np.random.default_rng(5)
    ids = rng.integers(0, V, prompt)
    feed = torch.tensor(rng.integers(0, V, N_STEPS), dtype=torch.int32, device=dev)
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    la = torch.empty((N_STEPS, V), dtype=torch.float32, device=dev)
    lb = torch.empty_like(la)
    for gen, lg in ((a, la), (b, lb)):
        gen.prefill(ids)
        for i in range(N_STEPS):
            gen.step_into(feed[i:i + 1], out, lg[i])
        gen.check_status()
    la, lb = la.cpu().numpy(), lb.cpu().numpy()
    scale = np.abs(la).max()
    err = np.abs(la - lb).max() / scale
    assert err < 2e-3, f"persistent vs per-op logits differ by {err:.3e} of the logit scale"
    # the greedy token agrees wherever the per-op run's top-2 margin is not a near tie
    top2 = np.sort(la, axis=1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 1e-2 * scale
    assert clear.sum() >= N_STEPS // 2
    assert np.array_equal(la.argmax(1)[clear], lb.argmax(1)[clear])


def test_persistent_graphed_equals_per_call():
    """The persistent step replayed from CUDA graphs (position on the device) gives the tokens of
    the persistent step called once per token, across graph and bucket boundaries."""
    dev = torch.device("cuda", 0)
    shape = SHAPES["hd128_rep4_long"]
    w = _weights(shape, dev)
    gen = _gen(shape, w, True, dev)
    ids = np.random.default_rng(7).integers(0, shape[6], shape[8])
    ref = gen.generate_ids(ids, N_STEPS)
    assert gen.generate_ids(ids, N_STEPS, graphed=True) == ref
    tok = gen.prefill(ids)
    hist = gen.decode_graphed(tok, N_STEPS - 1, steps_per_graph=5, bucket=16)
    n0 = len(ids)
    assert hist[n0:n0 + N_STEPS].cpu().tolist() == ref


def test_persistent_workspace_reused():
    """Repeated generations on one workspace (the kernel leaves counters, accumulators and the
    queue ready for the next call; flags are tagged with the call's epoch) give the same tokens."""
    dev = torch.device("cuda", 0)
    shape = SHAPES["hd64_rep4_bias"]
    gen = _gen(shape, _weights(shape, dev), True, dev)
    ids = np.random.default_rng(9).integers(0, shape[6], shape[8])
    first = gen.generate_ids(ids, N_STEPS, graphed=True)
    for _ in range(3):
        assert gen.generate_ids(ids, N_STEPS, graphed=True) == first
    import ctypes
    from pyre_b200 import _native as N
    v = ctypes.c_int(-1)
    N.call("pyre_decoder_persistent_status", ctypes.c_void_p(gen._pws.data_ptr()), ctypes.byref(v))
    assert v.value == 0
