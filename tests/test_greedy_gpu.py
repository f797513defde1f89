"""Greedy-token parity with the reference on the seeded SmolLM-135M-shaped model.

tests/golden/greedy_golden*.npz hold the reference orchestrator's own runs (RootNode's
head-partitioned layers + Generator's prefill and greedy loop, src/orchestrator/
root_node.py:344-1007, generator.py:73-145) on the weights of tests/golden/greedy_model.py
(projections N(0, 0.02), the configured model, and N(0, 0.07), whose greedy tokens all differ):
the 8-token prompt, the 32 greedy token ids, the logits of the first step and the top-8
logits (ids and values) of every step. This runs the same model on this library's kernels
(pyre_b200.generator.Generator) and asks for the same 32 ids, and for every step's top-8
logits and the whole first-step logit vector within LOGIT_ATOL (device differences: f16 KV
cache, f16 operands in the tensor-core prefill, other summation orders).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

import greedy_model as gm  # noqa: E402

from oracle.q80 import dequantize_q80, quantize_q80  # noqa: E402

LOGIT_ATOL = 2e-2


GOLDENS = sorted(gm.GOLDENS.items())


def _golden(name):
    return np.load(HERE / "golden" / name)


def _weights(std):
    """The model's weights as this library's Q8_0 matrices (the exact q and f16 scales whose
    dequantized values the reference ran on) plus the f16 embedding and final norm."""
    import torch
    from pyre_b200.quantizer import Q80Weight

    rec = []

    def roundtrip(a):
        q, s, shape = quantize_q80(a)
        s16 = s.astype(np.float16)
        rec.append((q.reshape(shape), s16.reshape(shape[0], shape[1] // 32)))
        return dequantize_q80(q, s16.astype(np.float32), shape)

    emb, layers, final_norm = gm.make_weights(roundtrip, std)
    names = ("q", "k", "v", "o", "gate", "up", "down")
    assert len(rec) == len(names) * len(layers)
    dev = torch.device("cuda", 0)
    out = []
    for i, lw in enumerate(layers):
        w = {n: Q80Weight(torch.from_numpy(rec[i * 7 + j][0]).to(dev), torch.from_numpy(rec[i * 7 + j][1]).to(dev))
             for j, n in enumerate(names)}
        out.append({"input_layernorm": lw["ln1"], "post_attention_layernorm": lw["ln2"],
                    "attn": {n: w[n] for n in ("q", "k", "v", "o")},
                    "ffn": {n: w[n] for n in ("gate", "up", "down")}})
    return emb, out, final_norm


@pytest.mark.parametrize("name,std", GOLDENS)
def test_golden_prompt_is_the_seeded_prompt(name, std):
    g = _golden(name)
    assert np.array_equal(g["prompt"], gm.prompt_ids())
    assert g["tokens"].shape == (gm.N_GREEDY,)
    assert g["top_idx"].shape == (gm.N_GREEDY, 8) and np.array_equal(g["top_idx"][:, 0], g["tokens"])


# (golden, projection std, decode steps through pyre_decoder_step, prompt fed stepwise).
# The N(0, 0.02) model (the configured one) runs its 8-token prompt as one tensor-core pass
# (f16 operands) and still matches all 32 tokens (measured top-8 logit error 1.8e-3 against a
# smallest top-1/top-2 margin of 3.4e-3). On the N(0, 0.07) model small differences grow over
# the 30 layers and its reference margins go down to 4.1e-3, below the f16 prefill's error
# there (1.0e-2), so it feeds the prompt through the decode kernels (f32 projections and
# FFN, f16 KV cache): measured top-8 error 7.4e-3 and all 32 tokens equal.
CASES = [("greedy_golden.npz", 0.02, True, False), ("greedy_golden.npz", 0.02, False, False),
         ("greedy_golden.npz", 0.02, True, True), ("greedy_golden_std07.npz", 0.07, True, True),
         ("greedy_golden_std07.npz", 0.07, False, True)]


def _generator(std):
    import torch
    from pyre_b200.generator import Generator
    emb, layers, final_norm = _weights(std)
    C = gm.CFG
    return Generator(layers, emb, final_norm, n_heads=C["n_heads"], n_kv_heads=C["n_kv"], head_dim=C["head_dim"],
                     rope_theta=C["theta"], eps=C["eps"], max_seq=128, max_prompt=64, device=torch.device("cuda", 0))


@pytest.mark.gpu
@pytest.mark.parametrize("name,std,stepwise", [("greedy_golden.npz", 0.02, False), ("greedy_golden_std07.npz", 0.07, True)])
def test_greedy_tokens_graphed_decode(name, std, stepwise):
    """Decode steps replayed from captured CUDA graphs (position read and advanced on the
    device), with graphs of 5 steps over 16-position buckets so that the run crosses bucket
    boundaries and replans the attention grid: the same 32 tokens, twice in a row (the
    second run replays the cached graphs)."""
    g = _golden(name)
    gen = _generator(std)
    for _ in range(2):
        ids = gen.generate_ids(g["prompt"], gm.N_GREEDY, stepwise_prefill=stepwise, graphed=True)
        assert ids == g["tokens"].tolist()
    tok = gen.prefill(g["prompt"], stepwise=stepwise)
    hist = gen.decode_graphed(tok, gm.N_GREEDY - 1, steps_per_graph=5, bucket=16)
    n0 = len(g["prompt"])
    assert hist[n0:n0 + gm.N_GREEDY].cpu().tolist() == g["tokens"].tolist()


@pytest.mark.gpu
@pytest.mark.parametrize("name,std,native,stepwise", CASES)
def test_greedy_tokens_match_reference(name, std, native, stepwise):
    g = _golden(name)
    gen = _generator(std)
    ids, logits = gen.generate_ids(g["prompt"], gm.N_GREEDY, want_logits=True, native=native,
                                   stepwise_prefill=stepwise)
    lg = logits.cpu().numpy()
    # logits first: a mismatch there says where the tokens would start to differ
    d0 = np.abs(lg[0] - g["first_logits"]).max()
    assert d0 <= LOGIT_ATOL, f"first-step logits differ by {d0}"
    n_match = 0
    for step in range(gm.N_GREEDY):
        if ids[step] != int(g["tokens"][step]):
            break
        n_match += 1
        got = lg[step][g["top_idx"][step]]
        err = np.abs(got - g["top_val"][step]).max()
        assert err <= LOGIT_ATOL, f"step {step}: top-8 logits differ by {err}"
    assert n_match == gm.N_GREEDY, f"tokens diverge at step {n_match}: {ids} vs {g['tokens'].tolist()}"
