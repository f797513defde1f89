"""Greedy-token parity with the reference on the seeded models of tests/golden/greedy_model.py.

tests/golden/greedy_golden*.npz hold the reference orchestrator's own runs (RootNode's
head-partitioned layers + Generator's prefill and greedy loop, src/orchestrator/
root_node.py:344-1007, generator.py:73-145): the prompt, the 32 greedy token ids, the logits
of the first step and the top-8 logits (ids and values) of every step. This runs the same
models on this library's kernels (pyre_b200.generator.Generator) through the default path —
the prompt as one pass (tensor-core GEMMs and attention for prompts longer than 4 tokens), then
the decode steps — and asks for the same 32 ids, and for every step's top-8 logits and the whole
first-step logit vector within LOGIT_ATOL (device differences: f16 KV cache, f16 operands in the
tensor-core prefill, other summation orders).

Models: SmolLM-135M shape (8-token prompt, projections N(0, 0.02)), reduced-layer Qwen2.5-0.5B
shape (QKV bias, 512-token prompt), reduced-layer Mistral-7B shape (untied lm_head, 512-token
prompt). The SmolLM-shaped N(0, 0.07) model is a separate case: its reference top-1/top-2 margin
at step 22 is 6.3e-3, below the logit error that storing K and V in f16 causes on its own
(7.7e-3 in an f32 CPU emulation with exact projections; the reference keeps f32), so whether
that step's token matches depends on rounding luck in either prefill form. That model runs
stepwise (every prompt token through the decode kernels) with all 32 tokens compared, and
through the default path teacher-forced (the reference's tokens fed back) with every step's
logits compared and the token compared at every step whose reference margin exceeds twice the
logit tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest

import greedy_device as G
from greedy_device import gm

LOGIT_ATOL = 2e-2
DECIDABLE = [m.name for m in gm.MODELS.values() if m.name != "smollm135m_std007"]


def test_golden_prompts_are_the_seeded_prompts():
    for m in gm.MODELS.values():
        g = G.golden(m)
        assert np.array_equal(g["prompt"], gm.prompt_ids(m)), m.name
        assert g["tokens"].shape == (gm.N_GREEDY,)
        assert g["top_idx"].shape == (gm.N_GREEDY, 8) and np.array_equal(g["top_idx"][:, 0], g["tokens"])


def _gen(name, persistent=False):
    import torch
    return G.generator(gm.MODELS[name], torch.device("cuda", 0), persistent=persistent)


def _check_run(g, ids, lg):
    d0 = np.abs(lg[0] - g["first_logits"]).max()
    assert d0 <= LOGIT_ATOL, f"first-step logits differ by {d0}"
    n_match = 0
    for step in range(gm.N_GREEDY):
        if ids[step] != int(g["tokens"][step]):
            break
        n_match += 1
        err = np.abs(lg[step][g["top_idx"][step]] - g["top_val"][step]).max()
        assert err <= LOGIT_ATOL, f"step {step}: top-8 logits differ by {err}"
    assert n_match == gm.N_GREEDY, f"tokens diverge at step {n_match}: {ids} vs {g['tokens'].tolist()}"


@pytest.mark.gpu
@pytest.mark.parametrize("name", DECIDABLE)
@pytest.mark.parametrize("mode", ["persistent", "decoder_step", "op_by_op"])
def test_greedy_tokens_match_reference(name, mode):
    """Default path: one-pass prefill, then decode steps (one native call per token: the
    persistent one-launch step or the launch-per-op step; or op by op from Python), with every
    step's logits."""
    g = G.golden(gm.MODELS[name])
    gen = _gen(name, persistent=mode == "persistent")
    assert gen.persistent == (mode == "persistent")
    ids, logits = gen.generate_ids(g["prompt"], gm.N_GREEDY, want_logits=True, native=mode != "op_by_op")
    _check_run(g, ids, logits.cpu().numpy())


@pytest.mark.gpu
@pytest.mark.parametrize("name", DECIDABLE)
@pytest.mark.parametrize("persistent", [True, False], ids=["persistent", "decoder_step"])
def test_greedy_tokens_graphed(name, persistent):
    """The benchmarked path: prefill replayed from a CUDA graph, decode steps replayed from
    CUDA graphs (position read and advanced on the device), twice in a row (the second run
    replays the cached graphs); then graphs of 5 steps over 16-position buckets, so the run
    crosses bucket boundaries and replans the attention grid."""
    g = G.golden(gm.MODELS[name])
    gen = _gen(name, persistent=persistent)
    for _ in range(2):
        assert gen.generate_ids(g["prompt"], gm.N_GREEDY, graphed=True) == g["tokens"].tolist()
    tok = gen.prefill(g["prompt"])
    hist = gen.decode_graphed(tok, gm.N_GREEDY - 1, steps_per_graph=5, bucket=16)
    n0 = len(g["prompt"])
    assert hist[n0:n0 + gm.N_GREEDY].cpu().tolist() == g["tokens"].tolist()


@pytest.mark.gpu
@pytest.mark.parametrize("native", [True, False], ids=["decoder_step", "op_by_op"])
def test_greedy_std07_stepwise_prompt(native):
    g = G.golden(gm.MODELS["smollm135m_std007"])
    gen = _gen("smollm135m_std007")
    ids, logits = gen.generate_ids(g["prompt"], gm.N_GREEDY, want_logits=True, native=native, stepwise_prefill=True)
    _check_run(g, ids, logits.cpu().numpy())
    assert gen.generate_ids(g["prompt"], gm.N_GREEDY, stepwise_prefill=True, graphed=True) == g["tokens"].tolist()


@pytest.mark.gpu
def test_greedy_std07_default_path_teacher_forced():
    """The default one-pass prefill on the N(0, 0.07) model with the reference's tokens fed
    back: every step's top-8 logits within LOGIT_ATOL, and the greedy token equal to the
    reference's wherever the reference's own top-1/top-2 margin exceeds 2 * LOGIT_ATOL."""
    import torch
    g = G.golden(gm.MODELS["smollm135m_std007"])
    gen = _gen("smollm135m_std007")
    tok, lg0 = gen.prefill(g["prompt"], want_logits=True)
    dev = gen.device
    feed = torch.tensor(g["tokens"], dtype=torch.int32, device=dev)
    out = torch.zeros(1, dtype=torch.int32, device=dev)
    logits = torch.empty((gm.N_GREEDY, gen.V), dtype=torch.float32, device=dev)
    logits[0].copy_(lg0[0])
    for step in range(1, gm.N_GREEDY):
        gen.step_into(feed[step - 1:step], out, logits[step])
    gen.check_status()
    lg = logits.cpu().numpy()
    margins = g["top_val"][:, 0] - g["top_val"][:, 1]
    checked = 0
    for step in range(gm.N_GREEDY):
        err = np.abs(lg[step][g["top_idx"][step]] - g["top_val"][step]).max()
        assert err <= LOGIT_ATOL, f"step {step}: top-8 logits differ by {err}"
        if margins[step] > 2 * LOGIT_ATOL:
            assert int(np.argmax(lg[step])) == int(g["tokens"][step]), f"step {step}"
            checked += 1
    assert checked >= 8
