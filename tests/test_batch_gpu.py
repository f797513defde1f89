"""Static-batch decode (B equally long prompts decoded in lockstep, Generator.generate_batch)
against one-sequence decoding on the same weights: the reduced-layer Mistral-7B-shaped golden
model with B = 4 (one row group) and B = 8 (two row groups of the projections and the FFN), the
golden prompt among random ones. Every sequence's tokens and logits must equal those of a
batch-1 run bit for bit (the batched kernels keep each sequence's arithmetic: the Q8_0 GEMV
accumulates each token alone and sums the splits as exact integers, the batched attention splits
each cache as a one-sequence step does), and the golden prompt's tokens must be the reference's.
"""
import numpy as np
import pytest
import torch

import greedy_device as G
from greedy_device import gm

pytestmark = pytest.mark.gpu

N_TOK = 16


@pytest.fixture(scope="module")
def weights():
    m = gm.MODELS["mistral7b_l2"]
    return m, G.device_weights(m, torch.device("cuda", 0))


def _gen(m, w, batch):
    from pyre_b200.generator import Generator
    emb, layers, fn, head = w
    return Generator(layers, emb, fn, n_heads=m.n_heads, n_kv_heads=m.n_kv, head_dim=m.head_dim, rope_theta=m.theta,
                     eps=m.eps, lm_head=head, max_seq=m.prompt_len + gm.N_GREEDY + 16, max_prompt=m.prompt_len,
                     device=torch.device("cuda", 0), batch=batch)


def _prompts(m, B):
    rng = np.random.default_rng(99)
    ps = rng.integers(0, m.vocab, (B, m.prompt_len))
    ps[1] = gm.prompt_ids(m)
    return ps


@pytest.mark.parametrize("B", [4, 8])
def test_batch_equals_single_sequences(weights, B):
    m, w = weights
    prompts = _prompts(m, B)
    single = _gen(m, w, 1)
    ref_ids, ref_lg = [], []
    for b in range(B):
        ids, lg = single.generate_ids(prompts[b], N_TOK, want_logits=True)
        ref_ids.append(ids)
        ref_lg.append(lg.cpu())
    del single
    gen = _gen(m, w, B)
    ids, lg = gen.generate_batch(prompts, N_TOK, want_logits=True, graphed=False)
    lg = lg.cpu()
    for b in range(B):
        assert ids[b] == ref_ids[b], b
        assert torch.equal(lg[:, b], ref_lg[b]), b
    assert gen.generate_batch(prompts, N_TOK) == ref_ids          # graphed decode
    want = G.golden(m)["tokens"][:N_TOK].tolist()
    assert ids[1] == want
