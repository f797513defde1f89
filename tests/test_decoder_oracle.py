"""The oracle's whole-decoder greedy loop (oracle/decoder.py) against the reference
orchestrator's own runs (tests/golden/greedy_golden*.npz): the same 32 greedy ids and every
step's top-8 logits within 1e-4 (both are f32 numpy; the reference ran the prompt padded to 64
positions, which changes only the blocking of its matrix products)."""
import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

import greedy_model as gm  # noqa: E402

from oracle import decoder as OD  # noqa: E402
from oracle.q80 import q80_roundtrip  # noqa: E402


@pytest.mark.parametrize("name,std", sorted(gm.GOLDENS.items()))
def test_oracle_decoder_equals_reference_goldens(name, std):
    g = np.load(HERE / "golden" / name)
    emb, layers, final_norm = gm.make_weights(lambda a: q80_roundtrip(a, np.float16), std)
    C = gm.CFG
    ids, logits = OD.greedy(emb, layers, final_norm, g["prompt"], gm.N_GREEDY, C["n_heads"], C["n_kv"],
                            C["head_dim"], C["theta"], C["eps"])
    assert ids == g["tokens"].tolist()
    np.testing.assert_allclose(logits[0], g["first_logits"], rtol=0, atol=1e-4)
    for step in range(gm.N_GREEDY):
        np.testing.assert_allclose(logits[step][g["top_idx"][step]], g["top_val"][step], rtol=0, atol=1e-4)


@pytest.mark.parametrize("name,steps", [("qwen05b_l4", 8), ("mistral7b_l2", 4)])
def test_oracle_decoder_equals_reference_wide_models(name, steps):
    """The reduced-layer Qwen2.5-0.5B-shaped (QKV bias, tied 151936 vocabulary) and Mistral-7B-
    shaped (untied lm_head) models with 512-token prompts: the oracle's first greedy steps equal
    the reference's tokens and top-8 logits (the first steps keep the CPU time bounded)."""
    m = gm.MODELS[name]
    g = np.load(HERE / "golden" / m.fixture)
    emb, layers, final_norm, head = gm.build(m, lambda a: q80_roundtrip(a, np.float16))
    ids, logits = OD.greedy(emb, layers, final_norm, g["prompt"], steps, m.n_heads, m.n_kv, m.head_dim, m.theta,
                            m.eps, lm_head_f16=head)
    assert ids == g["tokens"][:steps].tolist()
    np.testing.assert_allclose(logits[0], g["first_logits"], rtol=0, atol=1e-4)
    for step in range(steps):
        np.testing.assert_allclose(logits[step][g["top_idx"][step]], g["top_val"][step], rtol=0, atol=1e-4)
