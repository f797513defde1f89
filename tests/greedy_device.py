"""The seeded greedy models of tests/golden/greedy_model.py on this library's kernels.

Weights follow the same generation order as the fixtures; each bf16-rounded matrix is quantized
on the device (pyre_q80_quantize is bit-exact with the reference's quantize_q80, and the f16
scale is the device format's), which gives exactly the Q8_0 blocks whose f32 dequantized values
the reference ran on.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))

import greedy_model as gm  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"


def golden(m: "gm.Model"):
    return np.load(GOLDEN / m.fixture)


def device_weights(m: "gm.Model", device):
    """(embedding f16, reference-shaped layer dicts of Q80Weight, final norm, lm_head or None)."""
    import torch
    from pyre_b200.quantizer import Q80Weight

    def to_q80(a):
        return Q80Weight.from_float(torch.from_numpy(np.ascontiguousarray(a)).to(device), torch.float16)

    emb, layers, final_norm, head = gm.build(m, to_q80)
    out = []
    for lw in layers:
        attn = {n: lw[n] for n in ("q", "k", "v", "o")}
        for n in ("q_bias", "k_bias", "v_bias"):
            if n in lw:
                attn[n] = lw[n]
        out.append({"input_layernorm": lw["ln1"], "post_attention_layernorm": lw["ln2"], "attn": attn,
                    "ffn": {n: lw[n] for n in ("gate", "up", "down")}})
    return emb, out, final_norm, head


def generator(m: "gm.Model", device, comm=None, ffn_plan=None, persistent=False):
    from pyre_b200.generator import Generator
    emb, layers, final_norm, head = device_weights(m, device)
    return Generator(layers, emb, final_norm, n_heads=m.n_heads, n_kv_heads=m.n_kv, head_dim=m.head_dim,
                     rope_theta=m.theta, eps=m.eps, lm_head=head, max_seq=m.prompt_len + gm.N_GREEDY + 16,
                     max_prompt=max(64, m.prompt_len), device=device, comm=comm, ffn_plan=ffn_plan,
                     persistent=persistent)
