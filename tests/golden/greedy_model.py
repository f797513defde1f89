"""Seeded SmolLM-135M-shaped Llama decoder (hidden 576, 30 layers, 9 q / 3 kv heads, head_dim
64, gated-SiLU 1536, vocab 49152, tied embeddings, RoPE theta 1e4) for the greedy-token parity
test. Shared by tests/golden/make_golden.py (which runs the reference orchestrator on these
weights) and tests/test_greedy_gpu.py (which runs this repository's kernels on them).

Weights: N(0, std) f32 (std 0.02, and 0.07 for a second fixture) from numpy seed 0 in a fixed order, rounded to bf16 (the loader's
cast), then Q8_0 with the f16-stored scale (the device format), given to both sides as the
f32 dequantized matrices; RMSNorm weights are ones. Prompt: 8 token ids from
np.random.default_rng(0).integers(0, 49152, 8)."""
from __future__ import annotations

import numpy as np

CFG = dict(hidden=576, layers=30, n_heads=9, n_kv=3, head_dim=64, ffn=1536, vocab=49152, theta=10000.0, eps=1e-6)
N_GREEDY = 32
# With N(0, 0.02) projections the random 30-layer stack maps every context to nearly the same
# last hidden state and greedy decoding repeats one token; with N(0, 0.07) the 32 tokens all differ,
# which makes the token-by-token comparison a real test. Both are fixtures.
GOLDENS = {"greedy_golden.npz": 0.02, "greedy_golden_std07.npz": 0.07}


def _bf16(a: np.ndarray) -> np.ndarray:
    u = a.astype(np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def prompt_ids() -> np.ndarray:
    return np.random.default_rng(0).integers(0, CFG["vocab"], 8)


def make_weights(q80_roundtrip, std: float = 0.02):
    """q80_roundtrip(w f32) -> f32 dequantized Q8_0 with f16 scales. Returns
    (embedding f16 [V, H], layers: list of dicts of f32 matrices, final_norm f32 [H]). std is
    the projection weights' standard deviation (the embedding keeps 0.02)."""
    H, L, nq, nkv, hd, I, V = (CFG[k] for k in ("hidden", "layers", "n_heads", "n_kv", "head_dim", "ffn", "vocab"))
    rng = np.random.default_rng(0)

    def w(shape):
        return q80_roundtrip(_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std)))

    emb = _bf16(rng.standard_normal((V, H), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    layers = []
    for _ in range(L):
        layers.append({
            "q": w((H, nq * hd)), "k": w((H, nkv * hd)), "v": w((H, nkv * hd)), "o": w((nq * hd, H)),
            "gate": w((H, I)), "up": w((H, I)), "down": w((I, H)),
            "ln1": np.ones(H, np.float32), "ln2": np.ones(H, np.float32),
        })
    return emb, layers, np.ones(H, np.float32)
