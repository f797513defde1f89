"""ORACLE (test infrastructure): numpy restatement of src/kernels/mojo/pyre_kernels.mojo.

Each function follows the Mojo loop it names (same accumulation types and order of
operations, vectorised where the result is the same).
"""
from __future__ import annotations

import numpy as np


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """pyre_kernels.mojo:18-35 — f64 sum of squares, rstd = 1/sqrt(mean + 1e-6),
    out = f32(f64(x) * rstd * f64(w))."""
    x64 = x.astype(np.float64)
    sq = np.sum(x64 * x64, axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt(sq / x.shape[-1] + eps)
    return (x64 * rstd * weight.astype(np.float64)).astype(np.float32)


def softmax(x: np.ndarray) -> np.ndarray:
    """pyre_kernels.mojo:39-58 — row max initialised to -1e10, f32 exp, times 1/sum."""
    x = x.astype(np.float32)
    mx = np.maximum(np.max(x, axis=-1, keepdims=True), np.float32(-1e10))
    e = np.exp(x - mx).astype(np.float32)
    inv = np.float32(1.0) / np.sum(e, axis=-1, keepdims=True, dtype=np.float32)
    return (np.exp(x - mx).astype(np.float32) * inv).astype(np.float32)


def rope_tables(theta: float, start_pos: int, seq: int, dims: int):
    """cos/sin tables of pyre_kernels.mojo:86-89: freq_i = 1/theta^(2i/dims) in f64,
    angle = f64(start_pos + pos) * freq_i, cast to f32."""
    half = dims // 2
    i = np.arange(half, dtype=np.float64)
    freq = 1.0 / (np.float64(theta) ** (2.0 * i / np.float64(dims)))
    pos = (start_pos + np.arange(seq, dtype=np.int64)).astype(np.float64)
    ang = pos[:, None] * freq[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def apply_rope(x: np.ndarray, theta: float = 10000.0, start_pos: int = 0, rope_fraction: float = 1.0) -> np.ndarray:
    """pyre_kernels.mojo:62-96 — rotate-half over the first int(D*rope_fraction) dims of
    x [B, H, S, D]; the rest is copied."""
    B, H, S, D = x.shape
    dims = int(float(D) * float(rope_fraction))
    if dims < 2:
        return x.astype(np.float32).copy()
    half = dims // 2
    c, s = rope_tables(theta, start_pos, S, dims)
    out = x.astype(np.float32).copy()
    x1 = x[..., :half].astype(np.float32)
    x2 = x[..., half:2 * half].astype(np.float32)
    out[..., :half] = x1 * c - x2 * s
    out[..., half:2 * half] = x1 * s + x2 * c
    return out


def silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """pyre_kernels.mojo:121-129 — g / (1 + exp(-g)) * up in f32."""
    g = gate.astype(np.float32)
    with np.errstate(over="ignore"):
        return (g / (np.float32(1.0) + np.exp(-g)) * up.astype(np.float32)).astype(np.float32)


def silu(g: np.ndarray) -> np.ndarray:
    g = g.astype(np.float32)
    with np.errstate(over="ignore"):
        return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)


def matmul_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """pyre_kernels.mojo:133-146 — [M, K] x [K, N] with an f32 accumulator per output
    (k ascending). The numpy product differs only in summation order; use
    oracle/csrc (pyre_matmul_f32) when the exact loop order matters."""
    return (a.astype(np.float32) @ b.astype(np.float32)).astype(np.float32)


def q80_dequantize(q: np.ndarray, scales: np.ndarray, n: int) -> np.ndarray:
    """pyre_kernels.mojo:172-185 — out[i] = f32(q[i]) * scales[i // 32]."""
    qf = q.ravel()[:n].astype(np.float32)
    return qf * np.repeat(scales.astype(np.float32), 32)[:n]
