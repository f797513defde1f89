"""ORACLE (test infrastructure): CPU restatement of the reference's last decode step.

Used only by tests/, __graft_entry__.smoke() and bench.py's CPU baseline, as the checker.

* ``final_rms_norm``  — Generator._rms_norm, src/orchestrator/generator.py:40-43 (f64 mean of
                        squares, x / sqrt(var + eps) in f64, times the f32 norm weight, to f32).
* ``compute_logits``  — Generator._compute_logits, generator.py:45-48 (norm, then h @ E^T with
                        the f16 lm_head table upcast to f32).
* ``greedy_token``    — Generator._sample with temperature < 0.01, generator.py:50-53
                        (np.argmax: the first index among equal maxima).
"""
from __future__ import annotations

import numpy as np


def final_rms_norm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    variance = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    x_norm = x / np.sqrt(variance + eps)
    return (x_norm * w.astype(np.float32)).astype(np.float32)


def compute_logits(h: np.ndarray, lm_head_f16: np.ndarray, norm_w: np.ndarray | None,
                   eps: float = 1e-6) -> np.ndarray:
    if norm_w is not None:
        h = final_rms_norm(h, norm_w, eps)
    return h @ lm_head_f16.astype(np.float32).T


def greedy_token(logits: np.ndarray) -> np.ndarray:
    return np.argmax(logits, axis=-1, keepdims=True)
