"""ORACLE (test infrastructure): Q8_0 restated in numpy.

Follows ``quantize_q80`` / ``dequantize_q80`` of src/orchestrator/quantizer.py:11-26 / :29-40
step by step: C-order flatten, zero padding to 32, per-block absmax with 0 -> 1.0,
f32 scale = absmax / 127, q = clip(round_half_even(x / scale), -128, 127) as int8.
"""
from __future__ import annotations

import numpy as np

BLOCK = 32
MIN_QUANTIZE_ELEMS = 4096  # quantizer.py:8


def quantize_q80(arr: np.ndarray, block_size: int = BLOCK):
    orig_shape = arr.shape
    flat = np.asarray(arr).ravel().astype(np.float32)              # quantizer.py:14
    n = flat.shape[0]
    n_blocks = (n + block_size - 1) // block_size                   # :16
    padded = np.zeros(n_blocks * block_size, dtype=np.float32)     # :17-18
    padded[:n] = flat
    blocks = padded.reshape(n_blocks, block_size)                   # :20
    absmax = np.max(np.abs(blocks), axis=1, keepdims=True)          # :21
    absmax = np.where(absmax == 0, np.float32(1.0), absmax).astype(np.float32)  # :22
    scales = (absmax / np.float32(127.0)).ravel()                   # :23 (f32 division)
    q = np.clip(np.round(blocks / scales.reshape(n_blocks, 1)), -128, 127).astype(np.int8)  # :24
    return q, scales, orig_shape


def dequantize_q80(qdata: np.ndarray, scales: np.ndarray, orig_shape) -> np.ndarray:
    flat = qdata.ravel().astype(np.float32)                         # quantizer.py:32
    n_blocks = scales.shape[0]
    bs = flat.shape[0] // n_blocks
    blocks = flat.reshape(n_blocks, bs)
    result = (blocks * scales.reshape(n_blocks, 1).astype(np.float32)).ravel()  # :36
    total = int(np.prod(orig_shape)) if len(orig_shape) else 1
    return np.ascontiguousarray(result[:total].reshape(orig_shape))


def q80_roundtrip(arr: np.ndarray, scale_dtype=np.float32) -> np.ndarray:
    """dequantize(quantize(arr)); with scale_dtype=float16 the scales are first rounded to
    f16, which is the device weight format's storage (34 bytes per 32 weights)."""
    q, s, sh = quantize_q80(arr)
    s = s.astype(scale_dtype).astype(np.float32)
    return dequantize_q80(q, s, sh)
