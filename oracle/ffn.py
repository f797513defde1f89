"""ORACLE (test infrastructure): the FFN shard and its tensor-parallel sum, on the CPU.

* :func:`ffn_shard` — the graph of src/ffn/builder.py:37-51 in f32 numpy
  (gated: silu(x@Wg) * (x@Wu) @ Wd; ungated: silu(x@Wu) @ Wd).
* :func:`worker_ffn_step` — what a reference worker does per FFN message
  (src/orchestrator/worker_node.py:59-69 dequantizes its Q8_0 layer cache on every
  access, then :319-329 runs the FFN graph).
* :func:`tp_ffn` — partials of every shard summed in rank order, as the root's
  ``ffn_out += partial`` (src/orchestrator/root_node.py:582-594, :982-995).
"""
from __future__ import annotations

import numpy as np

from . import kernels as K
from . import q80


def ffn_shard(x: np.ndarray, gate, up: np.ndarray, down: np.ndarray) -> np.ndarray:
    """x [..., H] f32; gate/up [H, W]; down [W, H] -> partial [..., H] f32."""
    x = x.astype(np.float32)
    if gate is not None:
        h = K.silu(x @ gate.astype(np.float32)) * (x @ up.astype(np.float32))
    else:
        h = K.silu(x @ up.astype(np.float32))
    return (h.astype(np.float32) @ down.astype(np.float32)).astype(np.float32)


def ffn_shard_f64(x: np.ndarray, gate, up: np.ndarray, down: np.ndarray) -> np.ndarray:
    """Same graph in f64 (a tighter yardstick for tolerance checks)."""
    x = x.astype(np.float64)
    up_ = x @ up.astype(np.float64)
    if gate is not None:
        g = x @ gate.astype(np.float64)
        h = g / (1.0 + np.exp(-g)) * up_
    else:
        h = up_ / (1.0 + np.exp(-up_))
    return h @ down.astype(np.float64)


def worker_ffn_step(x: np.ndarray, qgate: tuple, qup: tuple, qdown: tuple) -> np.ndarray:
    """One reference worker FFN call on Q8_0-cached weights: dequantize, then the graph."""
    gate = q80.dequantize_q80(*qgate) if qgate is not None else None
    up = q80.dequantize_q80(*qup)
    down = q80.dequantize_q80(*qdown)
    return ffn_shard(x, gate, up, down)


def tp_ffn(x: np.ndarray, gate, up: np.ndarray, down: np.ndarray, bounds, f64: bool = False) -> np.ndarray:
    """Sum of the shard partials over ``bounds`` = [(start, end), ...] in order."""
    fn = ffn_shard_f64 if f64 else ffn_shard
    out = None
    for s, e in bounds:
        part = fn(x, None if gate is None else gate[:, s:e], up[:, s:e], down[s:e, :])
        out = part if out is None else out + part
    return out
