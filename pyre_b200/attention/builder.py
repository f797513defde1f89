"""Attention builder with the interface of ``src/attention/builder.py``.

``ShardSpec`` (``builder.py:9-24``) keeps its fields and methods;
``build_ulysses_attention_graph`` (``:27-65``) keeps its arguments and the head counts it
derives (``full_q_weights``: the shard's own head counts, else ``ffn_width // head_dim`` q
heads and all kv heads). Executing the graph computes ``q, k, v = x @ Wq, x @ Wk, x @ Wv``
reshaped to ``[1, S, heads, head_dim]`` with the Q8_0 projection kernel of this library.
Weights may be :class:`~pyre_b200.quantizer.Q80Weight`, reference Q8_0 tuples, or float
arrays / tensors (quantized to Q8_0 on the GPU, as a reference worker quantizes them,
``worker_node.py:59-69``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _device as D
from ..engine import DeviceRef, Graph, InferenceSession, Tensor
from ..quantizer import Q80Weight
from .ops import Q80Linear


@dataclass(frozen=True)
class ShardSpec:
    ffn_dim_start: int
    ffn_dim_end: int
    seq_start: int
    seq_end: int
    n_q_heads: int = 0
    n_kv_heads: int = 0
    q_head_start: int = 0
    kv_head_start: int = 0

    def ffn_width(self) -> int:
        return self.ffn_dim_end - self.ffn_dim_start

    def local_seq_len(self) -> int:
        return self.seq_end - self.seq_start


@dataclass(frozen=True)
class AttentionGraph(Graph):
    shard: ShardSpec
    hidden_dim: int
    n_q_local: int
    n_kv_local: int
    head_dim: int
    device: DeviceRef
    name = "ulysses_attention_shard"

    def _load(self, session: InferenceSession) -> "AttentionModel":
        return AttentionModel(self, session)


def _as_weight(w, shape) -> Q80Weight:
    if isinstance(w, Q80Weight):
        q = w
    elif isinstance(w, tuple):
        q = Q80Weight.from_tuple(w)
    else:
        q = Q80Weight.from_float(D.to_device(w))
    if tuple(q.shape) != tuple(shape):
        raise ValueError(f"weight shape {tuple(q.shape)} does not match the graph's {tuple(shape)}")
    return q


class AttentionModel:
    """A loaded attention graph (``session.load(graph)``)."""

    def __init__(self, graph: AttentionGraph, session: InferenceSession):
        self.graph = graph
        self.device = graph.device.cuda_device() if graph.device.kind == "gpu" else session.cuda_device
        self._lin = {}

    def execute(self, x, wq, wk, wv) -> tuple:
        g = self.graph
        S, H, hd = g.shard.local_seq_len(), g.hidden_dim, g.head_dim
        with torch.cuda.device(self.device):
            xt = D.to_device(x, self.device)
            if tuple(xt.shape) != (1, S, H):
                raise ValueError(f"{g.name}: x must be [1, {S}, {H}], got {tuple(xt.shape)}")
            if xt.dtype not in (torch.float32, torch.bfloat16):
                xt = xt.to(torch.float32)
            outs = []
            for name, w, n in (("q", wq, g.n_q_local), ("k", wk, g.n_kv_local), ("v", wv, g.n_kv_local)):
                lin = Q80Linear(_as_weight(w, (H, n * hd)), S, self.device)
                y = lin(xt.reshape(S, H))
                outs.append(Tensor(y.reshape(1, S, n, hd)))
            return tuple(outs)


def build_ulysses_attention_graph(
    shard: ShardSpec,
    hidden_dim: int,
    n_heads: int,
    n_kv_heads: int,
    head_dim: int,
    device: DeviceRef,
    full_q_weights: bool = False,
) -> AttentionGraph:
    if full_q_weights:
        n_q_local = shard.n_q_heads if shard.n_q_heads > 0 else n_heads
        n_kv_local = shard.n_kv_heads if shard.n_kv_heads > 0 else n_kv_heads
    else:
        n_q_local = shard.ffn_width() // head_dim
        n_kv_local = n_kv_heads
    return AttentionGraph(shard=shard, hidden_dim=hidden_dim, n_q_local=n_q_local, n_kv_local=n_kv_local,
                          head_dim=head_dim, device=device)
