"""FFN shard builder with the interface of ``src/ffn/builder.py``.

``ShardSpec`` (``builder.py:11-17``), ``build_ffn_graph`` (``:20-53``) and
``compile_and_run`` (``:56-83``) keep their names, arguments and errors. The returned
graph runs the Q8_0 FFN kernels of this library:

* gated:   ``partial = (silu(x @ gate) * (x @ up)) @ down``   (``builder.py:37-45``)
* ungated: ``partial = silu(x @ up) @ down``                  (``builder.py:46-51``)

Weights passed to ``execute`` may be :class:`~pyre_b200.quantizer.Q80Weight` (the device
format, used as is), reference Q8_0 tuples ``("q8", q, s, shape)``, or float arrays /
tensors of shape ``[hidden, width]`` / ``[width, hidden]`` (quantized to Q8_0 on the GPU
first, as a reference worker quantizes its shard, ``worker_node.py:59-69``).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .. import _device as D
from ..engine import DeviceRef, Graph, InferenceSession, Tensor
from ..quantizer import Q80Weight
from .op import FfnShardOp, FfnWeights


@dataclass(frozen=True)
class ShardSpec:
    ffn_dim_start: int
    ffn_dim_end: int

    def ffn_width(self) -> int:
        return self.ffn_dim_end - self.ffn_dim_start


@dataclass(frozen=True)
class FfnGraph(Graph):
    shard: object
    hidden_dim: int
    device: DeviceRef
    seq_len: int
    name: str
    gated: bool

    def _load(self, session: InferenceSession) -> "FfnModel":
        return FfnModel(self, session)


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


class FfnModel:
    """A loaded FFN graph (``session.load(graph)``)."""

    def __init__(self, graph: FfnGraph, session: InferenceSession, comm=None):
        self.graph = graph
        self.device = graph.device.cuda_device() if graph.device.kind == "gpu" else session.cuda_device
        with torch.cuda.device(self.device):
            self.op = FfnShardOp(graph.hidden_dim, graph.shard.ffn_width(), graph.seq_len,
                                 gated=graph.gated, comm=comm, device=self.device)

    def execute(self, *inputs) -> tuple:
        g = self.graph
        n_expected = 4 if g.gated else 3
        if len(inputs) != n_expected:
            raise ValueError(f"{g.name}: expected {n_expected} inputs, got {len(inputs)}")
        H, W, S = g.hidden_dim, g.shard.ffn_width(), g.seq_len
        with torch.cuda.device(self.device):
            x = D.to_device(inputs[0], self.device)
            if tuple(x.shape) != (1, S, H):
                raise ValueError(f"{g.name}: x must be [1, {S}, {H}], got {tuple(x.shape)}")
            if x.dtype not in (torch.float32, torch.bfloat16):
                x = x.to(torch.float32)
            if g.gated:
                gate = _as_weight(inputs[1], (H, W))
                up = _as_weight(inputs[2], (H, W))
                down = _as_weight(inputs[3], (W, H))
            else:
                gate = None
                up = _as_weight(inputs[1], (H, W))
                down = _as_weight(inputs[2], (W, H))
            out = self.op.run(x.reshape(S, H), FfnWeights.prepare(gate, up, down))
            return (Tensor(out.reshape(1, S, H)),)


def build_ffn_graph(
    shard: ShardSpec,
    hidden_dim: int,
    device: DeviceRef,
    *,
    seq_len: int = 1,
    name: str = "ffn_shard",
    gated: bool = False,
) -> FfnGraph:
    width = shard.ffn_width()
    if width <= 0:
        raise ValueError(f"ShardSpec width must be positive, got {width}")
    return FfnGraph(shard=shard, hidden_dim=hidden_dim, device=device, seq_len=seq_len, name=name, gated=gated)


def compile_and_run(
    shard: ShardSpec,
    hidden_dim: int,
    x,
    ffn_up_slice,
    ffn_down_slice,
    *,
    seq_len: int | None = None,
    device: DeviceRef | None = None,
):
    """Ungated shard, run once; returns a numpy ``[1, seq_len, hidden_dim]`` f32 partial."""
    if seq_len is None:
        seq_len = x.shape[1]
    if device is None:
        device = DeviceRef.CPU()
    graph = build_ffn_graph(shard, hidden_dim, device, seq_len=seq_len)
    session = InferenceSession()
    model = session.load(graph)
    (out,) = model.execute(
        np.ascontiguousarray(x) if isinstance(x, np.ndarray) else x,
        ffn_up_slice,
        ffn_down_slice,
    )
    return out.to_numpy()
