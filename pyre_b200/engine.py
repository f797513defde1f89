"""Session / graph / tensor objects with the shape of the reference's MAX engine usage.

The reference builds a graph per op (``build_ffn_graph``, ``build_ulysses_attention_graph``)
and runs it with ``InferenceSession(devices=[CPU()]).load(graph).execute(*arrays)``,
reading results back with ``.to_numpy()`` (``src/ffn/builder.py:74-83``,
``src/orchestrator/root_node.py:99``, ``:151``, ``:574-580``,
``src/orchestrator/worker_node.py:123-130``). Here a "graph" is a descriptor of one of the
fixed CUDA ops of this library and ``load`` binds it to a GPU; ``execute`` launches the
sm_100a kernels on the current CUDA stream. There is no graph compiler and no CPU path:
``DeviceRef.CPU()`` only means that inputs and outputs may be host arrays, while the
arithmetic still runs on the GPU.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _device as D


@dataclass(frozen=True)
class DeviceRef:
    """Where a graph's inputs and outputs live (mirrors ``max.graph.DeviceRef``)."""

    kind: str = "gpu"
    id: int = 0

    @staticmethod
    def CPU(id: int = 0) -> "DeviceRef":  # noqa: N802 - reference spelling
        return DeviceRef("cpu", id)

    @staticmethod
    def GPU(id: int = 0) -> "DeviceRef":  # noqa: N802 - reference spelling
        return DeviceRef("gpu", id)

    def cuda_device(self) -> torch.device:
        if self.kind == "gpu":
            return torch.device("cuda", self.id)
        return torch.device("cuda", torch.cuda.current_device())


class CPU:
    """Host device handle (``max.driver.CPU``): host-resident inputs/outputs."""

    def __init__(self, id: int = 0):
        self.id = id


class Accelerator:
    """GPU device handle (``max.driver.Accelerator``)."""

    def __init__(self, id: int = 0):
        self.id = id


class Tensor:
    """Result tensor (``max.driver.Tensor``): a CUDA tensor with ``to_numpy()``."""

    def __init__(self, t: torch.Tensor):
        self._t = t

    @property
    def torch(self) -> torch.Tensor:
        return self._t

    @property
    def shape(self):
        return tuple(self._t.shape)

    @property
    def dtype(self):
        return self._t.dtype

    def to_numpy(self) -> np.ndarray:
        return self._t.detach().to("cpu").numpy()

    def __array__(self, dtype=None):
        a = self.to_numpy()
        return a if dtype is None else a.astype(dtype)


class Graph:
    """Base of the op descriptors returned by the builders."""

    def _load(self, session: "InferenceSession"):
        raise NotImplementedError


class InferenceSession:
    """Binds graphs to the GPU (``max.engine.InferenceSession``)."""

    def __init__(self, devices=None):
        D.require_cuda()
        self.devices = list(devices) if devices else [CPU()]
        gpus = [d for d in self.devices if isinstance(d, Accelerator)]
        self.cuda_device = torch.device("cuda", gpus[0].id if gpus else torch.cuda.current_device())

    def load(self, graph: Graph):
        if not isinstance(graph, Graph):
            raise TypeError(f"InferenceSession.load expects a pyre_b200 graph, got {type(graph).__name__}")
        return graph._load(self)
