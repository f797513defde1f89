"""A compiled FFN shard call for fixed shapes: host buffers in, host buffers out.

The reference compiles one FFN graph per (shard, seq_len) at start-up and then calls
``model.execute(...)`` per layer and token (src/orchestrator/root_node.py:143-151,
:574-580; src/orchestrator/worker_node.py:122-130, :319-329). The B200 equivalent of that
compile step is a CUDA graph: :class:`CapturedFfn` captures the host->device copy of the
activations, the two FFN kernels (and, with a communicator, the in-kernel NVLink
reduction) and the device->host copy of the partial sum, so one ``execute`` is one graph
launch plus a stream synchronisation, with no per-kernel launch cost on the CPU.
"""
from __future__ import annotations

import torch

from .op import FfnShardOp, FfnWeights


class CapturedFfn:
    def __init__(self, op: FfnShardOp, weights: FfnWeights, tokens: int, x_dtype: torch.dtype = torch.bfloat16):
        if tokens > op.max_tokens:
            raise ValueError("tokens exceeds the op's max_tokens")
        self.op = op
        self.tokens = tokens
        dev = op.device
        self.x_host = torch.empty((tokens, op.hidden), dtype=x_dtype, pin_memory=True)
        self.out_host = torch.empty((tokens, op.hidden), dtype=torch.float32, pin_memory=True)
        self.x_dev = torch.zeros((tokens, op.hidden), dtype=x_dtype, device=dev)
        self.out_dev = torch.zeros((tokens, op.hidden), dtype=torch.float32, device=dev)
        self._w = weights
        self.stream = torch.cuda.Stream(device=dev)
        # one eager call on the capture stream first (sets up lazy state, checks arguments)
        with torch.cuda.stream(self.stream):
            op.run(self.x_dev, weights, out=self.out_dev, stream=self.stream)
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.x_dev.copy_(self.x_host, non_blocking=True)
            op.run(self.x_dev, weights, out=self.out_dev, stream=self.stream)
            self.out_host.copy_(self.out_dev, non_blocking=True)

    @property
    def h2d_bytes(self) -> int:
        return self.x_host.numel() * self.x_host.element_size()

    @property
    def d2h_bytes(self) -> int:
        return self.out_host.numel() * self.out_host.element_size()

    def execute(self, x) -> torch.Tensor:
        """Runs one call on host activations ``x [tokens, hidden]``; returns the host f32
        partial (the op's cross-rank sum when it has a communicator). The returned tensor
        is the runner's pinned output buffer, overwritten by the next call."""
        self.x_host.copy_(torch.as_tensor(x).reshape(self.x_host.shape))
        with torch.cuda.stream(self.stream):
            self.graph.replay()
        self.stream.synchronize()
        return self.out_host
