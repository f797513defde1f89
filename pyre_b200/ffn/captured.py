"""A compiled FFN shard call for fixed shapes: host buffers in, host buffers out.

The reference compiles one FFN graph per (shard, seq_len) at start-up and then calls
``model.execute(...)`` per layer and token (src/orchestrator/root_node.py:143-151,
:574-580; src/orchestrator/worker_node.py:122-130, :319-329). The B200 equivalent of that
compile step is a CUDA graph: :class:`CapturedFfn` captures the host->device copy of the
activations, the two FFN kernels (and, with a communicator, the in-kernel NVLink
reduction) and the device->host copy of the partial sum, so one ``execute`` is one native
call (``pyre_graph_run``: host copy into the pinned input, graph launch, stream wait), with
no per-kernel launch cost on the CPU.
"""
from __future__ import annotations

import torch

from .. import _native as N
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
        # decode path (one streaming launch): its kernel stores the result straight into the
        # pinned host buffer over PCIe (zero-copy), so the graph has no device->host copy node;
        # larger T keep the device output and a copy node
        self.zero_copy_out = tokens <= N.PYRE_FUSED_REDUCE_MAX_T and op.fused
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.x_dev.copy_(self.x_host, non_blocking=True)
            if self.zero_copy_out:
                op.run(self.x_dev, weights, out=self.out_host, stream=self.stream)
            else:
                op.run(self.x_dev, weights, out=self.out_dev, stream=self.stream)
                self.out_host.copy_(self.out_dev, non_blocking=True)
        # the instantiated graph, launched by the library's native runner
        lib = N.load()
        self._exec = self.graph.raw_cuda_graph_exec()
        self._stream_ptr = self.stream.cuda_stream
        self._x_ptr = self.x_host.data_ptr()
        fn = lib.pyre_graph_run

        def run(*args):
            N.check(fn(*args))
        self._run = run

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
        if (isinstance(x, torch.Tensor) and x.dtype == self.x_host.dtype and not x.is_cuda and x.is_contiguous()
                and x.numel() == self.x_host.numel()):
            # same-dtype host tensor: the native runner copies it into the pinned buffer
            src, nbytes = x.data_ptr(), self.h2d_bytes
        else:
            self.x_host.copy_(torch.as_tensor(x).reshape(self.x_host.shape))
            src, nbytes = None, 0
        # one native call: host copy into the pinned input, graph launch, wait
        self._run(self._exec, self._stream_ptr, src, self._x_ptr, nbytes)
        return self.out_host
