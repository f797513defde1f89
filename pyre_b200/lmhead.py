"""Last step of a decode token on the GPU: final RMSNorm, lm_head logits, greedy token.

Mirrors ``Generator._rms_norm`` / ``_compute_logits`` / ``_sample(temperature < 0.01)``
(src/orchestrator/generator.py:40-53), whose table is stored as f16 (``generator.py:32``).
One launch of ``lm_head_kernel`` streams the table once. With the table sharded by
vocabulary over the ranks of a process group (rank r holds rows ``vocab_start ..
vocab_start + V_r - 1``), each rank's best (value, index) key is combined across the ranks:
through the peer-memory communicator (``pyre_argmax_combine``, one small launch) when a
:class:`~pyre_b200.tp.TPComm` is given, or with one max all-reduce of T int64 values over a
``torch.distributed`` group.
"""
from __future__ import annotations

import ctypes

import torch

from . import _device as D
from . import _native as N

_KEY_TOP = -(1 << 63)


class LmHeadOp:
    def __init__(self, lm_head: torch.Tensor, norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                 vocab_start: int = 0, group=None, max_tokens: int = 1, comm=None):
        if lm_head.dtype != torch.float16 or lm_head.dim() != 2 or not lm_head.is_cuda:
            raise ValueError("lm_head must be a CUDA f16 tensor [V, H]")
        if not 1 <= max_tokens <= 4:
            raise ValueError("max_tokens must be in [1, 4]")
        self.table = lm_head.contiguous()
        self.V, self.H = self.table.shape
        self.norm = None if norm_weight is None else norm_weight.to(self.table.device, torch.float32).contiguous()
        if self.norm is not None and self.norm.numel() != self.H:
            raise ValueError(f"norm weight must have {self.H} elements")
        self.eps = float(eps)
        self.v0 = int(vocab_start)
        self.group = group
        self.comm = comm if (comm is not None and comm.world > 1) else None
        if self.comm is not None and group is not None:
            raise ValueError("give either a communicator or a process group")
        self.max_tokens = max_tokens
        b = ctypes.c_int64(0)
        N.call("pyre_lm_head_workspace_bytes", max_tokens, ctypes.byref(b))
        self.workspace = torch.zeros(int(b.value), dtype=torch.uint8, device=self.table.device)

    def __call__(self, h: torch.Tensor, want_logits: bool = False, stream=None):
        """h: f32 [T, H] (the last hidden states). Returns the greedy tokens, int64 [T, 1] (the
        reference's ``np.argmax(..., keepdims=True)``), and with ``want_logits`` also this
        rank's logits f32 [T, V]."""
        if h.dtype != torch.float32 or h.dim() != 2 or h.shape[1] != self.H:
            raise ValueError(f"h must be f32 [T, {self.H}]")
        T = h.shape[0]
        if not 1 <= T <= self.max_tokens:
            raise ValueError(f"T={T} outside [1, {self.max_tokens}]")
        h = h.contiguous()
        dev = h.device
        token = torch.empty(T, dtype=torch.int32, device=dev)
        key = torch.empty(T, dtype=torch.int64, device=dev)
        logits = torch.empty((T, self.V), dtype=torch.float32, device=dev) if want_logits else None
        N.call("pyre_lm_head_argmax", D.ptr(h), T, self.H, D.ptr(self.norm) if self.norm is not None else None,
               self.eps, D.ptr(self.table), self.V, self.v0, D.ptr(logits) if logits is not None else None,
               D.ptr(token), D.ptr(key), D.ptr(self.workspace), self.workspace.numel(), D.stream_ptr(stream))
        if self.comm is not None:
            N.call("pyre_argmax_combine", ctypes.c_void_p(self.comm.handle), D.ptr(key), T, D.ptr(token), None,
                   D.stream_ptr(stream))
            tok = token.to(torch.int64)
        elif self.group is not None:
            import torch.distributed as dist
            dist.all_reduce(key, op=dist.ReduceOp.MAX, group=self.group)
            low = (key ^ _KEY_TOP) & 0xFFFFFFFF
            tok = (0xFFFFFFFF - low).to(torch.int64)
        else:
            tok = token.to(torch.int64)
        tok = tok.view(T, 1)
        return (tok, logits) if want_logits else tok
