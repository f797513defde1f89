"""The FFN shard op on Q8_0 weights: ``partial = (silu(x@Wg) * (x@Wu)) @ Wd``.

This is the compute of ``build_ffn_graph`` (``src/ffn/builder.py:37-45``) and of the root's
decode FFN (``src/orchestrator/root_node.py:956-980``), plus, when a :class:`TPComm` is
given, the cross-rank sum ``ffn_out += partial`` (``root_node.py:582-594``, ``:982-995``)
done inside the down-projection's epilogue over NVLink.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from .. import _device as D
from .. import _native as N
from ..quantizer import Q80Packed, Q80Weight


def workspace_bytes(tokens: int, hidden: int, width: int) -> int:
    out = ctypes.c_int64(0)
    N.call("pyre_ffn_workspace_bytes", int(tokens), int(hidden), int(width), ctypes.byref(out))
    return int(out.value)


@dataclass
class FfnWeights:
    """One shard's weights in the kernels' packed layout (prepare once, call many times):
    gate and up packed as a pair (or up alone when ungated), down packed alone."""

    gateup: Q80Packed
    down: Q80Packed
    gated: bool

    @property
    def hidden(self) -> int:
        return self.gateup.k

    @property
    def width(self) -> int:
        return self.gateup.n

    @classmethod
    def prepare(cls, gate: Q80Weight | None, up: Q80Weight, down: Q80Weight) -> "FfnWeights":
        H, W = up.shape
        if gate is not None and (gate.shape != (H, W) or gate.scale.dtype != up.scale.dtype):
            raise ValueError(f"gate weight must be {(H, W)} with the up weight's scale dtype")
        if down.shape != (W, H):
            raise ValueError(f"down weight must be {(W, H)}, got {down.shape}")
        if down.scale.dtype != up.scale.dtype:
            raise ValueError("down and up scales must share a dtype")
        gu = Q80Packed.pack([gate, up] if gate is not None else [up])
        return cls(gu, Q80Packed.pack(down), gate is not None)


class FfnShardOp:
    """One rank's FFN shard for up to ``max_tokens`` tokens.

    Holds the zero-initialised scratch the kernels need (reused call after call on one
    stream). Decode (T <= 4) is one persistent launch (``pyre_ffn_decode_q80``: gate/up +
    SiLU·mul, then down + the tensor-parallel reduction when ``comm`` is set); larger T,
    or ``fused=False``, uses the two-call form (``pyre_ffn_gateup_silu_q80`` then
    ``pyre_ffn_down_q80``).
    """

    def __init__(self, hidden_dim: int, width: int, max_tokens: int = 1, *, gated: bool = True,
                 comm=None, device: torch.device | None = None, fused: bool = True):
        D.require_cuda()
        if width <= 0 or hidden_dim <= 0:
            raise ValueError(f"ShardSpec width must be positive, got {width}")
        if width % 32 or hidden_dim % 32:
            raise ValueError("FFN shard width and hidden dim must be multiples of 32 (Q8_0 blocks)")
        self.hidden = int(hidden_dim)
        self.width = int(width)
        self.max_tokens = int(max_tokens)
        self.gated = gated
        self.comm = comm
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        wsb = workspace_bytes(self.max_tokens, self.hidden, self.width)
        self.workspace = torch.zeros(wsb, dtype=torch.uint8, device=self.device)
        self.fused = fused

    def launches(self, tokens: int) -> int:
        """Kernel launches of one call with ``tokens`` tokens."""
        if tokens <= N.PYRE_FUSED_REDUCE_MAX_T:
            return 1 if self.fused else 2
        return 2 + (1 if (self.comm is not None and self.comm.world > 1) else 0)

    def status(self) -> int:
        """Status word of the op's kernels (PYRE_OK, or PYRE_ETIMEOUT if a pipeline or flag
        wait ran out); read after synchronising the stream."""
        return int(self.workspace[8:12].view(torch.int32).item())

    def reset(self) -> None:
        """Zero the scratch (status, counters, flags). Needed after a call that reported
        PYRE_ETIMEOUT: the kernels stop early then and leave their counters part-way."""
        self.workspace.zero_()

    def h_dtype(self, tokens: int) -> torch.dtype:
        # decode keeps the intermediate in f32; larger T stores f16, the tensor-core operand
        # type of the down GEMM
        return torch.float32 if tokens <= N.PYRE_FUSED_REDUCE_MAX_T else torch.float16

    def __call__(self, x: torch.Tensor, gate: Q80Weight | None, up: Q80Weight, down: Q80Weight,
                 out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """Convenience form on Q8_0 weights (packs them on every call); prepare an
        :class:`FfnWeights` once and use :meth:`run` on a hot path."""
        return self.run(x, FfnWeights.prepare(gate, up, down), out=out, stream=stream)

    def run(self, x: torch.Tensor, w: FfnWeights, out: torch.Tensor | None = None,
            stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError(f"x must be [T, {self.hidden}], got {tuple(x.shape)}")
        T = x.shape[0]
        if T < 1 or T > self.max_tokens:
            raise ValueError(f"T={T} outside [1, {self.max_tokens}]")
        if x.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("x must be float32 or bfloat16")
        if not x.is_contiguous():
            x = x.contiguous()
        if w.hidden != self.hidden or w.width != self.width:
            raise ValueError(f"weights are [{w.hidden}, {w.width}], op is [{self.hidden}, {self.width}]")
        if self.gated != w.gated:
            raise ValueError("gated op needs gated weights (and ungated op ungated ones)")
        s = D.stream_ptr(stream)
        if out is None:
            out = torch.empty((T, self.hidden), dtype=torch.float32, device=x.device)
        ws = self.workspace
        comm = ctypes.c_void_p(self.comm.handle if self.comm is not None else 0)
        gated = 1 if w.gated else 0
        code = w.gateup.scale_code
        if self.fused and T <= N.PYRE_FUSED_REDUCE_MAX_T:
            N.call("pyre_ffn_decode_q80", D.ptr(x), D.dtype_code(x), T, self.hidden, D.ptr(w.gateup.data), gated,
                   D.ptr(w.down.data), code, self.width, D.ptr(out), D.ptr(ws), ws.numel(), comm, s)
            return out
        h = torch.empty((T, self.width), dtype=self.h_dtype(T), device=x.device)
        N.call("pyre_ffn_gateup_silu_q80", D.ptr(x), D.dtype_code(x), T, self.hidden, D.ptr(w.gateup.data), gated,
               code, self.width, D.ptr(h), D.dtype_code(h), D.ptr(ws), ws.numel(), s)
        N.call("pyre_ffn_down_q80", D.ptr(h), D.dtype_code(h), T, self.width, D.ptr(w.down.data), code,
               self.hidden, D.ptr(out), D.ptr(ws), ws.numel(), comm, s)
        return out
