"""Ulysses sequence-parallel causal attention inside one box (one process per GPU).

The reference runs Ulysses attention when P > n_kv (root_node.py:110) and otherwise gathers
every node's q/k/v at the root over TCP (root_node.py:250-314). Here each rank keeps its
slice of the sequence: it rotates its tokens' q and k and stores every head straight into the
buffer of the rank that owns that head (the QKV all-gather fused into RoPE, NVLink peer
stores); each rank runs causal attention for its heads over the whole sequence and its
epilogue stores every output row into the buffer of the rank that owns the token (the
output scatter fused into the attention). Two flag barriers separate the phases.
"""
from __future__ import annotations

import ctypes
from typing import List

import torch

from .. import _device as D
from .. import _native as N
from ..tp import IPC_HANDLE_BYTES, dist_rank_world, exchange_handles


class UlyssesAttention:
    """Causal attention of an S-token sequence split evenly over the ranks of ``group``."""

    def __init__(self, seq_len: int, n_heads: int, n_kv_heads: int, head_dim: int, rope_theta: float = 10000.0,
                 rope_fraction: float = 1.0, group=None, timeout_s: float = 5.0):
        lib = N.load()
        self.rank, self.world = dist_rank_world(group)
        self.S, self.nq, self.nkv, self.hd = int(seq_len), int(n_heads), int(n_kv_heads), int(head_dim)
        self.theta, self.frac = float(rope_theta), float(rope_fraction)
        self.timeout_ns = int(timeout_s * 1e9)
        nbytes = ctypes.c_int64(0)
        N.check(lib.pyre_ulysses_buffer_bytes(self.S, self.world, self.nq, self.nkv, self.hd, ctypes.byref(nbytes)))
        local = ctypes.c_void_p(0)
        handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        N.check(lib.pyre_comm_alloc(nbytes.value, ctypes.byref(local), handle))
        self._local = local.value
        self._opened: List[int] = []
        ptrs = []
        for r, h in enumerate(exchange_handles(handle.raw, group)):
            if r == self.rank:
                ptrs.append(self._local)
                continue
            p = ctypes.c_void_p(0)
            N.check(lib.pyre_comm_open_peer(ctypes.create_string_buffer(h, IPC_HANDLE_BYTES), ctypes.byref(p)))
            self._opened.append(p.value)
            ptrs.append(p.value)
        self._bufs = (ctypes.c_void_p * self.world)(*ptrs)
        from .ops import rope_table
        self.rope = rope_table(self.theta, self.frac, self.hd, self.S, torch.device("cuda", torch.cuda.current_device()))

    @property
    def local_tokens(self) -> int:
        return self.S // self.world

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, stream=None) -> torch.Tensor:
        """q: f32 [S/P, n_heads * hd], k, v: f32 [S/P, n_kv * hd] for this rank's tokens
        (positions rank*S/P ..). Returns f32 [S/P, n_heads * hd]; raises PyreTimeout if a
        peer did not arrive."""
        Sl = self.local_tokens
        for t, n in ((q, self.nq), (k, self.nkv), (v, self.nkv)):
            if t.dtype != torch.float32 or tuple(t.shape) != (Sl, n * self.hd) or t.stride(1) != 1:
                raise ValueError(f"q, k, v must be f32 [{Sl}, heads * {self.hd}] with unit column stride")
        if k.stride(0) != v.stride(0):
            raise ValueError("k and v must share a row stride")
        s = D.stream_ptr(stream)
        args = (self.S, self.nq, self.nkv, self.hd)
        N.call("pyre_ulysses_rope_scatter", self._bufs, self.rank, self.world, D.ptr(q), D.ptr(k), D.ptr(v),
               q.stride(0), k.stride(0), *args, D.ptr(self.rope), self.frac, s)
        N.call("pyre_ulysses_barrier", self._bufs, self.rank, self.world, *args, 0, self.timeout_ns, s)
        N.call("pyre_ulysses_attention", self._bufs, self.rank, self.world, *args, s)
        N.call("pyre_ulysses_barrier", self._bufs, self.rank, self.world, *args, 1, self.timeout_ns, s)
        out = torch.empty((Sl, self.nq * self.hd), dtype=torch.float32, device=q.device)
        st = ctypes.c_int(0)
        N.call("pyre_ulysses_finish", ctypes.c_void_p(self._local), self.world, *args, D.ptr(out), ctypes.byref(st), s)
        if st.value != N.PYRE_OK:
            raise N.PyreTimeout(st.value, f"rank {self.rank}: a Ulysses barrier wait timed out")
        return out

    def reset(self, group=None) -> None:
        """After a PyreTimeout: every rank calls this (host barrier, clear this rank's flags,
        epoch and status with pyre_ulysses_reset, host barrier) to start again in step."""
        import torch.distributed as dist
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=group)
        N.call("pyre_ulysses_reset", ctypes.c_void_p(self._local), self.world, self.S, self.nq, self.nkv, self.hd,
               D.stream_ptr())
        if self.world > 1:
            dist.barrier(group=group)

    def close(self) -> None:
        if self._local is None:
            return
        lib = N.load()
        torch.cuda.synchronize()
        for p in self._opened:
            lib.pyre_comm_close_peer(ctypes.c_void_p(p))
        lib.pyre_comm_free(ctypes.c_void_p(self._local))
        self._local = None
        self._opened = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
