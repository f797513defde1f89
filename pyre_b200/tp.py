"""Tensor-parallel group: one process per GPU, peer buffers over CUDA IPC.

This replaces the reference's star of TCP sockets between the root and its workers for
the FFN partial sum (src/orchestrator/root_node.py:164-180 handshake, :582-594 and
:982-995 gather-sum; src/orchestrator/net.py:18-48 framing). Inside one box every rank
exports one receive buffer (``pyre_comm_alloc``), the 64-byte IPC handles are exchanged
over ``torch.distributed`` (any backend: gloo or NCCL), and each rank maps the peers'
buffers into its own address space. The device kernels then push partials straight into
peers' memory over NVLink and wait on bounded flags.

The handle exchange and the shard bookkeeping are plain host logic, kept separate from
the CUDA calls so they can be tested with ``gloo`` ranks on the CPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Sequence

import torch
import torch.distributed as dist

from . import _native as N
from .partitioner import dirichlet_block_widths, widths_to_bounds

IPC_HANDLE_BYTES = 64


def dist_rank_world(group=None) -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def exchange_handles(local: bytes, group=None) -> List[bytes]:
    """All-gather one opaque byte string per rank (rank order)."""
    rank, world = dist_rank_world(group)
    if world == 1:
        return [bytes(local)]
    out: List[object] = [None] * world
    dist.all_gather_object(out, bytes(local), group=group)
    return [bytes(o) for o in out]


def gather_timings(t: float, group=None) -> List[float]:
    """Per-rank FFN times (seconds) gathered on every rank, for the adaptive partitioner."""
    rank, world = dist_rank_world(group)
    if world == 1:
        return [float(t)]
    out: List[object] = [None] * world
    dist.all_gather_object(out, float(t), group=group)
    return [float(o) for o in out]


@dataclass(frozen=True)
class ShardPlan:
    """Which slice of the intermediate dim each rank owns (identical on every rank)."""

    ffn_dim: int
    widths: tuple

    @property
    def bounds(self) -> List[tuple]:
        return widths_to_bounds(list(self.widths))

    @classmethod
    def dirichlet(cls, ffn_dim: int, world: int, alpha: float = 5.0, seed: int = 1, block: int = 32) -> "ShardPlan":
        return cls(ffn_dim, tuple(dirichlet_block_widths(ffn_dim, world, alpha, seed, block)))

    @classmethod
    def equal(cls, ffn_dim: int, world: int, block: int = 32) -> "ShardPlan":
        units = ffn_dim // block
        base, rem = divmod(units, world)
        return cls(ffn_dim, tuple((base + (1 if r < rem else 0)) * block for r in range(world)))

    @classmethod
    def from_partitions(cls, ffn_dim: int, parts: dict) -> "ShardPlan":
        """From a reference partition dict ``{rank: {"ffn_start", "ffn_end", ...}}``."""
        ids = sorted(parts)
        widths = []
        expect = 0
        for i in ids:
            s, e = parts[i]["ffn_start"], parts[i]["ffn_end"]
            if s != expect:
                raise ValueError("partitions must be contiguous and in rank order")
            widths.append(e - s)
            expect = e
        if expect != ffn_dim:
            raise ValueError("partitions must cover the whole intermediate dim")
        return cls(ffn_dim, tuple(widths))


class TPComm:
    """Peer-memory communicator of one rank (owns its receive buffer and peer mappings)."""

    def __init__(self, hidden: int, max_tokens: int = N.PYRE_FUSED_REDUCE_MAX_T, group=None,
                 timeout_s: float | None = None):
        lib = N.load()
        self.rank, self.world = dist_rank_world(group)
        self.hidden = int(hidden)
        self.max_tokens = int(max_tokens)
        nbytes = ctypes.c_int64(0)
        N.check(lib.pyre_comm_buffer_bytes(self.world, self.max_tokens, self.hidden, ctypes.byref(nbytes)))
        self.nbytes = int(nbytes.value)
        local = ctypes.c_void_p(0)
        handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        N.check(lib.pyre_comm_alloc(self.nbytes, ctypes.byref(local), handle))
        self._local = local.value
        self._opened: List[int] = []
        handles = exchange_handles(handle.raw, group)
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._local)
                continue
            p = ctypes.c_void_p(0)
            N.check(lib.pyre_comm_open_peer(ctypes.create_string_buffer(h, IPC_HANDLE_BYTES), ctypes.byref(p)))
            self._opened.append(p.value)
            ptrs.append(p.value)
        arr = (ctypes.c_void_p * self.world)(*ptrs)
        c = ctypes.c_void_p(0)
        N.check(lib.pyre_comm_create(self.rank, self.world, arr, self.max_tokens, self.hidden, ctypes.byref(c)))
        self._comm = c.value
        if timeout_s is not None:
            self.set_timeout(timeout_s)

    @property
    def handle(self) -> int:
        if self._comm is None:
            raise RuntimeError("TPComm is closed")
        return self._comm

    def set_timeout(self, seconds: float) -> None:
        N.call("pyre_comm_set_timeout_ns", ctypes.c_void_p(self.handle), int(seconds * 1e9))

    def check(self, stream: torch.cuda.Stream | None = None) -> None:
        """Synchronise and raise :class:`~pyre_b200._native.PyreTimeout` if any device
        wait on a peer ran out since the last check."""
        st = ctypes.c_int(0)
        s = stream if stream is not None else torch.cuda.current_stream()
        N.call("pyre_comm_check", ctypes.c_void_p(self.handle), ctypes.byref(st), ctypes.c_void_p(s.cuda_stream))
        if st.value != N.PYRE_OK:
            raise N.PyreTimeout(st.value, f"rank {self.rank}: a wait on a peer flag timed out")

    def reset(self, group=None) -> None:
        """Start every rank again from a common state after a wait ran out (PyreTimeout): all
        ranks call this; it waits for this rank's work, meets the others on the host, clears
        this rank's flags, epoch and status (pyre_comm_reset) and meets them again. Ops whose
        kernels stopped early also clear their own scratch (FfnShardOp.reset)."""
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=group)
        N.call("pyre_comm_reset", ctypes.c_void_p(self.handle), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        if self.world > 1:
            dist.barrier(group=group)

    def allreduce_(self, buf: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """In-place f32 sum over ranks (rank order) through peer memory."""
        if buf.dtype != torch.float32 or not buf.is_contiguous():
            raise ValueError("allreduce_ needs a contiguous float32 tensor")
        s = stream if stream is not None else torch.cuda.current_stream()
        N.call("pyre_allreduce_sum_f32", ctypes.c_void_p(self.handle), ctypes.c_void_p(buf.data_ptr()),
               buf.numel(), ctypes.c_void_p(s.cuda_stream))
        return buf

    def close(self) -> None:
        if self._comm is None:
            return
        lib = N.load()
        torch.cuda.synchronize()
        lib.pyre_comm_destroy(ctypes.c_void_p(self._comm))
        for p in self._opened:
            lib.pyre_comm_close_peer(ctypes.c_void_p(p))
        lib.pyre_comm_free(ctypes.c_void_p(self._local))
        self._comm = None
        self._opened = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def shard_weights(gate, up, down, bounds: Sequence[tuple], rank: int):
    """This rank's slices of full Q8_0 weights: gate/up columns, down rows."""
    s, e = bounds[rank]
    return (gate.cols(s, e) if gate is not None else None), up.cols(s, e), down.rows(s, e)
