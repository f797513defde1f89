"""FLOPs-proportional split of the FFN intermediate dim over nodes.

Restates ``solve_partitions`` of ``src/partitioner/solver.mojo:30-52`` (a Mojo file; the
logic is plain host arithmetic, so it lives in Python here):
``size_i = max(1, int(flops_i / sum(flops) * ffn_dim))`` and the last node takes the
remainder. ``block`` > 1 additionally rounds every width to whole Q8_0 blocks (the
device GEMV wants shard boundaries on 32-element block edges).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List

import numpy as np


@dataclass
class NodeCap:
    """``NodeCap`` of solver.mojo:1-13 / cluster.py:14-20."""

    id: int
    flops_gflops: float
    mem_bytes: int
    net_bps: float
    barrier_latency_us: float


@dataclass
class ShardSpec:
    """``ShardSpec`` of solver.mojo:15-28."""

    start: int
    end: int
    seq_start: int = 0
    seq_end: int = 0

    def size(self) -> int:
        return self.end - self.start


def solve_partitions(nodes: List[NodeCap], ffn_dim: int, block: int = 1) -> Dict[int, ShardSpec]:
    if not nodes:
        raise ValueError("solve_partitions: need at least one node")
    if block > 1 and ffn_dim % block:
        raise ValueError(f"ffn_dim {ffn_dim} is not a multiple of block {block}")
    total_flops = 0.0
    for n in nodes:
        total_flops += n.flops_gflops
    units = ffn_dim // block
    partitions: Dict[int, ShardSpec] = {}
    current = 0
    for i, n in enumerate(nodes):
        if i == len(nodes) - 1:
            size = units - current
        else:
            fraction = n.flops_gflops / total_flops
            size = max(1, int(fraction * float(units)))
        end = current + size
        partitions[n.id] = ShardSpec(current * block, end * block)
        current = end
    return partitions


def dirichlet_block_widths(ffn_dim: int, n: int, alpha: float = 5.0, seed: int = 1, block: int = 32) -> List[int]:
    """Non-uniform widths: ratios ~ Dirichlet(alpha) rounded to whole blocks.

    ``r = default_rng(seed).dirichlet([alpha]*n)``; ``blocks_p = floor(r_p * ffn_dim/block)``;
    the leftover blocks go one each to the largest fractional parts; every rank keeps at
    least one block. Returns widths (multiples of ``block``) summing to ``ffn_dim``.
    """
    if ffn_dim % block:
        raise ValueError(f"ffn_dim {ffn_dim} is not a multiple of {block}")
    total = ffn_dim // block
    if n < 1 or n > total:
        raise ValueError(f"cannot split {total} blocks over {n} ranks")
    if n == 1:
        return [ffn_dim]
    r = np.random.default_rng(seed).dirichlet([alpha] * n)
    raw = r * total
    blocks = np.floor(raw).astype(np.int64)
    frac = raw - blocks
    left = total - int(blocks.sum())
    for idx in np.argsort(-frac, kind="stable")[:left]:
        blocks[idx] += 1
    # every rank keeps at least one block: take from the largest
    for i in range(n):
        while blocks[i] < 1:
            j = int(np.argmax(blocks))
            blocks[j] -= 1
            blocks[i] += 1
    return [int(b) * block for b in blocks]


def widths_to_bounds(widths: List[int]) -> List[tuple]:
    out, s = [], 0
    for w in widths:
        out.append((s, s + w))
        s += w
    return out
