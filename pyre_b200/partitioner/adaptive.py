"""Adaptive non-uniform FFN partitioner and drift detector.

Behaviour (the reference's ``AdaptivePartitioner``, src/orchestrator/cluster.py:228-403, and
``ClusterOrchestrator.detect_drift``, cluster.py:217-225), stated as rules:

* Timings. ``update({node: seconds})`` appends one FFN time per node for the current pass
  (unknown node ids are ignored); ``reset_pass()`` starts a new pass.
* Speed estimate. Folding a pass into the estimate takes each node's mean time m_i over the
  pass (nodes without timings are skipped), their plain mean M, and moves node i's relative
  speed e_i towards M / m_i: ``e_i <- e_i * (1 - alpha) + (M / max(m_i, 1e-9)) * alpha``,
  alpha = 0.3, all e_i starting at 1. Both ``drift_detected()`` (when the pass has timings)
  and ``get_partitions()`` fold the current pass in, each time they are called, as the
  reference does.
* Drift: some e_i above ``threshold`` (1.15) or below 1 / threshold.
* Widths. Node 0 (the root, whose time the reference cannot isolate) keeps
  ``units // n``. The other nodes split the rest R in proportion to e_i (``int(R * e_i /
  sum e)``; an even split if the sum is not positive), each clamped to [lo, R - (n - 2) lo]
  with lo = max(1, int(units * min_fraction / n)); a positive leftover goes to the fastest
  node (first of equals), an overdraft is taken from the slowest (first of equals) down to
  lo at most.
* Sequence split of the partition dicts (root_node.py:202-207): ``seq_len // n`` per node,
  the last node up to ``seq_len``.

Units are Q8_0 blocks of ``block`` elements (``block`` = 1 is the reference's element
granularity; 32 keeps every shard boundary on a Q8_0 block, which the device format needs).
The timings consumed here are per-rank CUDA-event FFN durations instead of TCP receive times.
"""
from __future__ import annotations

from typing import Dict, List


def detect_drift(execution_times: List[float], threshold: float = 1.15) -> bool:
    """True when some time is above ``threshold`` x the mean of all of them."""
    if not execution_times:
        return False
    limit = sum(execution_times) / len(execution_times) * threshold
    return any(t > limit for t in execution_times)


def _seq_range(node: int, n: int, seq_len: int) -> tuple:
    chunk = seq_len // n
    if node == n - 1:
        return (n - 1) * chunk, seq_len
    return node * chunk, (node + 1) * chunk


def split_in_proportion(total: int, weights: List[float], lo: int) -> List[int]:
    """``total`` units over len(weights) parts in proportion to the weights, each part clamped
    to [lo, total - (parts - 1) lo]; leftover units go to the heaviest part, an overdraft is
    taken from the lightest (not below lo)."""
    parts = len(weights)
    hi = total - (parts - 1) * lo
    wsum = sum(weights)
    shares = [int(total * w / wsum) for w in weights] if wsum > 0 else [total // parts] * parts
    shares = [max(lo, min(s, hi)) for s in shares]
    left = total - sum(shares)
    if left > 0:
        shares[weights.index(max(weights))] += left
    elif left < 0:
        k = weights.index(min(weights))
        shares[k] = max(lo, shares[k] + left)
    return shares


class AdaptivePartitioner:
    """Relative node speeds (an exponential moving average over passes) -> FFN shard widths."""

    def __init__(self, ffn_dim: int, num_nodes: int, seq_len: int = 64, min_fraction: float = 0.25,
                 max_fraction: float = 1.75, ema_alpha: float = 0.3, block: int = 1):
        if num_nodes < 1 or ffn_dim < num_nodes * block:
            raise ValueError("need at least one block of the FFN dim per node")
        if ffn_dim % block:
            raise ValueError(f"ffn_dim {ffn_dim} is not a multiple of the block {block}")
        self.ffn_dim, self.num_nodes, self.seq_len, self.block = ffn_dim, num_nodes, seq_len, block
        self.alpha = ema_alpha
        # max_fraction is accepted for signature parity: the reference derives an upper width
        # from it but never applies it, so the widths here do not depend on it either
        self.max_fraction = max_fraction
        self.units = ffn_dim // block
        self.min_units = max(1, int(self.units * min_fraction / num_nodes))
        self.ema: List[float] = [1.0] * num_nodes
        self._times: List[List[float]] = [[] for _ in range(num_nodes)]

    # ---- timings ------------------------------------------------------------------------
    def update(self, node_timings: Dict[int, float]) -> None:
        for node, t in node_timings.items():
            if 0 <= node < self.num_nodes:
                self._times[node].append(t)

    def reset_pass(self) -> None:
        self._times = [[] for _ in range(self.num_nodes)]

    def _fold_pass(self) -> None:
        means = [(i, sum(ts) / len(ts)) for i, ts in enumerate(self._times) if ts]
        if not means:
            return
        overall = sum(m for _, m in means) / len(means)
        a = self.alpha
        for i, m in means:
            self.ema[i] = self.ema[i] * (1 - a) + (overall / max(m, 1e-9)) * a

    # ---- decisions ----------------------------------------------------------------------
    def drift_detected(self, threshold: float = 1.15) -> bool:
        if not any(self._times):
            return False
        self._fold_pass()
        return any(e > threshold or e < 1.0 / threshold for e in self.ema)

    def get_partitions(self) -> Dict[int, dict]:
        """Partition dicts ``{node: {ffn_start, ffn_end, seq_start, seq_end}}`` for the next pass."""
        self._fold_pass()
        n = self.num_nodes
        if n == 1:
            widths = [self.units]
        else:
            root = self.units // n
            widths = [root] + split_in_proportion(self.units - root, self.ema[1:], self.min_units)
        parts, start = {}, 0
        for node, w in enumerate(widths):
            s0, s1 = _seq_range(node, n, self.seq_len)
            end = self.ffn_dim if n == 1 else (start + w) * self.block
            parts[node] = {"ffn_start": start * self.block, "ffn_end": end, "seq_start": s0, "seq_end": s1}
            start += w
        return parts

    def layer_partition(self, node_id: int, layer_idx: int) -> dict:
        """This node's dict from :meth:`get_partitions` (the reference ignores ``layer_idx`` too)."""
        return self.get_partitions().get(node_id, {})

    @staticmethod
    def equal_partitions(ffn_dim: int, num_nodes: int, seq_len: int = 64) -> Dict[int, dict]:
        """``ffn_dim // n`` per node, the last one up to ``ffn_dim`` (``RootNode._solve_partitions``)."""
        chunk = ffn_dim // num_nodes
        parts = {}
        for i in range(num_nodes):
            s0, s1 = _seq_range(i, num_nodes, seq_len)
            parts[i] = {"ffn_start": i * chunk, "ffn_end": ffn_dim if i == num_nodes - 1 else (i + 1) * chunk,
                        "seq_start": s0, "seq_end": s1}
        return parts
