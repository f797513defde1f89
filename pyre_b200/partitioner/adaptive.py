"""Adaptive non-uniform FFN partitioner and drift detector.

Restates ``AdaptivePartitioner`` (src/orchestrator/cluster.py:228-403) and
``ClusterOrchestrator.detect_drift`` (cluster.py:217-225) with the same names, defaults
(EMA alpha 0.3, drift threshold 1.15, width clamp [0.25, 1.75] x base) and partition dict
format (``ffn_start/ffn_end/seq_start/seq_end``, root_node.py:202-207). The timings it
consumes here are per-rank CUDA-event durations of the FFN kernels instead of TCP
receive wall times. ``block`` > 1 rounds widths to whole Q8_0 blocks after the
reference's allocation (the reference itself uses block = 1).
"""
from __future__ import annotations

from typing import Dict, List


def detect_drift(execution_times: List[float], threshold: float = 1.15) -> bool:
    """True when any time exceeds ``threshold`` x the mean (cluster.py:217-225)."""
    if not execution_times:
        return False
    avg_time = sum(execution_times) / len(execution_times)
    for t in execution_times:
        if t > avg_time * threshold:
            return True
    return False


class AdaptivePartitioner:
    """EMA of per-node relative speed -> non-uniform FFN widths (cluster.py:228-403)."""

    def __init__(self, ffn_dim: int, num_nodes: int, seq_len: int = 64,
                 min_fraction: float = 0.25, max_fraction: float = 1.75,
                 ema_alpha: float = 0.3, block: int = 1):
        self.ffn_dim = ffn_dim
        self.num_nodes = num_nodes
        self.seq_len = seq_len
        self.block = block
        self.base_width = ffn_dim // num_nodes
        self.min_width = max(1, int(ffn_dim * min_fraction / num_nodes))
        self.max_width = min(ffn_dim, int(ffn_dim * max_fraction / num_nodes))
        self.max_width = min(self.max_width, ffn_dim - (num_nodes - 1) * self.min_width)
        self.alpha = ema_alpha
        self.ema: List[float] = [1.0] * num_nodes
        self._layer_timings: Dict[int, List[float]] = {i: [] for i in range(num_nodes)}
        self._drift_counter = 0

    def update(self, node_timings: Dict[int, float]):
        for nid, t in node_timings.items():
            if nid in self._layer_timings:
                self._layer_timings[nid].append(t)

    def _recompute_ema(self):
        timings = {nid: ts for nid, ts in self._layer_timings.items() if ts}
        if not timings:
            return
        avg_times = {nid: sum(ts) / len(ts) for nid, ts in timings.items()}
        global_avg = sum(avg_times.values()) / len(avg_times)
        for nid, t in avg_times.items():
            relative = global_avg / max(t, 1e-9)
            self.ema[nid] = self.ema[nid] * (1 - self.alpha) + relative * self.alpha

    def drift_detected(self, threshold: float = 1.15) -> bool:
        if not self._has_data():
            return False
        self._recompute_ema()
        for v in self.ema:
            if v > threshold or v < 1.0 / threshold:
                return True
        return False

    def _has_data(self) -> bool:
        return any(len(ts) > 0 for ts in self._layer_timings.values())

    def get_partitions(self) -> Dict[int, dict]:
        self._recompute_ema()
        parts = self._allocate_partitions()
        return self._round_to_blocks(parts) if self.block > 1 else parts

    def _allocate_partitions(self) -> Dict[int, dict]:
        total_nodes = self.num_nodes
        seq_chunk = self.seq_len // total_nodes
        if total_nodes == 1:
            return {0: {"ffn_start": 0, "ffn_end": self.ffn_dim, "seq_start": 0, "seq_end": self.seq_len}}
        root_base = self.base_width
        remaining = self.ffn_dim - root_base
        worker_emas = self.ema[1:]
        total_worker_weight = sum(worker_emas)
        raw_widths = []
        for v in worker_emas:
            w = int(remaining * v / total_worker_weight) if total_worker_weight > 0 else remaining // (total_nodes - 1)
            raw_widths.append(max(self.min_width, min(w, remaining - (total_nodes - 2) * self.min_width)))
        clamped = [max(self.min_width, min(w, remaining - (total_nodes - 2) * self.min_width)) for w in raw_widths]
        allocated = sum(clamped)
        residual = remaining - allocated
        if residual > 0:
            fastest_wi = max(range(len(clamped)), key=lambda i: worker_emas[i])
            clamped[fastest_wi] += residual
        elif residual < 0:
            slowest_wi = min(range(len(clamped)), key=lambda i: worker_emas[i])
            clamped[slowest_wi] = max(self.min_width, clamped[slowest_wi] + residual)
        partitions: Dict[int, dict] = {0: {"ffn_start": 0, "ffn_end": root_base, "seq_start": 0, "seq_end": seq_chunk}}
        offset = root_base
        for wi, width in enumerate(clamped):
            nid = wi + 1
            partitions[nid] = {
                "ffn_start": offset,
                "ffn_end": offset + width,
                "seq_start": nid * seq_chunk if nid < total_nodes - 1 else (total_nodes - 1) * seq_chunk,
                "seq_end": (nid + 1) * seq_chunk if nid < total_nodes - 1 else self.seq_len,
            }
            offset += width
        return partitions

    def _round_to_blocks(self, parts: Dict[int, dict]) -> Dict[int, dict]:
        """Snap every interior boundary to the nearest block edge (keeping each width
        >= one block); the first start and the last end stay 0 and ffn_dim."""
        b = self.block
        ids = sorted(parts)
        ends = [parts[i]["ffn_end"] for i in ids]
        snapped = []
        prev = 0
        for k, e in enumerate(ends):
            if k == len(ends) - 1:
                e2 = self.ffn_dim
            else:
                e2 = int(round(e / b)) * b
                e2 = max(e2, prev + b)
                e2 = min(e2, self.ffn_dim - (len(ends) - 1 - k) * b)
            snapped.append(e2)
            prev = e2
        out, start = {}, 0
        for i, e in zip(ids, snapped):
            d = dict(parts[i])
            d["ffn_start"], d["ffn_end"] = start, e
            out[i] = d
            start = e
        return out

    def layer_partition(self, node_id: int, layer_idx: int) -> dict:
        return self.get_partitions().get(node_id, {})

    @staticmethod
    def equal_partitions(ffn_dim: int, num_nodes: int, seq_len: int = 64) -> Dict[int, dict]:
        seq_chunk = seq_len // num_nodes
        ffn_chunk = ffn_dim // num_nodes
        partitions = {}
        for i in range(num_nodes):
            partitions[i] = {
                "ffn_start": i * ffn_chunk,
                "ffn_end": (i + 1) * ffn_chunk if i < num_nodes - 1 else ffn_dim,
                "seq_start": i * seq_chunk,
                "seq_end": (i + 1) * seq_chunk if i < num_nodes - 1 else seq_len,
            }
        return partitions

    def reset_pass(self):
        self._layer_timings = {i: [] for i in range(self.num_nodes)}
