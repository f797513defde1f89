"""Non-uniform FFN partitioner and drift detector (src/partitioner, src/orchestrator/cluster.py)."""
from .adaptive import AdaptivePartitioner, detect_drift
from .solver import NodeCap, ShardSpec, dirichlet_block_widths, solve_partitions, widths_to_bounds

__all__ = ["AdaptivePartitioner", "detect_drift", "NodeCap", "ShardSpec", "solve_partitions",
           "dirichlet_block_widths", "widths_to_bounds"]
