"""FFN shard: builder interface (``src/ffn/builder.py``) over the Q8_0 CUDA kernels."""
from .builder import FfnGraph, FfnModel, ShardSpec, build_ffn_graph, compile_and_run
from .op import FfnShardOp, FfnWeights, workspace_bytes

__all__ = ["FfnGraph", "FfnModel", "ShardSpec", "build_ffn_graph", "compile_and_run", "FfnShardOp",
           "FfnWeights", "workspace_bytes"]
