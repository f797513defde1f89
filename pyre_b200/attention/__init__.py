"""Attention path: builder interface (``src/attention/builder.py``) and the CUDA ops of the
attention block (projections, RoPE + KV cache, prefill and decode attention, RMSNorm)."""
from .builder import AttentionGraph, AttentionModel, ShardSpec, build_ulysses_attention_graph
from .ops import AttentionOp, KVCache, Q80Linear, q80_linear, rms_norm, softmax
from .ulysses import UlyssesAttention

__all__ = ["AttentionGraph", "AttentionModel", "ShardSpec", "build_ulysses_attention_graph", "AttentionOp",
           "KVCache", "Q80Linear", "q80_linear", "rms_norm", "softmax", "UlyssesAttention"]
