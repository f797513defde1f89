"""Attention-path ops on the CUDA kernels of this library.

* :func:`q80_linear` — ``x @ W`` on packed Q8_0 weights (the Q/K/V/O projections).
* :func:`rms_norm`, :func:`softmax` — pyre_kernels.mojo:18-58 on the GPU.
* :class:`KVCache` — one layer's f16 K/V cache ``[n_kv, max_t, hd]``, preallocated (the
  reference grows numpy arrays by concatenation every step, root_node.py:919-929).
* :class:`AttentionOp` — RoPE + clip + cache append, then causal prefill attention
  (root_node.py:250-314) or one-token decode attention (root_node.py:900-933, :1009-1031).
"""
from __future__ import annotations

import ctypes
import math

import torch

from .. import _device as D
from .. import _native as N
from ..quantizer import Q80Packed, Q80Weight


def _workspace(tokens: int, k: int, n: int, device) -> torch.Tensor:
    b = ctypes.c_int64(0)
    N.call("pyre_ffn_workspace_bytes", int(tokens), int(k), int(n), ctypes.byref(b))
    return torch.zeros(int(b.value), dtype=torch.uint8, device=device)


class Q80Linear:
    """``out[T, N] = x[T, K] @ W (+ bias)`` for a packed single Q8_0 matrix, up to
    ``max_tokens`` rows per call; holds the kernels' zero-initialised scratch. ``bias`` (f32
    [N], optional) is added to the finished f32 products in the kernels' epilogue, as the
    reference adds q_bias / k_bias / v_bias right after the projections
    (src/orchestrator/root_node.py:443-451)."""

    def __init__(self, weight: Q80Weight | Q80Packed, max_tokens: int, device=None, bias=None):
        self.w = weight if isinstance(weight, Q80Packed) else Q80Packed.pack(weight)
        if self.w.m != 1:
            raise ValueError("Q80Linear takes one matrix")
        self.k, self.n = self.w.k, self.w.n
        self.max_tokens = int(max_tokens)
        dev = device if device is not None else self.w.data.device
        self.workspace = _workspace(self.max_tokens, self.k, self.n, dev)
        self.bias = None
        if bias is not None:
            b = torch.as_tensor(bias).detach().to(dev, torch.float32).reshape(-1).contiguous()
            if b.numel() != self.n:
                raise ValueError(f"bias must have {self.n} elements, got {b.numel()}")
            self.bias = b

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        if x.dim() != 2 or x.shape[1] != self.k:
            raise ValueError(f"x must be [T, {self.k}], got {tuple(x.shape)}")
        T = x.shape[0]
        if T < 1 or T > self.max_tokens:
            raise ValueError(f"T={T} outside [1, {self.max_tokens}]")
        x = x.contiguous()
        if out is None:
            out = torch.empty((T, self.n), dtype=torch.float32, device=x.device)
        ws = self.workspace
        N.call("pyre_q80_linear_bias", D.ptr(x), D.dtype_code(x), T, self.k, D.ptr(self.w.data), self.w.scale_code,
               self.n, D.ptr(self.bias) if self.bias is not None else None, D.ptr(out), D.ptr(ws), ws.numel(),
               D.stream_ptr(stream))
        return out


def q80_linear(x: torch.Tensor, weight: Q80Weight | Q80Packed, stream=None) -> torch.Tensor:
    """One-off ``x @ W`` (allocates its scratch; use :class:`Q80Linear` on a hot path)."""
    return Q80Linear(weight, x.shape[0], x.device)(x, stream=stream)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, stream=None) -> torch.Tensor:
    """pyre_kernels.mojo:18-35 on f32 ``[..., H]``."""
    x = x.contiguous().float()
    w = weight.contiguous().float()
    H = x.shape[-1]
    out = torch.empty_like(x)
    N.call("pyre_rms_norm", D.ptr(x), x.numel() // H, H, D.ptr(w), float(eps), D.ptr(out), D.stream_ptr(stream))
    return out


def softmax(x: torch.Tensor, stream=None) -> torch.Tensor:
    """pyre_kernels.mojo:39-58 over the last axis of an f32 tensor."""
    x = x.contiguous().float()
    C = x.shape[-1]
    out = torch.empty_like(x)
    N.call("pyre_softmax_rows", D.ptr(x), x.numel() // C, C, D.ptr(out), D.stream_ptr(stream))
    return out


def rope_table(theta: float, rope_fraction: float, head_dim: int, n_pos: int, device) -> torch.Tensor:
    """cos/sin of pos * freq_i for positions 0..n_pos-1 (pyre_kernels.mojo:86-89: freq_i =
    1 / theta^(2i/dims) and the angle in f64, cast to f32), as f32 [n_pos, dims/2, 2] on the
    device; an empty tensor when nothing is rotated."""
    dims = int(float(head_dim) * float(rope_fraction))
    half = dims // 2 if dims >= 2 else 0
    host = torch.empty((max(n_pos, 1), max(half, 1), 2), dtype=torch.float32)
    N.call("pyre_rope_table", float(theta), float(rope_fraction), int(head_dim), int(n_pos),
           ctypes.c_void_p(host.data_ptr()))
    return host.to(device)


class KVCache:
    """One layer's K and V cache, f16 ``[n_kv, max_t, hd]`` (values clipped to +-1000)."""

    def __init__(self, n_kv: int, max_t: int, head_dim: int, device=None, k=None, v=None):
        """``k`` / ``v``: existing contiguous f16 ``[n_kv, max_t, hd]`` tensors to use (a slice of
        a batch's stacked caches) instead of new ones."""
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        if k is None:
            k = torch.zeros((n_kv, max_t, head_dim), dtype=torch.float16, device=dev)
            v = torch.zeros_like(k)
        if tuple(k.shape) != (n_kv, max_t, head_dim) or k.shape != v.shape or not (k.is_contiguous() and v.is_contiguous()):
            raise ValueError("cache tensors must be contiguous f16 [n_kv, max_t, head_dim]")
        self.k, self.v = k, v
        self.n_kv, self.max_t, self.head_dim = n_kv, max_t, head_dim
        self.length = 0


class AttentionOp:
    """Attention of one layer (one sequence) over a preallocated :class:`KVCache`."""

    def __init__(self, n_heads: int, n_kv_heads: int, head_dim: int, max_t: int, rope_theta: float = 10000.0,
                 rope_fraction: float = 1.0, device=None, cache: KVCache | None = None,
                 rope: torch.Tensor | None = None):
        if n_heads % n_kv_heads:
            raise ValueError("n_heads must be a multiple of n_kv_heads")
        if head_dim not in (64, 128):
            raise ValueError("head_dim must be 64 or 128")
        self.nq, self.nkv, self.hd = n_heads, n_kv_heads, head_dim
        self.theta, self.frac = float(rope_theta), float(rope_fraction)
        self.cache = cache if cache is not None else KVCache(n_kv_heads, max_t, head_dim, device)
        self.rope = rope if rope is not None else rope_table(self.theta, self.frac, head_dim, max_t,
                                                             self.cache.k.device)
        b = ctypes.c_int64(0)
        N.call("pyre_attn_decode_workspace_bytes", n_heads, n_kv_heads, head_dim, max_t, ctypes.byref(b))
        self.dec_ws = torch.zeros(int(b.value), dtype=torch.uint8, device=self.cache.k.device)

    def reset(self) -> None:
        self.cache.length = 0

    def _append(self, q, k, v, stream):
        T = q.shape[0]
        for t, n in ((q, self.nq), (k, self.nkv), (v, self.nkv)):
            if t.dtype != torch.float32 or t.dim() != 2 or t.shape[1] != n * self.hd or t.stride(1) != 1:
                raise ValueError(f"q, k, v must be f32 [T, heads * {self.hd}] with unit column stride")
        if k.stride(0) != v.stride(0):
            raise ValueError("k and v must share a row stride")
        start = self.cache.length
        if start + T > self.cache.max_t:
            raise ValueError("KV cache full")
        q_out = torch.empty((self.nq, T, self.hd), dtype=torch.float16, device=q.device)
        N.call("pyre_rope_kv_append", D.ptr(q), D.ptr(k), D.ptr(v), q.stride(0), k.stride(0), T, self.nq, self.nkv,
               self.hd, start, D.ptr(self.rope), self.frac, D.ptr(q_out), D.ptr(self.cache.k), D.ptr(self.cache.v),
               self.cache.max_t, D.stream_ptr(stream))
        self.cache.length = start + T
        return q_out

    def prefill(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, stream=None) -> torch.Tensor:
        """Causal attention of T tokens at positions 0..T-1 (the cache must be empty);
        returns f32 ``[T, n_heads * head_dim]``."""
        if self.cache.length != 0:
            raise ValueError("prefill starts from an empty cache (call reset())")
        T = q.shape[0]
        q_out = self._append(q, k, v, stream)
        out = torch.empty((T, self.nq * self.hd), dtype=torch.float32, device=q.device)
        N.call("pyre_attn_prefill", D.ptr(q_out), D.ptr(self.cache.k), D.ptr(self.cache.v), T, self.nq, self.nkv,
               self.hd, self.cache.max_t, D.ptr(out), D.stream_ptr(stream))
        return out

    def decode(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, prefill_real: int = 0,
               prefill_max_seq: int = 0, stream=None) -> torch.Tensor:
        """One token at position = cache length; positions in [prefill_real,
        prefill_max_seq) of the cache are masked. Returns f32 ``[1, n_heads * head_dim]``."""
        if q.shape[0] != 1:
            raise ValueError("decode takes one token")
        for x, n in ((q, self.nq), (k, self.nkv), (v, self.nkv)):
            if x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != n * self.hd or not x.is_contiguous():
                raise ValueError(f"q, k, v must be contiguous f32 [1, heads * {self.hd}]")
        start = self.cache.length
        if start + 1 > self.cache.max_t:
            raise ValueError("KV cache full")
        out = torch.empty((1, self.nq * self.hd), dtype=torch.float32, device=q.device)
        lo, hi = (int(prefill_real), int(prefill_max_seq)) if prefill_max_seq > prefill_real else (0, 0)
        ws = self.dec_ws
        # RoPE + clip + KV append + flash-decoding in one launch
        N.call("pyre_attn_decode_step", D.ptr(q), D.ptr(k), D.ptr(v), start, D.ptr(self.rope), self.frac, self.nq,
               self.nkv, self.hd, D.ptr(self.cache.k), D.ptr(self.cache.v), self.cache.max_t, lo, hi, D.ptr(out),
               D.ptr(ws), ws.numel(), D.stream_ptr(stream))
        self.cache.length = start + 1
        return out
