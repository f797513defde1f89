"""Q8_0 block format on the device.

Mirrors ``src/orchestrator/quantizer.py`` (same names, argument meaning and tuple layout)
with the arithmetic done by the sm_100a kernels of ``libpyre_b200.so``:

* :func:`quantize_q80` / :func:`dequantize_q80` — ``quantizer.py:11-26`` / ``:29-40``;
  the quantized bits are identical to the reference's for finite inputs.
* :func:`quantize_activation` / :func:`dequantize_activation` — ``quantizer.py:54-67``.
* :func:`quantize_weights_dict` / :func:`dequantize_weights_dict` — ``quantizer.py:70-114``
  (``("q8", q, s, shape)`` tags, ``MIN_QUANTIZE_ELEMS`` threshold).

:class:`Q80Weight` holds one ``[K, N]`` weight (stored ``[in, out]`` like the reference) as
its Q8_0 blocks in the reference orientation: ``q [K, N]`` int8 and ``scale [K, N/32]`` (f16
by default, f32 for the exact-scale variant). :class:`Q80Packed` is the kernels' operand:
one or two such weights (gate and up) in the packed block layout of ``include/pyre_b200.h``
(one ~17 KB block per 256-column slab and 64/M-row unit, streamed with one bulk copy).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Tuple

import numpy as np
import torch

from . import _device as D
from . import _native as N

MIN_QUANTIZE_ELEMS = 4096
BLOCK = 32


def _flat_f32_or_bf16(arr) -> torch.Tensor:
    t = D.to_device(arr)
    if t.dtype not in (torch.float32, torch.bfloat16):
        t = t.to(torch.float32)
    return t.reshape(-1)


def quantize_q80(arr, block_size: int = BLOCK) -> Tuple[torch.Tensor, torch.Tensor, Tuple[int, ...]]:
    """Quantize to Q8_0 (block int8 + f32 scale) on the GPU.

    Returns ``(qdata [n_blocks, 32] int8, scales [n_blocks] f32, orig_shape)`` as CUDA
    tensors, bit-identical to ``quantize_q80`` of ``src/orchestrator/quantizer.py:11-26``.
    """
    if block_size != BLOCK:
        raise ValueError(f"Q8_0 uses 32-element blocks; block_size={block_size} is not supported")
    orig_shape = tuple(arr.shape)
    flat = _flat_f32_or_bf16(arr)
    n = flat.numel()
    n_blocks = (n + BLOCK - 1) // BLOCK
    q = torch.empty((n_blocks, BLOCK), dtype=torch.int8, device=flat.device)
    s = torch.empty((n_blocks,), dtype=torch.float32, device=flat.device)
    N.call("pyre_q80_quantize", D.ptr(flat), D.dtype_code(flat), n, D.ptr(q), D.ptr(s), None, D.stream_ptr())
    return q, s, orig_shape


def dequantize_q80(qdata, scales, orig_shape: Tuple[int, ...]) -> torch.Tensor:
    """Dequantize Q8_0 back to float32 on the GPU (``quantizer.py:29-40``)."""
    q = D.to_device(qdata, dtype=torch.int8).reshape(-1)
    s = D.to_device(scales)
    if s.dtype not in (torch.float32, torch.float16):
        s = s.to(torch.float32)
    total = int(np.prod(orig_shape)) if len(orig_shape) else 1
    n_blocks = s.numel()
    if n_blocks == 0 or q.numel() % n_blocks != 0 or q.numel() // n_blocks != BLOCK:
        raise ValueError("dequantize_q80: qdata must hold 32 int8 values per scale")
    if total > q.numel():
        raise ValueError("dequantize_q80: orig_shape larger than the quantized data")
    out = torch.empty(total, dtype=torch.float32, device=q.device)
    N.call("pyre_q80_dequantize", D.ptr(q), D.ptr(s), D.dtype_code(s), total, D.ptr(out), D.stream_ptr())
    return out.reshape(orig_shape)


def quantize_to_f16(arr) -> tuple:
    """``("f16", arr.astype(float16), shape)`` as in ``quantizer.py:43-45``."""
    t = D.to_device(arr)
    return ("f16", t.to(torch.float16), tuple(t.shape))


def dequantize_from_f16(data: tuple) -> torch.Tensor:
    _, arr, shape = data
    return D.to_device(arr).to(torch.float32).reshape(shape).contiguous()


def quantize_activation(arr) -> tuple:
    """Q8_0 activation tuple ``(qdata, scales, orig_shape)`` (``quantizer.py:54-61``)."""
    return quantize_q80(arr)


def dequantize_activation(data: tuple) -> torch.Tensor:
    qdata, scales, orig_shape = data
    return dequantize_q80(qdata, scales, orig_shape)


def quantize_weights_dict(weights: dict, mode: str = "q8") -> dict:
    """Recursively quantize every array with >= MIN_QUANTIZE_ELEMS elements
    (``quantizer.py:70-87``); smaller ones (norms, biases) pass through."""
    qd = {}
    for k, v in weights.items():
        if isinstance(v, dict):
            qd[k] = quantize_weights_dict(v, mode=mode)
        elif isinstance(v, (np.ndarray, torch.Tensor)) and _numel(v) >= MIN_QUANTIZE_ELEMS:
            if mode == "f16":
                qd[k] = quantize_to_f16(v)
            else:
                q, s, sh = quantize_q80(v)
                qd[k] = ("q8", q, s, sh)
        else:
            qd[k] = v
    return qd


def dequantize_weights_dict(qd: dict, subset: str = "") -> dict:
    """Inverse of :func:`quantize_weights_dict` (``quantizer.py:90-114``)."""
    result = {}
    for k, v in qd.items():
        if subset and k != subset:
            result[k] = v
            continue
        if isinstance(v, dict):
            result[k] = dequantize_weights_dict(v)
        elif isinstance(v, tuple):
            tag = v[0]
            if tag == "q8":
                _, q, s, sh = v
                result[k] = dequantize_q80(q, s, sh)
            elif tag == "f16":
                result[k] = dequantize_from_f16(v)
            else:
                result[k] = v
        else:
            result[k] = v
    return result


def _numel(v) -> int:
    return int(v.numel()) if isinstance(v, torch.Tensor) else int(v.size)


SLAB = 256


@dataclass
class Q80Weight:
    """A ``[K, N]`` weight in Q8_0 on the device: ``q [K, N]`` int8, ``scale [K, N/32]``."""

    q: torch.Tensor
    scale: torch.Tensor

    def __post_init__(self):
        K, Nn = self.q.shape
        if Nn % BLOCK or tuple(self.scale.shape) != (K, Nn // BLOCK):
            raise ValueError("Q80Weight needs q [K, N] with N % 32 == 0 and scale [K, N/32]")

    @property
    def shape(self) -> Tuple[int, int]:
        return tuple(self.q.shape)

    @property
    def scale_code(self) -> int:
        return D.dtype_code(self.scale)

    @property
    def nbytes(self) -> int:
        return self.q.numel() + self.scale.numel() * self.scale.element_size()

    @classmethod
    def from_float(cls, w, scale_dtype: torch.dtype = torch.float16) -> "Q80Weight":
        """Quantize a float ``[K, N]`` weight (N % 32 == 0) on the device."""
        t = D.to_device(w)
        if t.dim() != 2:
            raise ValueError("Q80Weight.from_float expects a 2-D [K, N] weight")
        K, Nn = t.shape
        if Nn % BLOCK != 0:
            raise ValueError(f"output width {Nn} must be a multiple of 32")
        if t.dtype not in (torch.float32, torch.bfloat16):
            t = t.to(torch.float32)
        if scale_dtype not in (torch.float16, torch.float32):
            raise ValueError("scale_dtype must be torch.float16 or torch.float32")
        q = torch.empty((K, Nn), dtype=torch.int8, device=t.device)
        s = torch.empty((K, Nn // BLOCK), dtype=scale_dtype, device=t.device)
        s32 = s if scale_dtype == torch.float32 else None
        s16 = s if scale_dtype == torch.float16 else None
        N.call("pyre_q80_quantize", D.ptr(t), D.dtype_code(t), K * Nn, D.ptr(q), D.ptr(s32), D.ptr(s16),
               D.stream_ptr())
        return cls(q, s)

    @classmethod
    def from_tuple(cls, tup, scale_dtype: torch.dtype | None = None) -> "Q80Weight":
        """From a reference tuple ``("q8", q, s, shape)`` or ``(q, s, shape)`` of a 2-D weight."""
        if len(tup) == 4:
            _, q, s, shape = tup
        else:
            q, s, shape = tup
        if len(shape) != 2 or shape[1] % BLOCK != 0:
            raise ValueError("Q80Weight.from_tuple needs a 2-D weight whose last dim is a multiple of 32")
        K, Nn = shape
        qt = D.to_device(q, dtype=torch.int8).reshape(K, Nn)
        st = D.to_device(s).reshape(K, Nn // BLOCK)
        if scale_dtype is not None:
            st = st.to(scale_dtype)
        elif st.dtype not in (torch.float16, torch.float32):
            st = st.to(torch.float32)
        return cls(qt.contiguous(), st.contiguous())

    def dequantize(self) -> torch.Tensor:
        K, Nn = self.shape
        out = torch.empty((K, Nn), dtype=torch.float32, device=self.q.device)
        N.call("pyre_q80_dequantize", D.ptr(self.q), D.ptr(self.scale), self.scale_code, K * Nn, D.ptr(out),
               D.stream_ptr())
        return out

    def to_tuple(self) -> tuple:
        """Reference tuple ``("q8", q [n_blocks, 32], scales [n_blocks], shape)`` (device tensors)."""
        return ("q8", self.q.reshape(-1, BLOCK), self.scale.reshape(-1), self.shape)

    def cols(self, start: int, end: int) -> "Q80Weight":
        """Columns [start, end) (a gate/up shard); both multiples of 32."""
        if start % BLOCK or end % BLOCK:
            raise ValueError("column shard bounds must be multiples of 32")
        return Q80Weight(self.q[:, start:end].contiguous(), self.scale[:, start // BLOCK:end // BLOCK].contiguous())

    def rows(self, start: int, end: int) -> "Q80Weight":
        """Rows [start, end) (a down shard)."""
        return Q80Weight(self.q[start:end].contiguous(), self.scale[start:end].contiguous())


@dataclass
class Q80Packed:
    """One weight (M = 1) or a gate/up pair (M = 2) in the packed block layout."""

    data: torch.Tensor      # uint8, pyre_q80_packed_bytes() bytes
    m: int
    k: int
    n: int
    scale_dtype: torch.dtype

    @property
    def scale_code(self) -> int:
        return N.PYRE_F16 if self.scale_dtype == torch.float16 else N.PYRE_F32

    @property
    def nbytes_payload(self) -> int:
        """Q8_0 bytes of the packed weights (padding excluded)."""
        es = 2 if self.scale_dtype == torch.float16 else 4
        return self.m * (self.k * self.n + self.k * (self.n // BLOCK) * es)

    @classmethod
    def pack(cls, weights) -> "Q80Packed":
        """Pack one Q80Weight, or a (gate, up) pair sharing shape and scale dtype."""
        ws = list(weights) if isinstance(weights, (list, tuple)) else [weights]
        if len(ws) not in (1, 2):
            raise ValueError("pack one weight or a (gate, up) pair")
        K, Nn = ws[0].shape
        for w in ws[1:]:
            if w.shape != (K, Nn) or w.scale.dtype != ws[0].scale.dtype:
                raise ValueError("packed matrices must share shape and scale dtype")
        code = ws[0].scale_code
        nbytes = ctypes.c_int64(0)
        N.call("pyre_q80_packed_bytes", len(ws), K, Nn, code, ctypes.byref(nbytes))
        out = torch.empty(int(nbytes.value), dtype=torch.uint8, device=ws[0].q.device)
        q1 = ws[1].q if len(ws) == 2 else None
        s1 = ws[1].scale if len(ws) == 2 else None
        N.call("pyre_q80_pack", len(ws), D.ptr(ws[0].q), D.ptr(ws[0].scale), D.ptr(q1), D.ptr(s1), K, Nn, code,
               D.ptr(out), D.stream_ptr())
        return cls(out, len(ws), K, Nn, ws[0].scale.dtype)
