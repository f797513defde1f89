"""Q8_0 block format on the device.

Mirrors ``src/orchestrator/quantizer.py`` (same names, argument meaning and tuple layout)
with the arithmetic done by the sm_100a kernels of ``libpyre_b200.so``:

* :func:`quantize_q80` / :func:`dequantize_q80` — ``quantizer.py:11-26`` / ``:29-40``;
  the quantized bits are identical to the reference's for finite inputs.
* :func:`quantize_activation` / :func:`dequantize_activation` — ``quantizer.py:54-67``.
* :func:`quantize_weights_dict` / :func:`dequantize_weights_dict` — ``quantizer.py:70-114``
  (``("q8", q, s, shape)`` tags, ``MIN_QUANTIZE_ELEMS`` threshold).

:class:`Q80Weight` is the GEMV/GEMM operand: the reference's Q8_0 blocks of a ``[K, N]``
weight (stored ``[in, out]``), laid out in column slabs of 256 (``q [NT, K, 256]`` int8,
``scale [NT, K, 8]`` f16 by default or f32), N zero-padded to a multiple of 256. Each
32-row unit of a slab is one contiguous 8 KB run that the kernels stream with bulk
copies; the int8 values and scales are exactly the reference's.
"""
from __future__ import annotations

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
SLAB_SCALES = SLAB // BLOCK


@dataclass
class Q80Weight:
    """A ``[K, N]`` weight in Q8_0, column-slab tiled on the device (see module doc)."""

    q: torch.Tensor       # [NT, K, 256] int8
    scale: torch.Tensor   # [NT, K, 8] f16 or f32
    n: int                # logical output width N

    @property
    def shape(self) -> Tuple[int, int]:
        return (int(self.q.shape[1]), int(self.n))

    @property
    def scale_code(self) -> int:
        return D.dtype_code(self.scale)

    @property
    def nbytes(self) -> int:
        """Bytes of the format proper (int8 + one scale per 32 weights, padding excluded)."""
        K, Nn = self.shape
        return K * Nn + K * (Nn // BLOCK) * self.scale.element_size()

    @classmethod
    def from_plain(cls, q: torch.Tensor, s: torch.Tensor) -> "Q80Weight":
        """From plain ``q [K, N]`` int8 and ``s [K, N/32]`` block scales (device tensors)."""
        K, Nn = q.shape
        if Nn % BLOCK or tuple(s.shape) != (K, Nn // BLOCK):
            raise ValueError("Q80Weight.from_plain: need q [K, N] with N % 32 == 0 and s [K, N/32]")
        nt = (Nn + SLAB - 1) // SLAB
        qp = torch.zeros((K, nt * SLAB), dtype=torch.int8, device=q.device)
        qp[:, :Nn] = q
        sp = torch.zeros((K, nt * SLAB_SCALES), dtype=s.dtype, device=s.device)
        sp[:, : Nn // BLOCK] = s
        return cls(qp.view(K, nt, SLAB).permute(1, 0, 2).contiguous(),
                   sp.view(K, nt, SLAB_SCALES).permute(1, 0, 2).contiguous(), Nn)

    def plain(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """Plain ``(q [K, N], s [K, N/32])`` views of the tiled storage (copies)."""
        nt, K, _ = self.q.shape
        q = self.q.permute(1, 0, 2).reshape(K, nt * SLAB)[:, : self.n]
        s = self.scale.permute(1, 0, 2).reshape(K, nt * SLAB_SCALES)[:, : self.n // BLOCK]
        return q.contiguous(), s.contiguous()

    @property
    def block_scales(self) -> torch.Tensor:
        return self.plain()[1]

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
        return cls.from_plain(q, s)

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
        return cls.from_plain(qt, st)

    def dequantize(self) -> torch.Tensor:
        K, Nn = self.shape
        q, s = self.plain()
        out = torch.empty((K, Nn), dtype=torch.float32, device=self.q.device)
        N.call("pyre_q80_dequantize", D.ptr(q), D.ptr(s), self.scale_code, K * Nn, D.ptr(out), D.stream_ptr())
        return out

    def to_tuple(self) -> tuple:
        """Reference tuple ``("q8", q [n_blocks, 32], scales [n_blocks], shape)`` (device tensors)."""
        q, s = self.plain()
        return ("q8", q.reshape(-1, BLOCK), s.reshape(-1), self.shape)

    def cols(self, start: int, end: int) -> "Q80Weight":
        """Columns [start, end) (a gate/up shard); both multiples of 32."""
        if start % BLOCK or end % BLOCK:
            raise ValueError("column shard bounds must be multiples of 32")
        q, s = self.plain()
        return Q80Weight.from_plain(q[:, start:end].contiguous(), s[:, start // BLOCK:end // BLOCK].contiguous())

    def rows(self, start: int, end: int) -> "Q80Weight":
        """Rows [start, end) (a down shard)."""
        return Q80Weight(self.q[:, start:end].contiguous(), self.scale[:, start:end].contiguous(), self.n)
