"""Glue between PyTorch tensors (device memory, streams) and the C ABI."""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N

_DTYPE_CODES = {torch.float32: N.PYRE_F32, torch.bfloat16: N.PYRE_BF16, torch.float16: N.PYRE_F16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError as e:
        raise ValueError(f"unsupported dtype {t.dtype}") from e


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream_ptr(stream: torch.cuda.Stream | None = None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def require_cuda() -> None:
    if not torch.cuda.is_available():
        raise RuntimeError("pyre_b200 needs a CUDA device (sm_100a); there is no CPU fallback")


def to_device(a, device=None, dtype: torch.dtype | None = None) -> torch.Tensor:
    """numpy array or tensor -> contiguous CUDA tensor (copy only when needed)."""
    require_cuda()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if isinstance(a, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(a))
    elif isinstance(a, torch.Tensor):
        t = a
    else:
        t = torch.as_tensor(a)
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    if t.device != dev:
        t = t.to(dev, non_blocking=False)
    return t.contiguous()
