"""ctypes binding of ``libpyre_b200.so`` (the C ABI declared in ``include/pyre_b200.h``).

There is no fallback: if the library is missing or cannot be loaded, every entry point
raises. Status codes become exceptions carrying the library's last-error text.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

PYRE_OK = 0
PYRE_EINVAL = 1
PYRE_ECUDA = 2
PYRE_ETIMEOUT = 3
PYRE_ENOMEM = 4
PYRE_ERANGE = 5
PYRE_NOALLOC_SCRATCH_BYTES = 4 << 20

PYRE_F32 = 0
PYRE_BF16 = 1
PYRE_F16 = 2

PYRE_FUSED_REDUCE_MAX_T = 4

LIB_PATH = Path(__file__).resolve().parent / "libpyre_b200.so"


class PyreError(RuntimeError):
    """A pyre_b200 C-ABI call returned a non-zero status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[pyre status {code}] {msg}")
        self.code = code


class PyreTimeout(PyreError):
    """A device-side wait on a peer flag ran out (PYRE_ETIMEOUT)."""


_c_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_i = ctypes.c_int

# name -> argtypes (every function returns int)
_SIGNATURES = {
    "pyre_version": [],
    "pyre_last_error": [ctypes.c_char_p, _i],
    "pyre_q80_quantize": [_vp, _i, _c_i64, _vp, _vp, _vp, _vp],
    "pyre_q80_dequantize": [_vp, _vp, _i, _c_i64, _vp, _vp],
    "pyre_ffn_workspace_bytes": [_i, _i, _i, ctypes.POINTER(_c_i64)],
    "pyre_q80_packed_bytes": [_i, _i, _i, _i, ctypes.POINTER(_c_i64)],
    "pyre_q80_pack": [_i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp],
    "pyre_ffn_gateup_silu_q80": [_vp, _i, _i, _i, _vp, _i, _i, _i, _vp, _i, _vp, _c_i64, _vp],
    "pyre_ffn_down_q80": [_vp, _i, _i, _i, _vp, _i, _i, _vp, _vp, _c_i64, _vp, _vp],
    "pyre_ffn_decode_q80": [_vp, _i, _i, _i, _vp, _i, _vp, _i, _i, _vp, _vp, _c_i64, _vp, _vp],
    "pyre_ffn_decode_q80_noalloc": [_vp, _i, _i, _i, _vp, _i, _vp, _i, _i, _vp, _vp],
    "pyre_ffn_decode_q80_noalloc_status": [ctypes.POINTER(_i), _vp],
    "pyre_comm_buffer_bytes": [_i, _i, _i, ctypes.POINTER(_c_i64)],
    "pyre_comm_alloc": [_c_i64, ctypes.POINTER(_vp), _vp],
    "pyre_comm_free": [_vp],
    "pyre_comm_open_peer": [_vp, ctypes.POINTER(_vp)],
    "pyre_comm_close_peer": [_vp],
    "pyre_comm_create": [_i, _i, ctypes.POINTER(_vp), _i, _i, ctypes.POINTER(_vp)],
    "pyre_comm_destroy": [_vp],
    "pyre_comm_set_timeout_ns": [_vp, ctypes.c_uint64],
    "pyre_comm_check": [_vp, ctypes.POINTER(_i), _vp],
    "pyre_comm_reset": [_vp, _vp],
    "pyre_ulysses_reset": [_vp, _i, _i, _i, _i, _i, _vp],
    "pyre_allreduce_sum_f32": [_vp, _vp, _c_i64, _vp],
    "pyre_q80_linear": [_vp, _i, _i, _i, _vp, _i, _i, _vp, _vp, _c_i64, _vp],
    "pyre_q80_linear_bias": [_vp, _i, _i, _i, _vp, _i, _i, _vp, _vp, _vp, _c_i64, _vp],
    "pyre_argmax_combine": [_vp, _vp, _i, _vp, _vp, _vp],
    "pyre_rms_norm": [_vp, _i, _i, _vp, ctypes.c_double, _vp, _vp],
    "pyre_add_rms_norm": [_vp, _vp, _i, _i, _vp, ctypes.c_double, _vp, _vp, _vp],
    "pyre_decoder_step": [_vp, _vp, _i, _i, _i, _vp, _vp, _vp],
    "pyre_attn_decode_step_dev": [_vp, _vp, _vp, _vp, _i, _vp, ctypes.c_double, _i, _i, _i, _vp, _vp, _i, _i, _i,
                                  _vp, _vp, _c_i64, _vp],
    "pyre_attn_decode_step_batch": [_vp, _vp, _vp, _c_i64, _i, _vp, _i, _vp, ctypes.c_double, _i, _i, _i, _vp, _vp,
                                    _i, _vp, _vp, _c_i64, _vp],
    "pyre_decoder_struct_sizes": [_vp, _vp],
    "pyre_decoder_persistent_workspace_bytes": [_vp, ctypes.POINTER(_c_i64)],
    "pyre_decoder_persistent_status": [_vp, ctypes.POINTER(_i)],
    "pyre_decoder_step_persistent": [_vp, _vp, _c_i64, _vp, _i, _vp, _vp, _vp],
    "pyre_embed_rms_norm": [_vp, _i, _vp, _i, _i, _vp, ctypes.c_double, _vp, _vp, _vp, _vp],
    "pyre_softmax_rows": [_vp, _c_i64, _i, _vp, _vp],
    "pyre_rope_table": [ctypes.c_double, ctypes.c_double, _i, _i, _vp],
    "pyre_rope_kv_append": [_vp, _vp, _vp, _c_i64, _c_i64, _i, _i, _i, _i, _i, _vp, ctypes.c_double,
                            _vp, _vp, _vp, _i, _vp],
    "pyre_attn_status": [ctypes.POINTER(_i)],
    "pyre_graph_run": [_vp, _vp, _vp, _vp, _c_i64],
    "pyre_lm_head_workspace_bytes": [_i, ctypes.POINTER(_c_i64)],
    "pyre_lm_head_argmax": [_vp, _i, _i, _vp, ctypes.c_double, _vp, _i, _c_i64, _vp, _vp, _vp, _vp, _c_i64, _vp],
    "pyre_attn_prefill": [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp],
    "pyre_attn_decode_workspace_bytes": [_i, _i, _i, _i, ctypes.POINTER(_c_i64)],
    "pyre_attn_decode": [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _c_i64, _vp],
    "pyre_attn_decode_step": [_vp, _vp, _vp, _i, _vp, ctypes.c_double, _i, _i, _i, _vp, _vp, _i, _i, _i, _vp, _vp,
                              _c_i64, _vp],
    "pyre_ulysses_buffer_bytes": [_i, _i, _i, _i, _i, ctypes.POINTER(_c_i64)],
    "pyre_ulysses_rope_scatter": [_vp, _i, _i, _vp, _vp, _vp, _c_i64, _c_i64, _i, _i, _i, _i, _vp,
                                  ctypes.c_double, _vp],
    "pyre_ulysses_barrier": [_vp, _i, _i, _i, _i, _i, _i, _i, ctypes.c_uint64, _vp],
    "pyre_ulysses_attention": [_vp, _i, _i, _i, _i, _i, _i, _vp],
    "pyre_ulysses_finish": [_vp, _i, _i, _i, _i, _i, _vp, ctypes.POINTER(_i), _vp],
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Loads the extension once per process (thread-safe)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("PYRE_B200_LIB", LIB_PATH))
        if not path.exists():
            raise ImportError(
                f"pyre_b200 CUDA extension not found at {path}; build it with "
                "`python -m pyre_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(str(path))
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = _i
        _lib = lib
        return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().pyre_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(code: int) -> None:
    if code == PYRE_OK:
        return
    msg = last_error()
    if code == PYRE_ETIMEOUT:
        raise PyreTimeout(code, msg)
    if code == PYRE_EINVAL:
        raise ValueError(f"[pyre status {code}] {msg}")
    raise PyreError(code, msg)


def call(name: str, *args) -> None:
    """Calls a C-ABI entry point and raises on a non-zero status."""
    check(getattr(load(), name)(*args))


def exported_symbols() -> list[str]:
    return sorted(_SIGNATURES)
