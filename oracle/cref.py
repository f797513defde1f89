"""ORACLE (test infrastructure): ctypes access to oracle/liboracle.so, the C restatement
of the reference's CPU loops (oracle/csrc/oracle_ref.c)."""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def load():
    global _lib
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "csrc" / "oracle_ref.c").stat().st_mtime:
            build()
        lib = ctypes.CDLL(str(LIB))
        vp, i64 = ctypes.c_void_p, ctypes.c_int64
        lib.oracle_q80_quantize.argtypes = [vp, i64, vp, vp]
        lib.oracle_q80_dequantize.argtypes = [vp, vp, i64, vp]
        lib.oracle_matmul_f32.argtypes = [vp, vp, vp, i64, i64, i64]
        lib.oracle_silu_mul.argtypes = [vp, vp, vp, i64]
        lib.oracle_root_decode_ffn.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, vp]
        for f in ("oracle_q80_quantize", "oracle_q80_dequantize", "oracle_matmul_f32", "oracle_silu_mul",
                  "oracle_root_decode_ffn"):
            getattr(lib, f).restype = None
        _lib = lib
    return _lib


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def q80_quantize(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    nb = (x.size + 31) // 32
    q = np.zeros((nb, 32), dtype=np.int8)
    s = np.zeros(nb, dtype=np.float32)
    load().oracle_q80_quantize(_p(x), x.size, _p(q), _p(s))
    return q, s


def matmul_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    M, K = a.shape
    K2, Nn = b.shape
    assert K == K2
    r = np.zeros((M, Nn), dtype=np.float32)
    load().oracle_matmul_f32(_p(a), _p(b), _p(r), M, K, Nn)
    return r


def root_decode_ffn(x, gate, up, down, c0: int, c1: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    gate = np.ascontiguousarray(gate, dtype=np.float32)
    up = np.ascontiguousarray(up, dtype=np.float32)
    down = np.ascontiguousarray(down, dtype=np.float32)
    H, W = gate.shape
    out = np.zeros(H, dtype=np.float32)
    load().oracle_root_decode_ffn(_p(x), _p(gate), _p(up), _p(down), H, W, c0, c1, _p(out))
    return out
