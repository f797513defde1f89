"""The C-ABI library loads, exports every symbol include/*.h declares, and its host-only
entry points validate arguments without touching a GPU."""
import ctypes
import re

import pytest

from conftest import ROOT
from pyre_b200 import _native as N


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"PYRE_API\s+int\s+(pyre_\w+)\s*\(", h.read_text()))
    return sorted(names)


def test_header_declares_entry_points():
    assert len(_declared_symbols()) >= 15


@pytest.mark.parametrize("sym", _declared_symbols())
def test_symbol_exported(native_lib, sym):
    assert hasattr(native_lib, sym), f"{sym} declared in include/ but not exported"


def test_binding_table_matches_header():
    assert set(N.exported_symbols()) == set(_declared_symbols())


def test_version_and_error_text(native_lib):
    assert native_lib.pyre_version() >= 100
    out = ctypes.c_int64(0)
    rc = native_lib.pyre_ffn_workspace_bytes(0, 4096, 14336, ctypes.byref(out))
    assert rc == N.PYRE_EINVAL
    assert "sizes must be positive" in N.last_error()


def test_workspace_and_buffer_sizes(native_lib):
    out = ctypes.c_int64(0)
    N.check(native_lib.pyre_ffn_workspace_bytes(1, 4096, 14336, ctypes.byref(out)))
    assert out.value > 0
    b = ctypes.c_int64(0)
    N.check(native_lib.pyre_comm_buffer_bytes(8, 4, 4096, ctypes.byref(b)))
    assert b.value % 256 == 0 and b.value > 2 * 8 * 4 * 4096 * 4
    with pytest.raises(ValueError):
        N.check(native_lib.pyre_comm_buffer_bytes(17, 4, 4096, ctypes.byref(b)))


def test_quantize_argument_checks_need_no_gpu(native_lib):
    assert native_lib.pyre_q80_quantize(None, N.PYRE_F32, 0, None, None, None, None) == N.PYRE_OK
    assert native_lib.pyre_q80_quantize(ctypes.c_void_p(16), 7, 32, ctypes.c_void_p(16),
                                        ctypes.c_void_p(16), None, None) == N.PYRE_EINVAL
    assert native_lib.pyre_ffn_gateup_silu_q80(None, N.PYRE_F32, 1, 64, None, 1, N.PYRE_F32, 64,
                                               None, N.PYRE_F32, None, 0, None) == N.PYRE_EINVAL
    ws = ctypes.c_void_p(256)
    assert native_lib.pyre_ffn_down_q80(ctypes.c_void_p(16), N.PYRE_F32, 1, 64, ctypes.c_void_p(16), N.PYRE_F32, 48,
                                        ctypes.c_void_p(16), ws, 1 << 20, None, None) == N.PYRE_EINVAL
    assert "multiple of 32" in N.last_error()
    # a workspace smaller than the header is refused before any launch
    assert native_lib.pyre_ffn_decode_q80(ctypes.c_void_p(16), N.PYRE_BF16, 1, 64, ctypes.c_void_p(16), 1,
                                          ctypes.c_void_p(16), N.PYRE_F16, 64, ctypes.c_void_p(16), ws, 64, None,
                                          None) == N.PYRE_EINVAL
    assert "workspace" in N.last_error()
    b = ctypes.c_int64(0)
    N.check(native_lib.pyre_q80_packed_bytes(2, 4096, 14336, N.PYRE_F16, ctypes.byref(b)))
    assert b.value == 56 * 128 * 2 * 32 * (256 + 16)
    assert native_lib.pyre_q80_packed_bytes(3, 64, 64, N.PYRE_F16, ctypes.byref(b)) == N.PYRE_EINVAL


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(N, "_lib", None)
    monkeypatch.setenv("PYRE_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(ImportError):
        N.load()
