"""pyre_ffn_decode_q80_noalloc (scratch in a static device array, no allocation) against
pyre_ffn_decode_q80 (caller-allocated workspace), both called through the C ABI.

Collected last on purpose (file name), and written to pass both on its own in a fresh
process and after every other test: the static scratch then already holds the contents of
earlier calls. Both entry points run the same kernel, whose slab sums are deterministic
(integer fixed point), so their outputs must be bit-identical.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _weights(H, W, gated, seed):
    from pyre_b200.ffn import FfnWeights
    from pyre_b200.quantizer import Q80Weight
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda shape: Q80Weight.from_float(torch.randn(shape, device="cuda", generator=g) * 0.02)
    gate = mk((H, W)) if gated else None
    return FfnWeights.prepare(gate, mk((H, W)), mk((W, H)))


def _decode_with_workspace(x, w, T, H, W):
    """The existing entry point, with a workspace allocated and zeroed here."""
    from pyre_b200 import _device as D, _native as N
    need = ctypes.c_int64(0)
    N.call("pyre_ffn_workspace_bytes", T, H, W, ctypes.byref(need))
    ws = torch.zeros(need.value, dtype=torch.uint8, device="cuda")
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    N.call("pyre_ffn_decode_q80", D.ptr(x), D.dtype_code(x), T, H, D.ptr(w.gateup.data), int(w.gated),
           D.ptr(w.down.data), w.gateup.scale_code, W, D.ptr(out), D.ptr(ws), ws.numel(), ctypes.c_void_p(0),
           D.stream_ptr())
    return out


def _decode_noalloc(x, w, T, H, W):
    from pyre_b200 import _device as D, _native as N
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    N.call("pyre_ffn_decode_q80_noalloc", D.ptr(x), D.dtype_code(x), T, H, D.ptr(w.gateup.data), int(w.gated),
           D.ptr(w.down.data), w.gateup.scale_code, W, D.ptr(out), D.stream_ptr())
    return out


@pytest.mark.parametrize("T,H,W,gated", [(1, 4096, 14336, True), (4, 1024, 2816, False), (3, 576, 768, True)])
def test_noalloc_matches_workspace_entry_two_calls(T, H, W, gated):
    w = _weights(H, W, gated, seed=T * 7 + H)
    _noalloc_status()       # start from a clear status word whatever ran before
    for call in range(2):   # two calls in a row: the second reuses the static scratch
        x = torch.randn((T, H), device="cuda").to(torch.bfloat16 if call else torch.float32)
        ref = _decode_with_workspace(x, w, T, H, W)
        got = _decode_noalloc(x, w, T, H, W)
        assert _noalloc_status() == 0, f"call {call}"
        assert torch.isfinite(got).all()
        assert torch.equal(got, ref), f"call {call}"


def _noalloc_status() -> int:
    from pyre_b200 import _device as D, _native as N
    st = ctypes.c_int(-1)
    N.call("pyre_ffn_decode_q80_noalloc_status", ctypes.byref(st), D.stream_ptr())
    return st.value


def test_noalloc_reports_range_status_then_recovers():
    """An infinite input makes a partial sum leave the fixed-point range: the call's status
    (read back through the status entry point) is PYRE_ERANGE, reading it clears it, and the
    next call is clean and equal to the workspace entry point."""
    from pyre_b200 import _native as N
    T, H, W = 1, 512, 768
    w = _weights(H, W, True, seed=5)
    bad = torch.zeros((T, H), device="cuda")
    bad[0, 7] = float("inf")
    _decode_noalloc(bad, w, T, H, W)
    assert _noalloc_status() == N.PYRE_ERANGE
    assert _noalloc_status() == N.PYRE_OK
    x = torch.randn((T, H), device="cuda")
    got = _decode_noalloc(x, w, T, H, W)
    assert _noalloc_status() == N.PYRE_OK
    assert torch.equal(got, _decode_with_workspace(x, w, T, H, W))


def test_noalloc_rejected_call_leaves_scratch_alone():
    """A call rejected by its argument checks queues nothing on the shared scratch: the status
    left by an earlier call survives it."""
    from pyre_b200 import _native as N
    T, H, W = 1, 512, 768
    w = _weights(H, W, True, seed=6)
    bad = torch.zeros((T, H), device="cuda")
    bad[0, 3] = float("nan")
    _decode_noalloc(bad, w, T, H, W)
    torch.cuda.synchronize()
    out = torch.empty((T, H), device="cuda")
    lib = N.load()
    rc = lib.pyre_ffn_decode_q80_noalloc(ctypes.c_void_p(bad.data_ptr()), N.PYRE_F32, T, H, ctypes.c_void_p(8), 1,
                                        ctypes.c_void_p(w.down.data.data_ptr()), w.gateup.scale_code, W,
                                        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(0))
    assert rc == N.PYRE_EINVAL and "16-byte aligned" in N.last_error()
    assert _noalloc_status() == N.PYRE_ERANGE


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from pyre_b200 import _native as N
    need = ctypes.c_int64(0)
    N.call("pyre_ffn_workspace_bytes", 4, 8192, 65536, ctypes.byref(need))
    assert need.value > N.PYRE_NOALLOC_SCRATCH_BYTES
    x = torch.zeros((4, 8192), device="cuda")
    out = torch.empty((4, 8192), device="cuda")
    lib = N.load()
    rc = lib.pyre_ffn_decode_q80_noalloc(ctypes.c_void_p(x.data_ptr()), N.PYRE_F32, 4, 8192, ctypes.c_void_p(16), 1,
                                        ctypes.c_void_p(16), N.PYRE_F16, 65536, ctypes.c_void_p(out.data_ptr()),
                                        ctypes.c_void_p(0))
    assert rc == N.PYRE_EINVAL
    assert "bytes of scratch" in N.last_error()
