"""Final norm + lm_head + greedy token on the GPU against the oracle (oracle/lmhead.py), which
tests/test_lmhead_oracle.py pins to the reference's own Generator methods.

Tolerances: logits max|dev - ref| / max|ref| < 1e-5 (f32 accumulation in another order); the
token equals the oracle's argmax, or (random data only) its oracle logit is within 1e-5 of the
maximum (a near tie decided by the last bit)."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import lmhead as OL

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.abs(a.astype(np.float64) - b).max() / np.abs(b).max())


def test_golden_cases_with_ties():
    from pyre_b200.lmhead import LmHeadOp
    z = np.load(GOLDEN / "lmhead_golden.npz")
    for name in ("small", "rows"):
        h, w, E = z[f"{name}__h"], z[f"{name}__w"], z[f"{name}__E"]
        op = LmHeadOp(torch.from_numpy(E).cuda(), torch.from_numpy(w.astype(np.float32)).cuda(),
                      max_tokens=h.shape[0])
        tok, logits = op(torch.from_numpy(h).cuda(), want_logits=True)
        assert rel(logits.cpu().numpy(), z[f"{name}__logits"]) < 1e-5, name
        assert np.array_equal(tok.cpu().numpy(), z[f"{name}__token"]), name   # ties: the first index


@pytest.mark.parametrize("T,H,V,norm", [(1, 4096, 32768, True), (4, 4096, 32768, True), (2, 896, 15193, False),
                                        (1, 576, 49152, True)])
def test_random_vs_oracle_and_repeat(T, H, V, norm):
    from pyre_b200.lmhead import LmHeadOp
    rng = np.random.default_rng(T * 7 + H)
    h = (rng.standard_normal((T, H)) * 2).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32) if norm else None
    E = (rng.standard_normal((V, H)) * 0.02).astype(np.float16)
    ref = OL.compute_logits(h, E, w)
    op = LmHeadOp(torch.from_numpy(E).cuda(), torch.from_numpy(w).cuda() if norm else None, max_tokens=T)
    for _ in range(2):       # the workspace is reused: its counter is back at zero after a call
        tok, logits = op(torch.from_numpy(h).cuda(), want_logits=True)
        assert rel(logits.cpu().numpy(), ref) < 1e-5
        for t in range(T):
            k = int(tok[t, 0])
            assert ref[t, k] >= ref[t].max() - 1e-5 * np.abs(ref[t]).max()


def test_vocab_shards_combine_by_key():
    """A table split over 3 shards (global offsets v0): the max of the shards' keys gives the
    full table's token, as the cross-rank max all-reduce does."""
    from pyre_b200 import _device as D, _native as N
    import ctypes
    rng = np.random.default_rng(5)
    T, H, V = 2, 1024, 5000
    h = rng.standard_normal((T, H)).astype(np.float32)
    E = (rng.standard_normal((V, H)) * 0.05).astype(np.float16)
    full = OL.greedy_token(OL.compute_logits(h, E, None))[:, 0]
    b = ctypes.c_int64(0)
    N.call("pyre_lm_head_workspace_bytes", T, ctypes.byref(b))
    ws = torch.zeros(b.value, dtype=torch.uint8, device="cuda")
    hd = torch.from_numpy(h).cuda()
    keys = []
    for a, e in ((0, 1700), (1700, 3333), (3333, V)):
        Ed = torch.from_numpy(np.ascontiguousarray(E[a:e])).cuda()
        tok = torch.empty(T, dtype=torch.int32, device="cuda")
        key = torch.empty(T, dtype=torch.int64, device="cuda")
        N.call("pyre_lm_head_argmax", D.ptr(hd), T, H, None, 1e-6, D.ptr(Ed), e - a, a, None, D.ptr(tok),
               D.ptr(key), D.ptr(ws), ws.numel(), D.stream_ptr())
        assert all(a <= int(x) < e for x in tok.cpu())
        keys.append(key)
    best = torch.stack(keys).max(dim=0).values
    low = (best ^ (-(1 << 63))) & 0xFFFFFFFF
    got = (0xFFFFFFFF - low).cpu().numpy()
    assert np.array_equal(got, full)
