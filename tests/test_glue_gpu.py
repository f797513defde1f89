"""Layer glue kernels against numpy: the residual add + next RMSNorm (root_node.py:947-951,
:997 + :752) and the embedding gather + first RMSNorm (generator.py:38-39 + root_node.py:752),
on the 16-byte-vector path (H % 4 == 0, H <= 16384) and the generic one. The residual add is
exact; the norm uses an f64 sum of squares, so it equals numpy's up to the order of that sum
(relative 1e-6 here)."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rms(h, w, eps):
    var = np.mean(h.astype(np.float64) ** 2, axis=-1, keepdims=True)
    return (h.astype(np.float64) / np.sqrt(var + eps) * w.astype(np.float64)).astype(np.float32)


@pytest.mark.parametrize("H", [30, 576, 4096, 20000])
@pytest.mark.parametrize("inplace", [False, True])
def test_add_rms_norm(H, inplace):
    from pyre_b200 import _device as D
    from pyre_b200 import _native as N
    rng = np.random.default_rng(H)
    rows = 3
    x = rng.standard_normal((rows, H)).astype(np.float32)
    d = rng.standard_normal((rows, H)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    xt, dt, wt = (torch.from_numpy(a).cuda() for a in (x, d, w))
    ht = xt if inplace else torch.empty_like(xt)
    nt = torch.empty_like(xt)
    N.call("pyre_add_rms_norm", D.ptr(xt), D.ptr(dt), rows, H, D.ptr(wt), 1e-6, D.ptr(ht), D.ptr(nt), D.stream_ptr())
    torch.cuda.synchronize()
    h_ref = x + d
    assert np.array_equal(ht.cpu().numpy(), h_ref)
    np.testing.assert_allclose(nt.cpu().numpy(), _rms(h_ref, w, 1e-6), rtol=1e-6, atol=1e-7)
    # add only
    h2 = torch.empty_like(xt)
    N.call("pyre_add_rms_norm", D.ptr(torch.from_numpy(x).cuda()), D.ptr(dt), rows, H, None, 1e-6, D.ptr(h2), None,
           D.stream_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(h2.cpu().numpy(), h_ref)


@pytest.mark.parametrize("H", [30, 576, 4096])
def test_embed_rms_norm_and_bad_id(H):
    from pyre_b200 import _device as D
    from pyre_b200 import _native as N
    rng = np.random.default_rng(H + 1)
    V = 1000
    table = (rng.standard_normal((V, H)) * 0.05).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    ids = np.array([3, 999, 0, 512], dtype=np.int32)
    tt, wt, it = torch.from_numpy(table).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda()
    x = torch.empty((len(ids), H), dtype=torch.float32, device="cuda")
    nrm = torch.empty_like(x)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    N.call("pyre_embed_rms_norm", D.ptr(it), len(ids), D.ptr(tt), V, H, D.ptr(wt), 1e-6, D.ptr(x), D.ptr(nrm),
           D.ptr(status), D.stream_ptr())
    torch.cuda.synchronize()
    x_ref = table[ids].astype(np.float32)
    assert np.array_equal(x.cpu().numpy(), x_ref)
    np.testing.assert_allclose(nrm.cpu().numpy(), _rms(x_ref, w, 1e-6), rtol=1e-6, atol=1e-7)
    assert int(status.item()) == 0
    # an id outside [0, V): zero row and PYRE_EINVAL in the status word
    bad = torch.tensor([5, V + 3], dtype=torch.int32, device="cuda")
    N.call("pyre_embed_rms_norm", D.ptr(bad), 2, D.ptr(tt), V, H, None, 1e-6, D.ptr(x), None, D.ptr(status),
           D.stream_ptr())
    torch.cuda.synchronize()
    assert int(status.item()) == N.PYRE_EINVAL
    assert np.array_equal(x[0].cpu().numpy(), table[5].astype(np.float32))
    assert not x[1].any()
