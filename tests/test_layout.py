"""Column-slab tiled Q8_0 device layout: a pure permutation of the reference's blocks
(host logic, CPU tensors)."""
import numpy as np
import pytest
import torch

from pyre_b200.quantizer import SLAB, Q80Weight


@pytest.mark.parametrize("K,N", [(32, 256), (64, 96), (40, 800), (3, 1024)])
def test_tiling_is_a_permutation(K, N):
    g = torch.Generator().manual_seed(K * N)
    q = torch.randint(-128, 128, (K, N), generator=g, dtype=torch.int8)
    s = torch.rand((K, N // 32), generator=g).to(torch.float16)
    w = Q80Weight.from_plain(q, s)
    nt = (N + SLAB - 1) // SLAB
    assert tuple(w.q.shape) == (nt, K, SLAB) and tuple(w.scale.shape) == (nt, K, 8)
    assert w.shape == (K, N)
    for j in range(nt):
        c1 = min(N, (j + 1) * SLAB)
        assert torch.equal(w.q[j, :, : c1 - j * SLAB], q[:, j * SLAB:c1])
        assert int(w.q[j, :, c1 - j * SLAB:].abs().sum()) == 0          # zero padding
        assert torch.equal(w.scale[j, :, : (c1 - j * SLAB) // 32], s[:, j * 8:c1 // 32])
    q2, s2 = w.plain()
    assert torch.equal(q2, q) and torch.equal(s2, s)
    assert w.nbytes == K * N + K * (N // 32) * 2


def test_rows_and_cols_slices():
    g = torch.Generator().manual_seed(1)
    q = torch.randint(-128, 128, (96, 640), generator=g, dtype=torch.int8)
    s = torch.rand((96, 20), generator=g)
    w = Q80Weight.from_plain(q, s)
    r = w.rows(32, 80)
    assert torch.equal(r.plain()[0], q[32:80]) and torch.equal(r.plain()[1], s[32:80])
    c = w.cols(96, 544)
    assert torch.equal(c.plain()[0], q[:, 96:544]) and torch.equal(c.plain()[1], s[:, 3:17])
    with pytest.raises(ValueError):
        w.cols(10, 64)
