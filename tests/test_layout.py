"""Q8_0 weight layouts: plain reference orientation (slicing, host logic on CPU tensors) and
the packed block layout of include/pyre_b200.h, restated here in numpy as the checker of
the device packing kernel."""
import numpy as np
import pytest
import torch

from pyre_b200.quantizer import Q80Weight


def pack_reference(qs, ss, es_dtype):
    """numpy restatement of the packed layout: blocks per (256-column slab j, R-row unit u),
    [q_0 | ... | q_{M-1} | s_0 | ... | s_{M-1}], K padded to R, N padded to 256 with zeros."""
    M = len(qs)
    K, N = qs[0].shape
    R = 32 if M == 2 else 64
    nt, upt = -(-N // 256), -(-K // R)
    out = []
    for j in range(nt):
        for u in range(upt):
            qpart, spart = [], []
            for m in range(M):
                qb = np.zeros((R, 256), np.int8)
                sb = np.zeros((R, 8), es_dtype)
                rows = slice(u * R, min(K, (u + 1) * R))
                cols = slice(j * 256, min(N, (j + 1) * 256))
                blk = qs[m][rows, cols]
                qb[: blk.shape[0], : blk.shape[1]] = blk
                sblk = ss[m][rows, j * 8: min(N // 32, j * 8 + 8)]
                sb[: sblk.shape[0], : sblk.shape[1]] = sblk
                qpart.append(qb.tobytes())
                spart.append(sb.tobytes())
            out.append(b"".join(qpart) + b"".join(spart))
    return np.frombuffer(b"".join(out), dtype=np.uint8)


def test_pack_reference_block_size():
    q = np.zeros((64, 256), np.int8)
    s = np.zeros((64, 8), np.float16)
    assert pack_reference([q], [s], np.float16).size == 64 * 256 + 64 * 8 * 2
    assert pack_reference([q, q], [s, s], np.float16).size == 2 * (64 * 256 + 64 * 8 * 2)


def test_rows_and_cols_slices():
    g = torch.Generator().manual_seed(1)
    q = torch.randint(-128, 128, (96, 640), generator=g, dtype=torch.int8)
    s = torch.rand((96, 20), generator=g)
    w = Q80Weight(q, s)
    r = w.rows(32, 80)
    assert torch.equal(r.q, q[32:80]) and torch.equal(r.scale, s[32:80])
    c = w.cols(96, 544)
    assert torch.equal(c.q, q[:, 96:544]) and torch.equal(c.scale, s[:, 3:17])
    with pytest.raises(ValueError):
        w.cols(10, 64)
    with pytest.raises(ValueError):
        Q80Weight(q, s[:, :5])
