"""Ulysses sequence-parallel attention (one spawned process per GPU): each rank holds its
slice of the sequence's q/k/v; RoPE + the QKV exchange, the per-head causal attention and the
output scatter run over NVLink. Every rank's output rows must equal the attention oracle within
the attention tolerance, and be bit-identical to the single-GPU prefill attention of the same
sequence (same kernels, same f16 operands).

Two shapes: a small one (384 tokens, 8/2 heads, hd 64) against the full oracle, and the
long-context configuration (32768 tokens, 32/8 heads, hd 128, theta 5e5) on 2, 4 and 8 GPUs and
on one GPU, where 256 seeded (position, head) outputs are checked against a row-wise f64
restatement of the reference's attention (its full score matrix would take ~137 GB).

Multi-GPU cases are skipped when the machine has fewer GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu]

TOL_ATTN = 5e-3
S, NQ, NKV, HD, THETA = 384, 8, 2, 64, 5e5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(77)
    q = (rng.standard_normal((S, NQ * HD)) * 2).astype(np.float32)
    k = (rng.standard_normal((S, NKV * HD)) * 2).astype(np.float32)
    v = (rng.standard_normal((S, NKV * HD)) * 2).astype(np.float32)
    return q, k, v


def _rank_main(rank, world, port, result_dir):
    import datetime
    import torch.distributed as dist
    from pyre_b200.attention import AttentionOp, UlyssesAttention

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    uly = None
    try:
        q, k, v = _inputs()
        Sl = S // world
        rows = slice(rank * Sl, (rank + 1) * Sl)
        uly = UlyssesAttention(S, NQ, NKV, HD, rope_theta=THETA, timeout_s=5.0)
        outs = []
        for _ in range(3):   # repeated calls: barrier epochs advance
            o = uly(*(torch.from_numpy(np.ascontiguousarray(a[rows])).cuda() for a in (q, k, v)))
            outs.append(o.cpu().numpy())
        single = AttentionOp(NQ, NKV, HD, max_t=S, rope_theta=THETA)
        full = single.prefill(*(torch.from_numpy(a).cuda() for a in (q, k, v))).cpu().numpy()
        np.savez(os.path.join(result_dir, f"rank{rank}.npz"), out=outs[0], out2=outs[2], single=full[rows])
    finally:
        if uly is not None:
            uly.close()
        dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ulysses_two_gpus(tmp_path):
    import torch.multiprocessing as mp
    from oracle import attention as OA
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    q, k, v = _inputs()
    ref = OA.compute_attention([(q.reshape(1, S, NQ, HD), k.reshape(1, S, NKV, HD), v.reshape(1, S, NKV, HD))],
                               NQ, NKV, 1.0, THETA)[0]
    Sl = S // world
    for r in range(world):
        z = np.load(tmp_path / f"rank{r}.npz")
        assert np.array_equal(z["out"], z["single"]), r
        assert np.array_equal(z["out2"], z["out"]), r
        want = ref[r * Sl:(r + 1) * Sl]
        assert float(np.abs(z["out"] - want).max() / np.abs(want).max()) < TOL_ATTN


# ---- the long-context configuration: Llama-3-8B attention shape, 32768 tokens -------------
S5, NQ5, NKV5, HD5, THETA5 = 32768, 32, 8, 128, 5e5
N_ROWS5 = 256        # seeded (position, head) samples checked against the f64 row oracle


def _inputs5():
    rng = np.random.default_rng(4)
    q = rng.standard_normal((S5, NQ5 * HD5), dtype=np.float32)
    k = rng.standard_normal((S5, NKV5 * HD5), dtype=np.float32)
    v = rng.standard_normal((S5, NKV5 * HD5), dtype=np.float32)
    return q, k, v


def _samples5():
    rng = np.random.default_rng(5)
    # every position range is represented: late rows attend over almost the whole sequence
    pos = np.sort(rng.integers(0, S5, N_ROWS5))
    return pos, rng.integers(0, NQ5, N_ROWS5)


def _check_rows5(out_rows: np.ndarray, pos, heads, q, k, v):
    from oracle import attention as OA
    ref = OA.attention_rows_f64(q, k, v, pos, heads, NQ5, NKV5, THETA5)
    got = np.stack([out_rows[i].reshape(NQ5, HD5)[h] for i, h in enumerate(heads)]).astype(np.float64)
    err = float(np.abs(got - ref).max() / np.abs(ref).max())
    assert err < TOL_ATTN, err


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_long_context_single_gpu_rows_vs_f64():
    """Causal prefill attention of 32768 tokens (32 q / 8 kv heads, hd 128, theta 5e5) on one
    GPU: 256 seeded (position, head) outputs against the row-wise f64 restatement."""
    from pyre_b200.attention import AttentionOp
    q, k, v = _inputs5()
    op = AttentionOp(NQ5, NKV5, HD5, max_t=S5, rope_theta=THETA5)
    out = op.prefill(*(torch.from_numpy(a).cuda() for a in (q, k, v)))
    pos, heads = _samples5()
    rows = out[torch.from_numpy(pos).cuda()].cpu().numpy()
    _check_rows5(rows, pos, heads, q, k, v)


def _rank_main5(rank, world, port, result_dir):
    import datetime
    import torch.distributed as dist
    from pyre_b200.attention import AttentionOp, UlyssesAttention

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    uly = None
    try:
        q, k, v = _inputs5()
        Sl = S5 // world
        rows = slice(rank * Sl, (rank + 1) * Sl)
        uly = UlyssesAttention(S5, NQ5, NKV5, HD5, rope_theta=THETA5, timeout_s=5.0)
        out = uly(*(torch.from_numpy(np.ascontiguousarray(a[rows])).cuda() for a in (q, k, v))).cpu().numpy()
        single = AttentionOp(NQ5, NKV5, HD5, max_t=S5, rope_theta=THETA5)
        full = single.prefill(*(torch.from_numpy(a).cuda() for a in (q, k, v)))[rank * Sl:(rank + 1) * Sl]
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), out)
        np.save(os.path.join(result_dir, f"single{rank}.npy"), full.cpu().numpy())
    finally:
        if uly is not None:
            uly.close()
        dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ulysses_long_context(tmp_path, world):
    """Ulysses over 2, 4 or 8 GPUs at 32768 tokens and the Llama-3-8B head shape: every rank's
    rows bit-identical to the single-GPU attention, and 256 seeded (position, head) outputs
    against the row-wise f64 restatement."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main5, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    Sl = S5 // world
    outs = [np.load(tmp_path / f"rank{r}.npy") for r in range(world)]
    for r in range(world):
        assert np.array_equal(outs[r], np.load(tmp_path / f"single{r}.npy")), r
    full = np.concatenate(outs)
    assert full.shape == (S5, NQ5 * HD5)
    pos, heads = _samples5()
    _check_rows5(full[pos], pos, heads, *_inputs5())
