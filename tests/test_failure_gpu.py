"""Failure detection on 2 GPUs, made on the host: one rank skips a call, so the waits of the other
rank's kernel run out (bounded waits, a flag that nothing sets); that kernel returns, the host
reads PyreTimeout from the status word, every rank resets on the host, and the next call is
correct again.

* tensor-parallel FFN (decode, reduce in the down-projection epilogue over NVLink): rank 1 skips
  one FfnShardOp call; rank 0's TPComm.check() raises PyreTimeout; after TPComm.reset() and
  FfnShardOp.reset() on both ranks the next call equals the f64 oracle on both.
* Ulysses attention: rank 1 skips one call; rank 0's call raises PyreTimeout from its phase-0
  barrier; after UlyssesAttention.reset() on both ranks the next call equals the single-GPU
  attention.

No rank leaves while its kernels are in flight, no GPU fault is involved: the skipping rank
simply does not launch, and the waiting kernel gives up after the communicator's timeout. The
process group is gloo (host only); NCCL's NVLS is switched off for the ranks all the same.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ffn_rank(rank, world, port, result_dir):
    import datetime
    import torch.distributed as dist
    from oracle import ffn as offn, q80 as oq80
    from pyre_b200 import _native as N
    from pyre_b200.ffn import FfnShardOp, FfnWeights
    from pyre_b200.quantizer import Q80Weight
    from pyre_b200.tp import ShardPlan, TPComm, shard_weights

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = None
    try:
        H, I = 1024, 3072
        rng = np.random.default_rng(3)
        w = {}
        for name, shape in (("gate", (H, I)), ("up", (H, I)), ("down", (I, H))):
            q, s, sh = oq80.quantize_q80((rng.standard_normal(shape) * 0.02).astype(np.float32))
            s = s.astype(np.float16).astype(np.float32)
            w[name] = (q, s, sh, oq80.dequantize_q80(q, s, sh))
        full = {n: Q80Weight.from_tuple(("q8", q, s, sh), scale_dtype=torch.float16) for n, (q, s, sh, _) in w.items()}
        plan = ShardPlan.equal(I, world)
        fw = FfnWeights.prepare(*shard_weights(full["gate"], full["up"], full["down"], plan.bounds, rank))
        comm = TPComm(H, max_tokens=1, timeout_s=0.05)
        op = FfnShardOp(H, plan.widths[rank], max_tokens=1, comm=comm)
        x = torch.from_numpy(np.random.default_rng(9).standard_normal((1, H)).astype(np.float32)).cuda()
        ref = offn.tp_ffn(x.cpu().numpy(), w["gate"][3], w["up"][3], w["down"][3], plan.bounds, f64=True)
        rel = lambda o: float(np.abs(o.cpu().numpy() - ref).max() / np.abs(ref).max())
        first = rel(op.run(x, fw))
        comm.check()
        dist.barrier()
        timed_out = False
        if rank == 0:                       # rank 1 skips this call
            op.run(x, fw)
            try:
                comm.check()
            except N.PyreTimeout:
                timed_out = True
        dist.barrier()
        comm.reset()
        op.reset()
        again = rel(op.run(x, fw))
        comm.check()
        np.savez(os.path.join(result_dir, f"ffn{rank}.npz"), first=first, timed_out=timed_out, again=again)
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def _ulysses_rank(rank, world, port, result_dir):
    import datetime
    import torch.distributed as dist
    from pyre_b200 import _native as N
    from pyre_b200.attention import AttentionOp
    from pyre_b200.attention.ulysses import UlyssesAttention

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    uly = None
    try:
        S, nq, nkv, hd = 256, 8, 2, 64
        g = torch.Generator().manual_seed(5)
        q, k, v = (torch.randn((S, n * hd), generator=g) for n in (nq, nkv, nkv))
        ref = AttentionOp(nq, nkv, hd, max_t=S, rope_theta=1e4).prefill(q.cuda(), k.cuda(), v.cuda()).cpu()
        Sl = S // world
        mine = [t[rank * Sl:(rank + 1) * Sl].contiguous().cuda() for t in (q, k, v)]
        uly = UlyssesAttention(S, nq, nkv, hd, rope_theta=1e4, timeout_s=0.05)
        want = ref[rank * Sl:(rank + 1) * Sl]
        first = bool(torch.equal(uly(*mine).cpu(), want))
        dist.barrier()
        timed_out = False
        if rank == 0:                       # rank 1 skips this call
            try:
                uly(*mine)
            except N.PyreTimeout:
                timed_out = True
        dist.barrier()
        uly.reset()
        again = bool(torch.equal(uly(*mine).cpu(), want))
        np.savez(os.path.join(result_dir, f"uly{rank}.npz"), first=first, timed_out=timed_out, again=again)
    finally:
        if uly is not None:
            uly.close()
        dist.destroy_process_group()


def _run(fn, tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(fn, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_ffn_peer_timeout_and_recovery(tmp_path):
    _run(_ffn_rank, tmp_path)
    r0, r1 = (np.load(tmp_path / f"ffn{r}.npz") for r in range(2))
    assert r0["first"] < 1e-4 and r1["first"] < 1e-4
    assert bool(r0["timed_out"]) and not bool(r1["timed_out"])
    assert r0["again"] < 1e-4 and r1["again"] < 1e-4


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ulysses_barrier_timeout_and_recovery(tmp_path):
    _run(_ulysses_rank, tmp_path)
    r0, r1 = (np.load(tmp_path / f"uly{r}.npz") for r in range(2))
    assert bool(r0["first"]) and bool(r1["first"])
    assert bool(r0["timed_out"]) and not bool(r1["timed_out"])
    assert bool(r0["again"]) and bool(r1["again"])
