"""Tensor-parallel FFN on 2+ GPUs: one spawned process per GPU, each holding a non-uniform
shard (Dirichlet(5) widths in 32-element blocks), the cross-rank sum done by this library's
peer-memory reduce (in the down-projection epilogue for T <= 4, the two-shot all-reduce
for larger T). Every rank's output must equal the f64 oracle of the sum of the shard
partials (src/orchestrator/root_node.py:582-594, `ffn_out += partial`) within the decode
path's tolerance, and all ranks must hold bit-identical sums.

Skipped with fewer than 2 GPUs. Each rank runs on its own GPU (ranks that wait on one
another are never placed on one device).
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

TOL_DECODE = 1e-4
TOL_PREFILL = 1e-2
H, I = 1024, 3072


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(seed):
    from oracle import q80 as oq80
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in (("gate", (H, I)), ("up", (H, I)), ("down", (I, H))):
        w = rng.standard_normal(shape).astype(np.float32) * 0.02
        q, s, sh = oq80.quantize_q80(w)
        s = s.astype(np.float16).astype(np.float32)
        out[name] = (q, s, sh, oq80.dequantize_q80(q, s, sh))
    return out


def _rank_main(rank, world, port, result_dir):
    import datetime
    import torch.distributed as dist
    from pyre_b200.ffn import FfnShardOp, FfnWeights
    from pyre_b200.quantizer import Q80Weight
    from pyre_b200.tp import ShardPlan, TPComm, shard_weights
    from oracle import ffn as offn

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = None
    try:
        w = _weights(7)
        full = {n: Q80Weight.from_tuple(("q8", q, s, sh), scale_dtype=torch.float16) for n, (q, s, sh, _) in w.items()}
        plan = ShardPlan.dirichlet(I, world, 5.0, 1)
        gate, up, down = shard_weights(full["gate"], full["up"], full["down"], plan.bounds, rank)
        fw = FfnWeights.prepare(gate, up, down)
        comm = TPComm(H, max_tokens=24, timeout_s=5.0)
        errs = []
        outs = []
        for T in (1, 3, 4, 17, 24):
            op = FfnShardOp(H, plan.widths[rank], max_tokens=T, comm=comm)
            rng = np.random.default_rng(100 + T)          # same x on every rank
            x = rng.standard_normal((T, H)).astype(np.float32)
            xt = torch.from_numpy(x).cuda().to(torch.bfloat16 if T > 4 else torch.float32)
            for _ in range(3):                            # repeated calls: epochs / slots alternate
                out = op.run(xt, fw)
            comm.check()
            ref = offn.tp_ffn(xt.float().cpu().numpy(), w["gate"][3], w["up"][3], w["down"][3], plan.bounds, f64=True)
            o = out.cpu().numpy().astype(np.float64)
            errs.append(float(np.abs(o - ref).max() / np.abs(ref).max()))
            outs.append(out.cpu().numpy())
        np.savez(os.path.join(result_dir, f"rank{rank}.npz"), errs=np.array(errs), *outs)
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_ffn_two_gpus(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    res = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    errs = res[0]["errs"]
    for i, T in enumerate((1, 3, 4, 17, 24)):
        assert errs[i] < (TOL_DECODE if T <= 4 else TOL_PREFILL), (T, errs[i])
        for r in range(1, world):
            assert res[r]["errs"][i] == errs[i]
            assert np.array_equal(res[r][f"arr_{i}"], res[0][f"arr_{i}"]), f"rank {r} differs at T={T}"
