"""Host-side tensor-parallel logic on world_size-2 gloo ranks (CPU): IPC-handle exchange,
identical shard plans on every rank, and the adaptive partitioner fed with gathered
per-rank timings reaching the same decision everywhere."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from pyre_b200.partitioner import AdaptivePartitioner
        from pyre_b200.tp import ShardPlan, exchange_handles, gather_timings
        h = bytes([rank]) * 64
        hs = exchange_handles(h)
        plan = ShardPlan.dirichlet(14336, world, 5.0, 1)
        times = gather_timings(0.010 if rank == 0 else 0.040)
        ap = AdaptivePartitioner(14336, world, block=32)
        ap.update({r: t for r, t in enumerate(times)})
        q.put((rank, hs, plan.widths, times, ap.drift_detected(), ap.get_partitions()))
    finally:
        dist.destroy_process_group()


def test_tp_host_logic_gloo_world2():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    (_, hs0, w0, t0, d0, p0), (_, hs1, w1, t1, d1, p1) = res
    assert hs0 == hs1 == [bytes([0]) * 64, bytes([1]) * 64]
    assert w0 == w1 and sum(w0) == 14336
    assert t0 == t1 == [0.010, 0.040]
    assert d0 == d1 is True
    assert p0 == p1
