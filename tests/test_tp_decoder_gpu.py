"""Tensor-parallel whole decoder on 2, 4 or 8 GPUs against the reference's greedy goldens.

One spawned process per GPU. Each rank builds pyre_b200.generator.Generator with a TPComm:
its share of the heads (the reference's head partition of a decode layer, root_node.py:182-210
and :763-858: local QKV, local KV cache and attention, the O projection of its heads), its FFN
shard (non-uniform Dirichlet(5) widths in 32-element blocks for the Mistral-shaped model) and its
rows of the lm_head; the O-projection and FFN partials are summed over the ranks in the kernels'
epilogues (NVLink peer stores) and the greedy token is the best of the ranks' (value, index) keys.
Every rank must produce the reference's 32 greedy tokens (one-pass prefill + graphed decode, and
one native call per token with logits), and the ranks' logit shards, put together, must match
the reference's top-8 logits of every step within the single-GPU tolerance.

Skipped when the machine has fewer GPUs than ranks (ranks that wait on one another are never
placed on one device).
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

LOGIT_ATOL = 2e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, name, result_dir):
    import datetime
    import torch.distributed as dist
    import greedy_device as G
    from greedy_device import gm
    from pyre_b200.tp import ShardPlan, TPComm

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    comm = None
    try:
        m = gm.MODELS[name]
        g = G.golden(m)
        comm = TPComm(m.hidden, max_tokens=max(64, m.prompt_len), timeout_s=5.0)
        plan = ShardPlan.dirichlet(m.ffn, world, 5.0, 1)
        gen = G.generator(m, torch.device("cuda", rank), comm=comm, ffn_plan=plan)
        graphed = [gen.generate_ids(g["prompt"], gm.N_GREEDY, graphed=True) for _ in range(2)]
        ids, logits = gen.generate_ids(g["prompt"], gm.N_GREEDY, want_logits=True)
        comm.check()
        np.savez(os.path.join(result_dir, f"rank{rank}.npz"), graphed=np.array(graphed), ids=np.array(ids),
                 logits=logits.cpu().numpy(), v0=gen.lm_v0, widths=np.array(plan.widths))
        del gen
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


CASES = [("mistral7b_l2", 2), ("qwen05b_l4", 2), ("mistral7b_l2", 4), ("mistral7b_l2", 8)]


@pytest.mark.parametrize("name,world", CASES, ids=[f"{n}-tp{w}" for n, w in CASES])
def test_tp_decoder_greedy_matches_reference(tmp_path, name, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    import greedy_device as G
    from greedy_device import gm
    g = G.golden(gm.MODELS[name])
    mp.start_processes(_rank_main, args=(world, _free_port(), name, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    res = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    want = g["tokens"].tolist()
    for r, d in enumerate(res):
        assert d["graphed"].tolist() == [want, want], f"rank {r}: graphed decode"
        assert d["ids"].tolist() == want, f"rank {r}: per-call decode"
    assert sorted(int(d["v0"]) for d in res) == [int(d["v0"]) for d in res]
    full = np.concatenate([d["logits"] for d in res], axis=1)        # vocabulary shards in rank order
    d0 = np.abs(full[0] - g["first_logits"]).max()
    assert d0 <= LOGIT_ATOL, f"first-step logits differ by {d0}"
    for step in range(gm.N_GREEDY):
        err = np.abs(full[step][g["top_idx"][step]] - g["top_val"][step]).max()
        assert err <= LOGIT_ATOL, f"step {step}: top-8 logits differ by {err}"
