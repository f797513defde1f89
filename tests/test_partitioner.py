"""Partitioner and drift detector: equal to the reference's AdaptivePartitioner outputs
(tests/golden/partition_golden.json, written by the reference's own cluster.py) and to
known answers of solve_partitions (src/partitioner/solver.mojo:30-52)."""
import json

import pytest

from conftest import GOLDEN
from pyre_b200.partitioner import (AdaptivePartitioner, NodeCap, detect_drift, dirichlet_block_widths,
                                   solve_partitions, widths_to_bounds)
from pyre_b200.tp import ShardPlan

GOLD = json.loads((GOLDEN / "partition_golden.json").read_text())


def _intkeys(d):
    return {int(k): v for k, v in d.items()}


@pytest.mark.parametrize("sc", GOLD["adaptive"], ids=lambda s: f"I{s['ffn_dim']}_n{s['n']}")
def test_adaptive_partitioner_matches_reference(sc):
    ap = AdaptivePartitioner(sc["ffn_dim"], sc["n"], seq_len=64)
    assert _intkeys(sc["equal"]) == AdaptivePartitioner.equal_partitions(sc["ffn_dim"], sc["n"])
    for layer_updates, want in zip(sc["passes"], sc["trace"]):
        ap.reset_pass()
        for upd in layer_updates:
            ap.update({int(k): v for k, v in upd.items()})
        assert ap.drift_detected() == want["drift"]
        parts = ap.get_partitions()
        assert ap.ema == pytest.approx(want["ema"], rel=0, abs=0)
        assert parts == _intkeys(want["partitions"])


@pytest.mark.parametrize("case", GOLD["drift"], ids=lambda c: str(c["times"]))
def test_detect_drift_matches_reference(case):
    assert detect_drift(case["times"]) == case["drift"]


def test_solve_partitions_known_answers():
    # solver.mojo: size_i = max(1, int(flops_i/total * ffn_dim)), last takes the remainder
    nodes = [NodeCap(0, 100.0, 1000, 1000.0, 10.0), NodeCap(1, 200.0, 2000, 2000.0, 20.0),
             NodeCap(2, 300.0, 3000, 3000.0, 30.0)]
    p = solve_partitions(nodes, 1024)
    assert [(p[i].start, p[i].end) for i in range(3)] == [(0, 170), (170, 511), (511, 1024)]
    nodes5 = [NodeCap(i, 50.0 * (i + 1), 0, 0.0, 0.0) for i in range(5)]
    p5 = solve_partitions(nodes5, 2048)
    assert sum(s.size() for s in p5.values()) == 2048          # tests/test_solver.mojo:38-44
    assert [p5[i].size() for i in range(4)] == [136, 273, 409, 546]
    tiny = solve_partitions([NodeCap(0, 1e-9, 0, 0, 0), NodeCap(1, 1.0, 0, 0, 0)], 10)
    assert tiny[0].size() == 1 and tiny[1].size() == 9          # max(1, ...) floor


def test_solve_partitions_block_rounding():
    nodes = [NodeCap(0, 100.0, 0, 0, 0), NodeCap(1, 200.0, 0, 0, 0), NodeCap(2, 300.0, 0, 0, 0)]
    p = solve_partitions(nodes, 14336, block=32)
    assert all(s.start % 32 == 0 and s.end % 32 == 0 for s in p.values())
    assert p[2].end == 14336


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_dirichlet_widths(world):
    w = dirichlet_block_widths(14336, world, 5.0, 1)
    assert sum(w) == 14336 and len(w) == world
    assert all(x % 32 == 0 and x >= 32 for x in w)
    assert w == dirichlet_block_widths(14336, world, 5.0, 1)   # deterministic
    b = widths_to_bounds(w)
    assert b[0][0] == 0 and b[-1][1] == 14336
    assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))


def test_adaptive_block_rounding_covers_dim():
    ap = AdaptivePartitioner(14336, 4, block=32)
    ap.update({1: 0.010, 2: 0.012, 3: 0.020})
    parts = ap.get_partitions()
    plan = ShardPlan.from_partitions(14336, parts)
    assert sum(plan.widths) == 14336 and all(w % 32 == 0 and w > 0 for w in plan.widths)


def test_shard_plan_from_partitions_rejects_gaps():
    with pytest.raises(ValueError):
        ShardPlan.from_partitions(100, {0: {"ffn_start": 0, "ffn_end": 40}, 1: {"ffn_start": 50, "ffn_end": 100}})


def test_decoder_head_and_vocab_splits():
    """Head partition of a tensor-parallel decode layer (the reference's _solve_partitions rule,
    src/orchestrator/root_node.py:182-210) and the lm_head vocabulary split."""
    from pyre_b200.generator import head_split, vocab_split
    assert head_split(32, 8, 1) == [((0, 32), (0, 8))]
    assert head_split(32, 8, 4) == [((0, 8), (0, 2)), ((8, 16), (2, 4)), ((16, 24), (4, 6)), ((24, 32), (6, 8))]
    assert head_split(14, 2, 2) == [((0, 7), (0, 1)), ((7, 14), (1, 2))]
    assert head_split(9, 3, 2) == [((0, 6), (0, 2)), ((6, 9), (2, 3))]      # uneven: first ranks take one more
    with pytest.raises(ValueError):
        head_split(14, 2, 4)                                                # more ranks than kv heads
    for V, world in ((32768, 8), (151936, 2), (49152, 3), (10, 4)):
        parts = vocab_split(V, world)
        assert parts[0][0] == 0 and parts[-1][1] == V
        assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
        assert max(b - a for a, b in parts) - min(b - a for a, b in parts) <= 1
