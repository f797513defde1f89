"""Writes the golden fixtures of tests/golden/ by running the reference's own code.

Run in a container that has the reference checkout (read-only) at /root/reference:

    python tests/golden/make_golden.py [--ref /root/reference]

* q80_golden.npz       — reference ``quantize_q80`` (src/orchestrator/quantizer.py:11-26)
                         on seeded inputs plus hand-made edge blocks (zeros, ties at
                         .5 of the scale, padding, tiny and huge magnitudes).
* ffn_golden.npz       — reference ``compile_and_run`` / ``build_ffn_graph``
                         (src/ffn/builder.py:20-83) evaluated with the numpy MAX stand-in
                         in tests/golden/max_shim: the reference test's ungated 3-shard
                         case (tests/test_ffn_builder.py:16-51) and a gated non-uniform
                         3-shard case on Q8_0-roundtripped weights.
* partition_golden.json— reference ``AdaptivePartitioner`` / ``detect_drift``
                         (src/orchestrator/cluster.py:217-403) on fixed timing traces.

Only this script touches /root/reference; tests read the fixtures.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bfloat16, returned as float32 (what the reference loader's
    ``.to(torch.bfloat16)`` then ``.to(torch.float32)`` produces)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def q80_cases() -> dict:
    rng = np.random.default_rng(0)
    cases = {}
    cases["normal_64x96"] = rng.standard_normal((64, 96)).astype(np.float32)
    cases["weights_bf16_128x64"] = bf16_round(rng.standard_normal((128, 64)).astype(np.float32) * 0.02)
    cases["ragged_1000"] = (rng.standard_normal(1000) * 3).astype(np.float32)
    cases["ragged_77"] = rng.uniform(-5, 5, 77).astype(np.float32)
    # tie blocks: absmax 127 -> scale exactly 1.0, values k + 0.5 tie; absmax 254 -> scale 2
    ties = np.zeros((4, 32), dtype=np.float32)
    ties[0, 0] = 127.0
    ties[0, 1:] = np.arange(-15.5, 15.5, 1.0, dtype=np.float32)[:31]
    ties[1, 0] = -127.0
    ties[1, 1:] = (np.arange(31, dtype=np.float32) - 15) + 0.5
    ties[2, 0] = 254.0
    ties[2, 1:] = (np.arange(31, dtype=np.float32) * 2 - 31)
    ties[3, :] = np.linspace(-63.5, 63.5, 32, dtype=np.float32)
    ties[3, 0] = 127.0
    cases["ties_4x32"] = ties
    edge = np.zeros((6, 32), dtype=np.float32)
    edge[1, 5] = 3.0                                   # one non-zero
    edge[2, :] = 1e-30 * np.linspace(-1, 1, 32)        # tiny normal values
    edge[3, :] = 3e38 * np.linspace(-1, 1, 32)         # near f32 max
    edge[4, :] = np.float32(1e-44) * np.arange(32)     # subnormal absmax (scale underflows to 0)
    edge[5, :] = -2.0
    edge[5, 7] = 2.0
    cases["edge_6x32"] = edge
    return cases


def make_q80(quantizer) -> None:
    out = {}
    for name, arr in q80_cases().items():
        with np.errstate(all="ignore"):
            q, s, shape = quantizer.quantize_q80(arr)
        out[f"{name}__x"] = arr
        out[f"{name}__q"] = q
        out[f"{name}__s"] = s
        out[f"{name}__shape"] = np.array(shape, dtype=np.int64)
    np.savez_compressed(HERE / "q80_golden.npz", **out)
    print("q80_golden.npz:", len(out) // 4, "cases")


def make_ffn(ref_root: Path, quantizer) -> None:
    from src.ffn.builder import ShardSpec, build_ffn_graph, compile_and_run  # reference code
    from max.engine import InferenceSession
    from max.graph import DeviceRef
    from max.driver import CPU

    out = {}
    # (1) the reference's own test: tests/test_ffn_builder.py:16-51 (ungated, 3 shards)
    hidden_dim, ffn_total, seq_len = 768, 3072, 4
    rng = np.random.default_rng(42)
    x = rng.standard_normal((1, seq_len, hidden_dim)).astype(np.float32)
    up = rng.standard_normal((hidden_dim, ffn_total)).astype(np.float32)
    down = rng.standard_normal((ffn_total, hidden_dim)).astype(np.float32)
    parts = []
    for s in [ShardSpec(0, 1024), ShardSpec(1024, 2048), ShardSpec(2048, 3072)]:
        with np.errstate(over="ignore"):
            parts.append(compile_and_run(s, hidden_dim, x, up[:, s.ffn_dim_start:s.ffn_dim_end],
                                         down[s.ffn_dim_start:s.ffn_dim_end, :]))
    out["ungated__partials"] = np.stack(parts)
    out["ungated__x_sha"] = np.array(sha(x))
    out["ungated__up_sha"] = np.array(sha(up))
    out["ungated__down_sha"] = np.array(sha(down))

    # (2) gated, non-uniform 3 shards, Q8_0 weights as a reference worker holds them
    H, I, T = 256, 384, 2
    bounds = [(0, 96), (96, 256), (256, 384)]
    rng = np.random.default_rng(7)
    wg = bf16_round(rng.standard_normal((H, I)).astype(np.float32) * 0.02)
    wu = bf16_round(rng.standard_normal((H, I)).astype(np.float32) * 0.02)
    wd = bf16_round(rng.standard_normal((I, H)).astype(np.float32) * 0.02)
    xg = bf16_round(rng.standard_normal((1, T, H)).astype(np.float32))
    parts = []
    qs = {}
    for name, w in (("gate", wg), ("up", wu), ("down", wd)):
        q, s, sh = quantizer.quantize_q80(w)
        qs[name] = (q, s, sh)
        out[f"gated__{name}_q"] = q
        out[f"gated__{name}_s"] = s
    deq = {k: quantizer.dequantize_q80(*v) for k, v in qs.items()}
    for a, b in bounds:
        g = build_ffn_graph(ShardSpec(a, b), H, DeviceRef.CPU(), seq_len=T, gated=True)
        model = InferenceSession(devices=[CPU()]).load(g)
        (p,) = model.execute(xg, np.ascontiguousarray(deq["gate"][:, a:b]), np.ascontiguousarray(deq["up"][:, a:b]),
                             np.ascontiguousarray(deq["down"][a:b, :]))
        parts.append(p.to_numpy())
    out["gated__x"] = xg
    out["gated__bounds"] = np.array(bounds, dtype=np.int64)
    out["gated__partials"] = np.stack(parts)
    np.savez_compressed(HERE / "ffn_golden.npz", **out)
    print("ffn_golden.npz written")


def make_partition() -> None:
    from src.orchestrator.cluster import AdaptivePartitioner, ClusterOrchestrator, NodeCap, ModelConfig

    res = {"adaptive": [], "drift": []}
    scenarios = [
        (14336, 2, [[{0: 1.0, 1: 1.3}] * 3]),
        (14336, 4, [[{1: 0.010, 2: 0.012, 3: 0.020}] * 4, [{1: 0.011, 2: 0.011, 3: 0.011}] * 2]),
        (1536, 3, [[{1: 0.5, 2: 0.25}]]),
        (4864, 8, [[{i: 0.01 * (1 + 0.1 * i) for i in range(1, 8)}] * 5]),
        (3072, 3, [[]]),
    ]
    for ffn_dim, n, passes in scenarios:
        ap = AdaptivePartitioner(ffn_dim, n, seq_len=64)
        trace = []
        for layer_updates in passes:
            ap.reset_pass()
            for upd in layer_updates:
                ap.update(upd)
            drift = ap.drift_detected()
            parts = ap.get_partitions()
            trace.append({"drift": drift, "ema": list(ap.ema),
                          "partitions": {str(k): v for k, v in parts.items()}})
        res["adaptive"].append({"ffn_dim": ffn_dim, "n": n,
                                "passes": [[{str(k): v for k, v in u.items()} for u in lu] for lu in passes],
                                "trace": trace,
                                "equal": {str(k): v for k, v in AdaptivePartitioner.equal_partitions(ffn_dim, n).items()}})
    nodes = [NodeCap(i, 100.0, 1, 1.0, 1.0) for i in range(3)]
    orch = ClusterOrchestrator(nodes, ModelConfig(hidden_dim=64, n_heads=1, n_kv_heads=1, head_dim=64, ffn_dim=128))
    for times in ([10.0, 10.1, 13.5], [1.0, 1.0, 1.0], [1.0, 1.14, 1.0], [], [5.0], [1.0, 2.0]):
        res["drift"].append({"times": times, "drift": bool(orch.detect_drift(list(times)))})
    (HERE / "partition_golden.json").write_text(json.dumps(res, indent=1, sort_keys=True))
    print("partition_golden.json written")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    args = ap.parse_args()
    ref = Path(args.ref)
    sys.path.insert(0, str(HERE / "max_shim"))
    sys.path.insert(0, str(ref))
    quantizer = _load_module(ref / "src" / "orchestrator" / "quantizer.py", "ref_quantizer")
    make_q80(quantizer)
    make_ffn(ref, quantizer)
    import io, contextlib
    with contextlib.redirect_stdout(io.StringIO()):
        make_partition()
    print("partition_golden.json written")


if __name__ == "__main__":
    main()
