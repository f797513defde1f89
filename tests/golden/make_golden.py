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
* attn_golden.npz      — reference ``build_ulysses_attention_graph`` (src/attention/
                         builder.py:27-65) through the numpy MAX stand-in, and
                         ``RootNode._compute_attention`` / ``_compute_attention_decode``
                         (src/orchestrator/root_node.py:250-314, :1009-1031) with the Mojo
                         kernel module replaced by the numpy restatement of
                         pyre_kernels.mojo in oracle/kernels.py (the compiled module is
                         never loaded). These pin the reference's attention orchestration:
                         concatenation order, layout, RoPE position, clipping, GQA, scale,
                         causal and padding masks.

* lmhead_golden.npz    — reference ``Generator._compute_logits`` / ``_rms_norm`` /
                         ``_sample`` at temperature 0 (src/orchestrator/generator.py:40-53):
                         final RMSNorm, logits against the f16 lm_head table, greedy token,
                         including rows with tied maxima.
* wire_golden.npz      — the reference's message framing (net.py send_msg) of three root /
                         worker messages with Q8_0 activation tuples (quantizer.py:54-67).
* greedy_golden*.npz   — the reference orchestrator's greedy decode (RootNode + Generator
                         loop) of 32 tokens on the seeded models of tests/golden/greedy_model.py:
                         the SmolLM-135M shape (projections N(0, 0.02) and N(0, 0.07)) and the
                         reduced-layer Qwen2.5-0.5B (QKV bias) and Mistral-7B shapes.

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


class _KernelShim:
    """Stands in for the pyre_kernels module: same call signatures (outputs written into
    the ``result`` array), arithmetic from oracle/kernels.py."""

    def __init__(self):
        sys.path.insert(0, str(HERE.parent.parent))
        from oracle import kernels
        self.k = kernels

    def softmax(self, x, out):
        with np.errstate(invalid="ignore", over="ignore"):
            out[...] = self.k.softmax(x)
        return out

    def apply_rope(self, x, out, theta, start_pos, frac):
        out[...] = self.k.apply_rope(x, float(theta), int(start_pos), float(frac))
        return out

    def rms_norm(self, x, w, out):
        out[...] = self.k.rms_norm(x, w)
        return out

    def apply_v_norm(self, v, out):
        v64 = v.astype(np.float64)
        out[...] = (v64 / np.sqrt(np.sum(v64 * v64, axis=-1, keepdims=True) / v.shape[-1] + 1e-6)).astype(np.float32)
        return out

    def matmul_f32(self, a, b, out):
        out[...] = (a.astype(np.float32) @ b.astype(np.float32)).astype(np.float32)
        return out

    def silu_mul(self, gate, up, out):
        out[...] = self.k.silu_mul(gate, up)
        return out


def make_attention() -> None:
    import types
    import src.orchestrator.root_node as rn
    from src.attention.builder import ShardSpec, build_ulysses_attention_graph
    from max.engine import InferenceSession
    from max.graph import DeviceRef
    from max.driver import CPU

    rn._PYRE_KERNELS = _KernelShim()
    out = {}
    # (1) QKV projection graph: 2 seq shards, GQA 8 q heads / 2 kv heads, hd 16
    H, nq, nkv, hd, S = 64, 8, 2, 16, 10
    rng = np.random.default_rng(21)
    x = bf16_round(rng.standard_normal((1, S, H)).astype(np.float32))
    wq = bf16_round(rng.standard_normal((H, nq * hd)).astype(np.float32) * 0.1)
    wk = bf16_round(rng.standard_normal((H, nkv * hd)).astype(np.float32) * 0.1)
    wv = bf16_round(rng.standard_normal((H, nkv * hd)).astype(np.float32) * 0.1)
    for i, (a, b) in enumerate(((0, 6), (6, 10))):
        shard = ShardSpec(0, nq * hd, a, b, nq, nkv, 0, 0)
        g = build_ulysses_attention_graph(shard, H, nq, nkv, hd, DeviceRef.CPU(), full_q_weights=True)
        model = InferenceSession(devices=[CPU()]).load(g)
        q, k, v = (t.to_numpy() for t in model.execute(np.ascontiguousarray(x[:, a:b]), wq, wk, wv))
        out[f"proj{i}__q"], out[f"proj{i}__k"], out[f"proj{i}__v"] = q, k, v
    out["proj__x"], out["proj__wq"], out["proj__wk"], out["proj__wv"] = x, wq, wk, wv
    out["proj__dims"] = np.array([H, nq, nkv, hd, S], dtype=np.int64)

    # (2) prefill attention over 2 nodes: seq-concatenated, and head-concatenated (GQA split)
    cfg = types.SimpleNamespace(head_dim=hd, n_heads=nq, n_kv_heads=nkv, rope_theta=10000.0)
    fake = types.SimpleNamespace(config=cfg, worker_ids=[1], _apply_rope=rn.RootNode._apply_rope,
                                 _softmax=rn.RootNode._softmax, _apply_v_norm=rn.RootNode._apply_v_norm)
    cases = [("seq_rope1", False, 1.0, False), ("seq_rope05_vnorm", False, 0.5, True), ("head_rope1", True, 1.0, False)]
    for ci, (name, by_head, frac, vn) in enumerate(cases):
        rng = np.random.default_rng(40 + ci)
        if by_head:   # each node holds all S positions of half the heads
            parts = [tuple((rng.standard_normal((1, S, n, hd)) * 3).astype(np.float32) for n in (nq // 2, nkv // 2, nkv // 2))
                     for _ in range(2)]
        else:         # each node holds a slice of the sequence with all heads
            parts = [tuple((rng.standard_normal((1, s, n, hd)) * 3).astype(np.float32) for n in (nq, nkv, nkv))
                     for s in (6, 4)]
        all_qkv = {0: parts[0], 1: parts[1]}
        props = {"rope_fraction": frac, "use_v_norm": vn}
        with np.errstate(invalid="ignore", over="ignore"):
            attn = rn.RootNode._compute_attention(fake, all_qkv, 0, None, None, props, by_head)
        for i in range(2):
            for j, t in enumerate("qkv"):
                out[f"{name}__n{i}_{t}"] = parts[i][j]
        out[f"{name}__attn"] = attn
        out[f"{name}__cfg"] = np.array([int(by_head), int(vn)], dtype=np.int64)
        out[f"{name}__frac"] = np.array(frac, dtype=np.float64)

    # (3) decode attention over a cache with a padded prefill (positions 5..7 masked)
    rng = np.random.default_rng(33)
    t = 12
    q = (rng.standard_normal((1, nq, 1, hd)) * 2).astype(np.float32)
    k = (rng.standard_normal((1, nkv, t, hd)) * 2).astype(np.float32)
    v = (rng.standard_normal((1, nkv, t, hd)) * 2).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        dec = rn.RootNode._compute_attention_decode(q, k, v, 0, prefill_real=5, prefill_max_seq=8)
    out["decode__q"], out["decode__k"], out["decode__v"], out["decode__attn"] = q, k, v, dec
    out["decode__mask"] = np.array([5, 8], dtype=np.int64)
    np.savez_compressed(HERE / "attn_golden.npz", **out)
    print("attn_golden.npz written")


def make_lmhead() -> None:
    import types
    from src.orchestrator.generator import Generator
    rng = np.random.default_rng(31)
    out = {}
    for name, (T, H, V) in {"small": (1, 64, 1000), "rows": (3, 96, 517)}.items():
        h = (rng.standard_normal((T, H)) * 3).astype(np.float32)
        w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        E = (rng.standard_normal((V, H)) * 0.05).astype(np.float16)
        if name == "rows":
            E[200] = E[7]                      # tied maxima: the first index wins
            E[301] = E[7]
            h[1] = E[7].astype(np.float32) * 40.0
        fake = types.SimpleNamespace(final_norm=w.astype(np.float16), lm_head=E)
        fake._rms_norm = lambda x, eps=1e-6, fake=fake: Generator._rms_norm(fake, x, eps)
        logits = Generator._compute_logits(fake, h)
        tok = np.concatenate([Generator._sample(logits[t:t + 1], temperature=0.0) for t in range(T)], axis=0)
        out[f"{name}__h"], out[f"{name}__w"], out[f"{name}__E"] = h, w.astype(np.float16), E
        out[f"{name}__logits"], out[f"{name}__token"] = logits.astype(np.float32), tok.astype(np.int64)
    np.savez_compressed(HERE / "lmhead_golden.npz", **out)
    print("lmhead_golden.npz written")


def make_wire(ref_root: Path, quantizer) -> None:
    """The reference's framing (src/orchestrator/net.py:18-48 send_msg, read back from a
    socketpair) of three messages a root and its workers exchange, with activations as the
    reference's Q8_0 tuples (quantize_activation, quantizer.py:54-67)."""
    import socket
    import threading
    net = _load_module(ref_root / "src" / "orchestrator" / "net.py", "ref_net")
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((1, 64, 576)) * 3).astype(np.float32)
    x1 = (rng.standard_normal((1, 1, 4096)) * 2).astype(np.float32)
    ffn = rng.standard_normal((1, 1, 896)).astype(np.float32)
    msgs = [(2, (3, quantizer.quantize_activation(x))), (10, (5, quantizer.quantize_activation(x1), 2175)),
            (6, ffn)]
    blobs = []
    for mtype, obj in msgs:
        a, b = socket.socketpair()
        t = threading.Thread(target=net.send_msg, args=(a, mtype, obj))
        t.start()
        out = bytearray()
        hdr = net.recv_exact(b, 12)
        out += hdr
        total = int.from_bytes(hdr[4:8], "big")
        out += net.recv_exact(b, total)
        t.join()
        a.close()
        b.close()
        blobs.append(np.frombuffer(bytes(out), dtype=np.uint8))
    q0, s0, sh0 = msgs[0][1][1]
    q1, s1, sh1 = msgs[1][1][1]
    np.savez_compressed(HERE / "wire_golden.npz", x=x, x1=x1, ffn=ffn, q0=q0, s0=s0, shape0=np.array(sh0),
                        q1=q1, s1=s1, shape1=np.array(sh1), msg0=blobs[0], msg1=blobs[1], msg2=blobs[2])
    print("wire_golden.npz written:", [len(b) for b in blobs], "bytes")


def make_greedy(quantizer, only: str | None = None) -> None:
    """The reference orchestrator (RootNode with no workers: head-partitioned, all heads at the
    root, src/orchestrator/root_node.py:344-380, :699-1007) and Generator's prefill / greedy
    loop (generator.py:73-145, the prompt padded to max(64, prompt length), padding masked) on
    the seeded models of greedy_model.py, with the Mojo kernels replaced by the numpy
    restatement and the MAX engine by the numpy stand-in. The root's weights are the f32
    dequantized Q8_0 matrices, as a reference worker uses them (worker_node.py:59-69), instead
    of its f16 cache; QKV biases are handed over as the root's q_bias / k_bias / v_bias."""
    import types
    import src.orchestrator.root_node as rn
    from src.orchestrator.cluster import ModelConfig
    from src.orchestrator.generator import Generator
    sys.path.insert(0, str(HERE))
    import greedy_model as gm

    def roundtrip(a):
        q, s, shape = quantizer.quantize_q80(a)
        s16 = s.astype(np.float16).astype(np.float32)
        return quantizer.dequantize_q80(q, s16, shape).astype(np.float32)

    import max.engine
    max.engine.ANY_SEQ_LEN = True       # prompts beyond the reference's fixed 64-token graph
    rn._PYRE_KERNELS = _KernelShim()
    for m in gm.MODELS.values():
        if only is not None and m.name != only:
            continue
        cfg = ModelConfig(hidden_dim=m.hidden, n_heads=m.n_heads, n_kv_heads=m.n_kv, head_dim=m.head_dim,
                          ffn_dim=m.ffn, num_layers=m.layers, vocab_size=m.vocab, rope_theta=m.theta)
        props = types.SimpleNamespace(head_dim=m.head_dim, has_v_proj=True, rope_fraction=1.0, use_v_norm=False,
                                      attention_type="full", kv_source_layer=None)
        wp = types.SimpleNamespace(get_layer_props=lambda i, props=props: props)
        emb, layers, final_norm, head = gm.build(m, roundtrip)
        root = rn.RootNode([], cfg, weight_provider=wp, num_layers=m.layers)
        _greedy_run(root, Generator, gm, m, emb, layers, final_norm, head, HERE / m.fixture)


def _greedy_run(root, Generator, gm, m, emb, layers, final_norm, head, path) -> None:
    def root_weights(i):
        lw = layers[i]
        attn = {"q": lw["q"], "k": lw["k"], "v": lw["v"], "o": lw["o"]}
        for n in ("q_bias", "k_bias", "v_bias"):
            if n in lw:
                attn[n] = lw[n]
        return {"input_layernorm": lw["ln1"], "post_attention_layernorm": lw["ln2"], "attn": attn,
                "ffn": {"gate": lw["gate"], "up": lw["up"], "down": lw["down"]},
                "_props": {"head_dim": m.head_dim, "has_v_proj": True, "rope_fraction": 1.0,
                           "use_v_norm": False, "attention_type": "full", "kv_source_layer": None}}
    root._get_root_layer_weights = root_weights
    ids = gm.prompt_ids(m)
    true_len = len(ids)
    seq_len = max(64, true_len)
    gen = Generator(root, None, lm_head=emb if head is None else head, embedding=emb, seq_len=seq_len,
                    final_norm=final_norm)
    input_ids = np.zeros((1, seq_len), dtype=np.int32)
    input_ids[0, :true_len] = ids
    kv = {}
    hs = root.run(gen._embed(input_ids), kv_cache=kv, prefill=True)
    kv["_pos"], kv["_prefill_len"], kv["_prefill_max_seq"] = true_len, true_len, seq_len
    logits = gen._compute_logits(hs)[:, true_len - 1, :]
    first_logits = logits[0].astype(np.float32)
    tokens, top_idx, top_val = [], [], []
    for step in range(gm.N_GREEDY):
        if step > 0:
            hs = root.run(gen._embed(tok.reshape(1, 1)), kv_cache=kv, prefill=False)
            logits = gen._compute_logits(hs)[:, 0, :]
        tok = gen._sample(logits, 0.0)
        tokens.append(int(tok[0, 0]))
        order = np.argsort(-logits[0], kind="stable")[:8]
        top_idx.append(order)
        top_val.append(logits[0][order].astype(np.float32))
    top_val = np.array(top_val, np.float32)
    np.savez_compressed(path, prompt=ids.astype(np.int64), tokens=np.array(tokens, np.int64),
                        first_logits=first_logits, top_idx=np.array(top_idx, np.int64), top_val=top_val)
    print(path.name, "written:", tokens, "smallest top-1/top-2 margin %.4g" % (top_val[:, 0] - top_val[:, 1]).min())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--only", default=None,
                    help="write one fixture: lmhead, wire, greedy (every greedy model) or greedy:<model name>")
    args = ap.parse_args()
    ref = Path(args.ref)
    sys.path.insert(0, str(HERE / "max_shim"))
    sys.path.insert(0, str(ref))
    if args.only == "lmhead":
        make_lmhead()
        return
    if args.only == "wire":
        make_wire(ref, _load_module(ref / "src" / "orchestrator" / "quantizer.py", "ref_quantizer"))
        return
    if args.only is not None and args.only.startswith("greedy"):
        name = args.only.split(":", 1)[1] if ":" in args.only else None
        make_greedy(_load_module(ref / "src" / "orchestrator" / "quantizer.py", "ref_quantizer"), name)
        return
    quantizer = _load_module(ref / "src" / "orchestrator" / "quantizer.py", "ref_quantizer")
    make_q80(quantizer)
    make_ffn(ref, quantizer)
    import io, contextlib
    with contextlib.redirect_stdout(io.StringIO()):
        make_partition()
    print("partition_golden.json written")
    make_attention()
    make_lmhead()
    make_wire(ref, quantizer)
    make_greedy(quantizer)


if __name__ == "__main__":
    main()
