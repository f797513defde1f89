#!/usr/bin/env python
"""Benchmark of the tensor-parallel Q8_0 FFN op (Mistral-7B shape) on 1..8 B200.

Workload (the isolated tensor-parallel FFN op with Mistral-7B shape): hidden 4096,
intermediate 14336, gated SiLU, gate/up/down N(0, 0.02) (seeded CUDA generator, bf16,
stored [in, out]) quantized to Q8_0 with f16 scales; activations bf16 N(0, 1). The
intermediate dim is split over the ranks with Dirichlet(5) ratios (seed 1) rounded to
32-element blocks; every rank ends with the full [T, 4096] sum.

A step is one FFN op call (gate/up + SiLU·mul, down + cross-rank sum) on one batch of
T tokens (T = 1: decode). Steps rotate over 32 distinct weight sets (one per layer of
the 7B shape), so the weights each step streams are never L2-resident (32 x shard >
126 MB L2 at every rank count). The K timed steps run as one captured CUDA graph.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
Multi-GPU: python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Q8_0 7B-shape decode tok/s + prefill tok/s at 1/2/4/8 B200; FFN % HBM roofline"
H, I = 4096, 14336
N_SETS = 32
Q8_BYTES_PER_PARAM = 34 / 32          # int8 + one f16 scale per 32
# DRAM bytes (read + write) per launch of the decode FFN kernel on the whole 4096 x 14336 shard,
# from one ncu capture (187.6 MB read, 0.7-3.3 MB written; algorithmic 187.3 MB)
FFN_DECODE_TRAFFIC_BYTES = 189_634_688
PEAKS = ROOT / "MEASURED_PEAKS.json"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--prefill-tokens", type=int, default=512)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU baseline sample")
    ap.add_argument("--sets", type=int, default=N_SETS, help="distinct weight sets the steps rotate over")
    ap.add_argument("--no-attention", action="store_true", help="skip the attention and lm_head measurements")
    ap.add_argument("--no-decoder", action="store_true", help="skip the whole-decoder (7B shape) measurement")
    ap.add_argument("--decoder-only", action="store_true",
                    help="run only the whole-decoder measurement (1 GPU) and print its JSON object")
    ap.add_argument("--decoder-prompt", type=int, default=2048)
    ap.add_argument("--decoder-tokens", type=int, default=256)
    return ap.parse_args()


def check_status(op, where):
    """A timed run counts only if no kernel stopped early on a bounded wait."""
    st = op.status()
    if st != 0:
        raise SystemExit(f"{where}: FFN kernel status {st} (a bounded wait ran out); the timing is invalid")


def peaks():
    try:
        d = json.loads(PEAKS.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), else the machine type."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or platform.machine()


# ---------------------------------------------------------------------------------------
# CPU leg: the reference's own per-call FFN arithmetic (oracle restatement).
# ---------------------------------------------------------------------------------------

def cpu_reference_leg(tokens: int, budget_s: float, steps: int | None = None):
    """Times what a reference worker does per FFN message on this host: dequantize its
    Q8_0 shard (src/orchestrator/worker_node.py:59-69 dequantizes on every access) and run
    the f32 graph (src/ffn/builder.py:37-45; numpy BLAS stands in for the MAX CPU engine),
    on the full 4096 x 14336 shard. Returns (tok/s, info)."""
    from oracle import ffn as offn, q80 as oq80
    rng = np.random.default_rng(1)
    qw = []
    for shape in ((H, I), (H, I), (I, H)):
        w = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02))
        qw.append(oq80.quantize_q80(w))
        del w
    x = rng.standard_normal((tokens, H)).astype(np.float32)
    offn.worker_ffn_step(x, *qw)                     # warm-up (page-in, BLAS threads)
    times = []
    t_all = time.perf_counter()
    n = steps if steps is not None else 10 ** 9
    while len(times) < n:
        t0 = time.perf_counter()
        offn.worker_ffn_step(x, *qw)
        times.append(time.perf_counter() - t0)
        if steps is None and time.perf_counter() - t_all > budget_s:
            break
    step = statistics.median(times)
    cores = os.cpu_count() or 1
    return tokens / step, {
        "value": tokens / step, "unit": "tok/s", "cores": cores, "kind": "port",
        "sample": f"{len(times)} reference-worker FFN calls (Q8_0 dequantize + f32 gated FFN, numpy BLAS "
                  f"with {cores} threads) on the full 4096x14336 shard at T={tokens}; median {step * 1e3:.1f} ms/call",
        "cpu_model": cpu_model(),
    }


# ---------------------------------------------------------------------------------------
# attention path (rank-local): decode attention over a 7B-shape KV cache, causal prefill
# ---------------------------------------------------------------------------------------

def attention_bench(dev, stream, hbm, tf_burst):
    """Mistral-7B attention shape (32 q heads, 8 kv heads, head_dim 128, RoPE theta 1e6).
    Decode: one token per layer over a t = 2175 cache (the mean cache length of a
    2048-token prompt plus 256 generated tokens), RoPE + append + flash-decoding, 16 layers'
    caches rotating (151 MB > L2). Prefill: causal attention of a 2048-token prompt."""
    import ctypes
    import torch
    from pyre_b200 import _native as N
    from pyre_b200.attention import AttentionOp
    nq, nkv, hd, t, layers = 32, 8, 128, 2175, 16
    gen = torch.Generator(device=dev).manual_seed(3)
    ops = [AttentionOp(nq, nkv, hd, max_t=t, rope_theta=1e6, device=dev) for _ in range(layers)]
    for o in ops:
        o.cache.k.normal_(generator=gen)
        o.cache.v.normal_(generator=gen)
    q1 = torch.randn((1, nq * hd), generator=gen, device=dev)
    k1 = torch.randn((1, nkv * hd), generator=gen, device=dev)
    v1 = torch.randn((1, nkv * hd), generator=gen, device=dev)

    def decode_all():
        for o in ops:
            o.cache.length = t - 1
            o.decode(q1, k1, v1, stream=stream)

    with torch.cuda.stream(stream):
        decode_all()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        decode_all()
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(reps):
            g.replay()
    e1.record(stream)
    stream.synchronize()
    dec_us = e0.elapsed_time(e1) * 1e3 / (reps * layers)
    kv_bytes = 2 * nkv * t * hd * 2
    del g, ops

    S = 2048
    op = AttentionOp(nq, nkv, hd, max_t=S, rope_theta=1e6, device=dev)
    qs = torch.randn((S, nq * hd), generator=gen, device=dev)
    ks = torch.randn((S, nkv * hd), generator=gen, device=dev)
    vs = torch.randn((S, nkv * hd), generator=gen, device=dev)

    def prefill_once():
        op.reset()
        op.prefill(qs, ks, vs, stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(3):
            prefill_once()
    reps = 10
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(reps):
            prefill_once()
    e1.record(stream)
    stream.synchronize()
    pf_ms = e0.elapsed_time(e1) / reps
    flops = 2 * 2 * hd * nq * S * S / 2          # causal: half of q k^T and of p v
    st = ctypes.c_int(0)
    N.call("pyre_attn_status", ctypes.byref(st))
    if st.value != 0:
        raise SystemExit(f"attention kernel status {st.value} (a bounded wait ran out); the timing is invalid")
    return {
        "shape": "Mistral-7B attention: 32 q heads, 8 kv heads, head_dim 128, f16 KV cache",
        "decode": {"cache_len": t, "us_per_layer": round(dec_us, 2), "kv_bytes_per_layer": kv_bytes,
                   "gbs": round(kv_bytes / (dec_us * 1e-6) / 1e9, 1),
                   "frac_of_hbm": round(kv_bytes / (dec_us * 1e-6) / 1e9 / hbm, 4),
                   "launches_per_layer": 1, "kernel": "attn_decode_kernel (RoPE + clip + KV append + flash-decoding, f16 mma.sync, cluster combine)",
                   "l2": f"{layers} layers' caches rotating"},
        "prefill": {"tokens": S, "ms": round(pf_ms, 4), "tflops": round(flops / (pf_ms * 1e-3) / 1e12, 1),
                    "frac_of_bf16_peak": round(flops / (pf_ms * 1e-3) / 1e12 / tf_burst, 4),
                    "kernel": "attn_prefill_tc_kernel (tcgen05, S and O in tensor memory, TMA-fed) + rope_append_kernel"},
    }


def lmhead_bench(dev, stream, hbm):
    """Mistral-7B shape last decode step: final RMSNorm + lm_head (f16 [32768, 4096], 268 MB,
    larger than L2) + greedy token, T = 1, one launch per token."""
    import torch
    from pyre_b200.lmhead import LmHeadOp
    V, Hh = 32768, 4096
    gen = torch.Generator(device=dev).manual_seed(7)
    table = (torch.randn((V, Hh), generator=gen, device=dev) * 0.02).to(torch.float16)
    norm = 1 + 0.1 * torch.randn(Hh, generator=gen, device=dev)
    op = LmHeadOp(table, norm, max_tokens=1)
    h = torch.randn((1, Hh), generator=gen, device=dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            op(h, stream=stream)
    stream.synchronize()
    reps = 20
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(reps):
            op(h, stream=stream)
    with torch.cuda.stream(stream):
        g.replay()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        g.replay()
    e1.record(stream)
    stream.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    nbytes = V * Hh * 2
    del g
    return {"shape": "Mistral-7B lm_head: vocab 32768, hidden 4096, f16 table, final RMSNorm, greedy token",
            "us_per_token": round(us, 2), "table_bytes": nbytes, "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
            "frac_of_hbm": round(nbytes / (us * 1e-6) / 1e9 / hbm, 4),
            "kernel": "lm_head_kernel (norm + f16 GEMV + argmax key, one launch)"}


# ---------------------------------------------------------------------------------------
# clocks sampler (NVML reads only)
# ---------------------------------------------------------------------------------------

class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, dev_index: int, period_s: float = 0.001):
        self.samples = []
        self.period = period_s
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(dev_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None
            self.max_mhz = None

    def _run(self):
        nv = self.nv
        get_r = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append((time.perf_counter(), nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM),
                                     int(get_r(self.h))))
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self, t0: float, t1: float):
        if self.nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        if not win and self.samples:
            mid = 0.5 * (t0 + t1)
            win = [min(self.samples, key=lambda s: abs(s[0] - mid))]
        mhz = [s[1] for s in win]
        bits = 0
        for s in win:
            bits |= s[2]
        reasons = [name for b, name in self.REASONS.items() if bits & b and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(win)}


# ---------------------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------------------

def decoder_bench(dev, hbm, prompt: int = 2048, decode: int = 256):
    """Whole Mistral-7B-shaped decoder on one GPU: hidden 4096, 32 layers, 32 query / 8 KV heads,
    head_dim 128, gated-SiLU 14336, vocab 32768 (untied f16 lm_head), RoPE theta 1e6; Q8_0
    N(0, 0.02) weights (f16 scales) made on the device from seed 3, a uniform-random prompt of
    `prompt` ids (seed 3), then `decode` greedy tokens at batch 1. Prefill: one pass of the
    prompt (tensor-core GEMMs, causal attention); decode: pyre_decoder_step replayed from CUDA
    graphs (no host synchronisation between tokens). Timed with CUDA events."""
    import numpy as np
    import torch
    from pyre_b200.generator import Generator
    from pyre_b200.quantizer import Q80Weight
    H, L, nq, nkv, hd, I, V = 4096, 32, 32, 8, 128, 14336, 32768
    g = torch.Generator(device=dev).manual_seed(3)

    def w(k, n):
        return Q80Weight.from_float((torch.randn((k, n), generator=g, device=dev) * 0.02).to(torch.bfloat16).float(),
                                    torch.float16)

    ones = torch.ones(H, device=dev)
    layers = [{"input_layernorm": ones, "post_attention_layernorm": ones,
               "attn": {"q": w(H, nq * hd), "k": w(H, nkv * hd), "v": w(H, nkv * hd), "o": w(nq * hd, H)},
               "ffn": {"gate": w(H, I), "up": w(H, I), "down": w(I, H)}} for _ in range(L)]
    emb = (torch.randn((V, H), generator=g, device=dev) * 0.02).half()
    head = (torch.randn((V, H), generator=g, device=dev) * 0.02).half()
    gen = Generator(layers, emb, ones, n_heads=nq, n_kv_heads=nkv, head_dim=hd, rope_theta=1e6, lm_head=head,
                    max_seq=prompt + decode + 1, max_prompt=prompt, device=dev)
    del layers
    ids = np.random.default_rng(3).integers(0, V, prompt)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    toks = torch.zeros(max(decode, 8) + 1, dtype=torch.int32, device=dev)
    # warm-up: a prefill and a few decode steps
    gen.prefill(ids)
    for i in range(4):
        gen.step_into(toks[i:i + 1], toks[i + 1:i + 2])
    torch.cuda.synchronize()
    pf = []
    for _ in range(3):
        e0.record()
        tok = gen.prefill(ids)
        e1.record()
        torch.cuda.synchronize()
        pf.append(e0.elapsed_time(e1))
    toks[0] = tok.reshape(-1)[0]
    torch.cuda.synchronize()
    e0.record()
    for i in range(decode - 1):
        torch.cuda.nvtx.range_push("decode")   # one step per range (ncu --nvtx-include "decode/")
        gen.step_into(toks[i:i + 1], toks[i + 1:i + 2])
        torch.cuda.nvtx.range_pop()
    e1.record()
    torch.cuda.synchronize()
    call_ms = e0.elapsed_time(e1) / (decode - 1)
    # the same steps replayed from captured CUDA graphs (16 steps per replay; the first pass
    # captures and is not timed)
    tok = gen.prefill(ids)
    gen.decode_graphed(tok, decode - 1)
    torch.cuda.synchronize()
    tok = gen.prefill(ids)
    torch.cuda.synchronize()
    e0.record()
    hist = gen.decode_graphed(tok, decode - 1)
    e1.record()
    torch.cuda.synchronize()
    dec_ms = e0.elapsed_time(e1) / (decode - 1)
    same = bool(torch.equal(hist[prompt:prompt + decode], toks[:decode]))
    gen.check_status()
    pf_ms = min(pf)
    layer_bytes = (H * (nq + 2 * nkv) * hd + nq * hd * H + 3 * H * I) * Q8_BYTES_PER_PARAM
    step_bytes = L * layer_bytes + V * H * 2
    flops = 2 * prompt * L * (H * (nq + 2 * nkv) * hd + nq * hd * H + 3 * H * I)
    del gen
    torch.cuda.empty_cache()
    return {"shape": "Mistral-7B-shaped decoder: hidden 4096, 32 layers, 32/8 heads, hd 128, FFN 14336, vocab 32768",
            "prompt_tokens": prompt, "decode_tokens": decode, "batch": 1,
            "prefill_ms": round(pf_ms, 3), "prefill_tok_s": round(prompt / (pf_ms * 1e-3), 1),
            "prefill_linear_tflops": round(flops / (pf_ms * 1e-3) / 1e12, 1),
            "decode_ms_per_token": round(dec_ms, 4), "decode_tok_s": round(1e3 / dec_ms, 1),
            "decode_ms_per_token_one_call_per_token": round(call_ms, 4),
            "graphed_tokens_equal_per_call_tokens": same,
            "decode_weight_bytes_per_token": int(step_bytes),
            "decode_frac_of_hbm": round(step_bytes / (dec_ms * 1e-3) / 1e9 / hbm, 4),
            "launches_per_decode_token": 3 + 6 * L,
            "how": "Generator.prefill (one pass); decode: Generator.decode_graphed (pyre_decoder_step with the "
                   "position on the device, 16 tokens per CUDA-graph replay), and one pyre_decoder_step call per "
                   "token for comparison; CUDA events"}


def smollm_bench(dev, reps: int = 5):
    """The SmolLM-135M-shaped decoder (hidden 576, 30 layers, 9/3 heads, hd 64, FFN 1536, vocab
    49152, tied f16 embedding, RoPE theta 1e4): 8 prompt ids from default_rng(0), 10 greedy
    tokens, end to end through Generator.generate_ids (host ids in, host ids out: prefill,
    graphed decode steps, the copies), Q8_0 N(0, 0.02) weights made on the device. Beside it,
    the oracle's numpy greedy loop (oracle/decoder.py, the reference's arithmetic) on the host
    cores for the same shapes, as the CPU baseline."""
    import numpy as np
    import torch
    from oracle import decoder as OD
    from pyre_b200.generator import Generator
    from pyre_b200.quantizer import Q80Weight
    H, L, nq, nkv, hd, I, V = 576, 30, 9, 3, 64, 1536, 49152
    g = torch.Generator(device=dev).manual_seed(0)

    def w(k, n):
        return Q80Weight.from_float(torch.randn((k, n), generator=g, device=dev) * 0.02, torch.float16)
    ones = torch.ones(H, device=dev)
    layers = [{"input_layernorm": ones, "post_attention_layernorm": ones,
               "attn": {"q": w(H, nq * hd), "k": w(H, nkv * hd), "v": w(H, nkv * hd), "o": w(nq * hd, H)},
               "ffn": {"gate": w(H, I), "up": w(H, I), "down": w(I, H)}} for _ in range(L)]
    emb = (torch.randn((V, H), generator=g, device=dev) * 0.02).half()
    gen = Generator(layers, emb, ones, n_heads=nq, n_kv_heads=nkv, head_dim=hd, rope_theta=1e4, max_seq=128,
                    max_prompt=64, device=dev)
    ids = np.random.default_rng(0).integers(0, V, 8)
    n_tok = 10
    for _ in range(2):
        gen.generate_ids(ids, n_tok, graphed=True)
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        out = gen.generate_ids(ids, n_tok, graphed=True)
        times.append(time.perf_counter() - t0)
    gpu_s = statistics.median(times)
    del gen, layers
    torch.cuda.empty_cache()
    # CPU: the oracle's greedy loop, f32 numpy, all host threads
    rng = np.random.default_rng(0)

    def wn(shape):
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    lw = [{"q": wn((H, nq * hd)), "k": wn((H, nkv * hd)), "v": wn((H, nkv * hd)), "o": wn((nq * hd, H)),
           "gate": wn((H, I)), "up": wn((H, I)), "down": wn((I, H)), "ln1": np.ones(H, np.float32),
           "ln2": np.ones(H, np.float32)} for _ in range(L)]
    emb_np = (rng.standard_normal((V, H), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    t0 = time.perf_counter()
    OD.greedy(emb_np, lw, np.ones(H, np.float32), ids, n_tok, nq, nkv, hd, 1e4)
    cpu_s = time.perf_counter() - t0
    return {"shape": "SmolLM-135M-shaped decoder: hidden 576, 30 layers, 9/3 heads, hd 64, FFN 1536, vocab 49152, "
                     "tied embeddings",
            "prompt_tokens": len(ids), "greedy_tokens": n_tok, "tokens": out,
            "e2e_s": round(gpu_s, 5), "e2e_tok_s": round(n_tok / gpu_s, 1),
            "how": "Generator.generate_ids(host ids, 10, graphed=True): prefill + CUDA-graph decode + copies, "
                   "median of 5 after 2 warm-up runs",
            "cpu_baseline": {"value": round(n_tok / cpu_s, 2), "unit": "tok/s", "cores": os.cpu_count(),
                             "kind": "port", "sample": "oracle/decoder.py greedy loop (numpy f32), same shapes, "
                                                       "one run of the 8-token prompt + 10 tokens"}}


def make_sets(rank, bounds, n_sets, device):
    """Per weight set (one per layer): full matrices from a seeded CUDA generator (identical
    on every rank), Q8_0 on the GPU, then this rank's shard."""
    import torch
    from pyre_b200.ffn import FfnWeights
    from pyre_b200.quantizer import Q80Weight
    s, e = bounds[rank]
    sets = []
    for layer in range(n_sets):
        g = torch.Generator(device=device).manual_seed(1 + 1000 * layer)
        trip = []
        for shape in ((I, H), (I, H), (H, I)):
            w = (torch.randn(shape, generator=g, device=device) * 0.02).to(torch.bfloat16).t().contiguous()
            trip.append(Q80Weight.from_float(w, torch.float16))
            del w
        gq, uq, dq = trip
        sets.append(FfnWeights.prepare(gq.cols(s, e), uq.cols(s, e), dq.rows(s, e)))
        del trip, gq, uq, dq
    torch.cuda.synchronize()
    return sets


def run_ours(args):
    import torch
    import torch.distributed as dist
    from pyre_b200 import _native as N
    from pyre_b200.ffn import FfnShardOp
    from pyre_b200.ffn.captured import CapturedFfn
    from pyre_b200.tp import ShardPlan, TPComm

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    N.load()
    hbm, tf_burst, tf_sust, peak_kind = peaks()
    T = args.tokens
    plan = ShardPlan.dirichlet(I, world, 5.0, 1)
    bounds = plan.bounds
    W = plan.widths[rank]
    n_sets = args.sets
    sets = make_sets(rank, bounds, n_sets, dev)
    comm = TPComm(H, max_tokens=max(T, args.prefill_tokens), timeout_s=5.0) if world > 1 else None
    op = FfnShardOp(H, W, max_tokens=max(T, args.prefill_tokens if not args.no_prefill else T), comm=comm, device=dev)
    gen = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn((T, H), generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty((T, H), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def capture(n_steps, with_events=False):
        g = torch.cuda.CUDAGraph()
        evs = []
        with torch.cuda.stream(stream):
            op.run(x, sets[0], out=out, stream=stream)       # eager once before capture
        stream.synchronize()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n_steps):
                wts = sets[i % n_sets]
                if with_events:
                    e = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(2)]
                    e[0].record(stream)
                    op.run(x, wts, out=out, stream=stream)     # one launch (decode kernel)
                    e[1].record(stream)
                    evs.append(e)
                else:
                    op.run(x, wts, out=out, stream=stream)
        return g, evs

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    # warm-up and timed graphs
    g_warm, _ = capture(max(args.warmup, 3))
    g_main, _ = capture(args.steps)
    g_probe, probe_ev = capture(n_sets, with_events=True)
    torch.cuda.synchronize()
    for _ in range(2):
        g_warm.replay()
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.05)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    barrier()
    with torch.cuda.stream(stream):
        g_warm.replay()
    stream.synchronize()
    barrier()
    t_wall0 = time.perf_counter()
    ev0.record(stream)
    with torch.cuda.stream(stream):
        g_main.replay()
    ev1.record(stream)
    stream.synchronize()
    t_wall1 = time.perf_counter()
    barrier()
    if comm is not None:
        comm.check(stream)
    elapsed_ms = ev0.elapsed_time(ev1)

    # per-launch durations of the decode kernel (probe graph with external event nodes
    # around each launch, over the distinct weight sets)
    k_ms = []
    for _ in range(4):
        barrier()
        with torch.cuda.stream(stream):
            g_probe.replay()
        stream.synchronize()
        for e in probe_ev:
            k_ms.append(e[0].elapsed_time(e[1]))
    sampler.stop()
    if comm is not None:
        comm.check(stream)

    # end-to-end through the public API: pinned host x in, host partial sum out, per call
    e2e_runners = [CapturedFfn(op, sets[i], tokens=T) for i in range(min(n_sets, 8))]
    xh = x.float().cpu().to(torch.bfloat16)
    for r in e2e_runners:
        r.execute(xh)
    barrier()
    e2e_steps = max(args.steps, 20)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_runners[i % len(e2e_runners)].execute(xh)
    e2e_s = time.perf_counter() - t0
    barrier()
    check_status(op, "decode and end-to-end")

    # prefill: T = 512 tokens per call, 4 weight sets rotating (prefill weight traffic is
    # amortised over 512 tokens; the GEMM is compute-bound)
    prefill = None
    if not args.no_prefill:
        TP = args.prefill_tokens
        xp = torch.randn((TP, H), generator=gen, device=dev).to(torch.bfloat16)
        outp = torch.empty((TP, H), dtype=torch.float32, device=dev)
        with torch.cuda.stream(stream):
            for i in range(3):
                op.run(xp, sets[i % n_sets], out=outp, stream=stream)
        stream.synchronize()
        n_pf = 8
        gp = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gp, stream=stream):
            for i in range(n_pf):
                op.run(xp, sets[i % n_sets], out=outp, stream=stream)
        with torch.cuda.stream(stream):
            gp.replay()
        stream.synchronize()
        barrier()
        p0 = torch.cuda.Event(enable_timing=True)
        p1 = torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        with torch.cuda.stream(stream):
            gp.replay()
        p1.record(stream)
        stream.synchronize()
        barrier()
        pf_ms = p0.elapsed_time(p1) / n_pf
        prefill = {"tokens": TP, "ms_per_step": pf_ms}
        check_status(op, "prefill")

    attn = None if args.no_attention else attention_bench(dev, stream, hbm, tf_burst)
    lmh = None if args.no_attention else lmhead_bench(dev, stream, hbm)
    barrier()
    decoder = None if (args.no_decoder or world > 1) else decoder_bench(dev, hbm, args.decoder_prompt,
                                                                        args.decoder_tokens)
    smollm = None if (args.no_decoder or world > 1) else smollm_bench(dev)

    # max over ranks
    vals = torch.tensor([elapsed_ms, e2e_s, statistics.mean(k_ms), prefill["ms_per_step"] if prefill else 0.0],
                        dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_s, k_avg, pf_ms = vals.tolist()
    clocks = sampler.summary(t_wall0, t_wall1)

    if rank == 0:
        ms_step = elapsed_ms / args.steps
        value = T / (ms_step / 1e3)
        # the decode kernel streams rank 0's shard of all three matrices once per launch
        W0 = plan.widths[0]
        k_bytes = 3 * H * W0 * Q8_BYTES_PER_PARAM + T * H * 2 + T * W0 * 4 * 2 + T * H * 4
        k_gbs = k_bytes / (k_avg * 1e-3) / 1e9
        step_bytes_all = 3 * H * I * Q8_BYTES_PER_PARAM
        res = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32 accumulate on int8 Q8_0 weights (f16 scales), bf16 activations",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": {"workload": "tensor-parallel gated-SiLU FFN op, Mistral-7B shape (hidden 4096, intermediate 14336), decode",
                       "tokens": T, "widths": list(plan.widths), "partition": "Dirichlet(5) seed 1, 32-element blocks",
                       "weight_sets": n_sets, "l2": f"inputs larger than L2: {n_sets} rotating weight sets per rank",
                       "parallelism": f"tp{world}", "timing": "K steps in one CUDA graph, CUDA events, max over ranks"},
            "roofline": {"bound": "hbm",
                         "kernel": "q80_ffn_stream_kernel (gate/up + SiLU\u00b7mul + down [+ NVLink reduce], one launch, chunk-scheduled), rank 0 shard",
                         "achieved": round(k_gbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(k_gbs / hbm, 4),
                         "peak_kind": peak_kind, "traffic": FFN_DECODE_TRAFFIC_BYTES,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, mean of 2 launches of "
                                           "q80_ffn_stream_kernel on the whole 4096x14336 shard at T=1 (one GPU)",
                         "algorithmic_bytes_per_launch": int(k_bytes), "avg_launch_us": round(k_avg * 1e3, 3),
                         "step_aggregate": {"bytes_all_ranks": int(step_bytes_all),
                                            "achieved_per_gpu": round(step_bytes_all / world / (ms_step * 1e-3) / 1e9, 1),
                                            "frac_of_aggregate": round(step_bytes_all / (ms_step * 1e-3) / 1e9 / (hbm * world), 4)}},
            "gpu_launches": args.steps * op.launches(T),
            "e2e": {"value": round(e2e_steps * T / e2e_s, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": e2e_runners[0].h2d_bytes, "d2h_bytes_per_step": e2e_runners[0].d2h_bytes,
                    "how": "CapturedFfn.execute(host x) per call: one native call (host copy into the pinned input, "
                           "graph launch: H2D copy, the op storing its result into pinned host memory "
                           "over PCIe; stream wait)"},
            "clocks": clocks,
        }
        if prefill:
            flops = 6 * args.prefill_tokens * H * I
            res["prefill"] = {"tokens": args.prefill_tokens, "ms_per_step": round(pf_ms, 4),
                              "tok_s": round(args.prefill_tokens / (pf_ms * 1e-3), 1),
                              "tflops": round(flops / (pf_ms * 1e-3) / 1e12, 2),
                              "frac_of_bf16_peak": round(flops / (pf_ms * 1e-3) / 1e12 / (tf_burst * world), 4)}
        if attn:
            res["attention"] = attn
        if lmh:
            res["lm_head"] = lmh
        if decoder:
            res["decoder_7b"] = decoder
        if smollm:
            res["decoder_smollm135m"] = smollm
        if not args.no_cpu:
            _, cpu = cpu_reference_leg(T, args.cpu_seconds)
            res["cpu_baseline"] = cpu
        print(json.dumps(res), flush=True)
    if world > 1:
        barrier()
        del g_main, g_warm, g_probe, e2e_runners
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def run_reference(args):
    """The reference's CPU FFN call on this host (rank 0 only; other ranks exit)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    T = args.tokens
    # size the sample so W + K calls fit in a few minutes
    from oracle import ffn as offn  # noqa: F401  (import check)
    steps = args.steps
    t0 = time.perf_counter()
    _, info0 = cpu_reference_leg(T, 0.0, steps=1)
    per_call = 1.0 / info0["value"] * T
    budget = 150.0
    n_w = max(0, min(args.warmup, int(budget * 0.2 / per_call)))
    n_k = max(1, min(steps, int(budget / per_call)))
    value, info = cpu_reference_leg(T, 0.0, steps=n_k + n_w)
    info["sample"] += f"; {n_k} timed of {steps} requested steps (bounded to ~{budget:.0f} s)"
    res = {"metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": "tok/s", "n_gpus": args.gpus,
           "steps": n_k, "warmup": n_w, "ms_per_step": round(1e3 * T / value, 3), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": "tensor-parallel gated-SiLU FFN op, Mistral-7B shape (hidden 4096, intermediate 14336), decode",
                      "tokens": T},
           "cpu_baseline": {k: info[k] for k in ("value", "unit", "cores", "kind", "sample")},
           "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "wall_s": round(time.perf_counter() - t0, 1)}
    print(json.dumps(res), flush=True)


def main():
    args = parse()
    if args.decoder_only:
        import torch
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        hbm, _, _, _ = peaks()
        print(json.dumps({"decoder_7b": decoder_bench(dev, hbm, args.decoder_prompt, args.decoder_tokens)}), flush=True)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
