"""Prefill + greedy decode of a Llama-style decoder on this library's kernels.

Mirrors the reference's single-sequence generation loop, ``Generator.generate``
(src/orchestrator/generator.py:60-145), over the head-partitioned root layer
(``RootNode._decode_single_layer``, src/orchestrator/root_node.py:739-1007, and the prefill
layer at :344-600): per layer

    xn = rms_norm(x, input_layernorm)                     root_node.py:752
    q, k, v = xn @ Wq, xn @ Wk, xn @ Wv                   :866-897   (one Q8_0 GEMM, [Wq|Wk|Wv])
    a = attention(rope(q), rope(k) -> cache, v -> cache)  :899-945   (clip +-1000, causal / masked)
    h = x + a @ Wo;  hn = rms_norm(h, post_attn_ln)       :940-951   (one add+norm launch)
    f = down(silu(hn @ Wgate) * (hn @ Wup))               :953-979   (the FFN shard op)
    x = h + f;  xn' = rms_norm(x, next input_ln)          :997       (one add+norm launch)

and ``_embed`` / ``_compute_logits`` / ``_sample(temperature < 0.01)`` (generator.py:38-53) as
one embedding-gather launch and one lm_head + argmax launch. The reference pads the prompt to
``seq_len`` and masks the padding in every decode step (generator.py:77-85, root_node.py:
1024-1025); padding sits after the prompt and attention is causal, so running the true
prompt alone gives the same hidden states, and decode positions (RoPE angle = number of
tokens so far, root_node.py:907-916) are the same.

Weights per layer are given as the reference's root weight dict
(``_get_root_layer_weights``, root_node.py:1033-1048): ``input_layernorm``,
``post_attention_layernorm``, ``attn: {q, k, v, o}``, ``ffn: {gate, up, down}``; matrices are
``[in, out]`` (``x @ W``) as :class:`~pyre_b200.quantizer.Q80Weight` (f16 scales) or float
arrays, which are quantized to Q8_0 on the device.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _device as D
from . import _native as N
from .attention.ops import AttentionOp, KVCache, Q80Linear
from .ffn.op import FfnShardOp, FfnWeights
from .lmhead import LmHeadOp
from .quantizer import Q80Weight


class DecoderLayerDesc(ctypes.Structure):
    """``pyre_decoder_layer`` of include/pyre_b200.h."""
    _fields_ = [("qkv_w", ctypes.c_void_p), ("qkv_ws", ctypes.c_void_p), ("qkv_ws_bytes", ctypes.c_int64),
                ("o_w", ctypes.c_void_p), ("o_ws", ctypes.c_void_p), ("o_ws_bytes", ctypes.c_int64),
                ("gateup_w", ctypes.c_void_p), ("down_w", ctypes.c_void_p), ("gated", ctypes.c_int),
                ("ffn_ws", ctypes.c_void_p), ("ffn_ws_bytes", ctypes.c_int64),
                ("ln1", ctypes.c_void_p), ("ln2", ctypes.c_void_p), ("k_cache", ctypes.c_void_p),
                ("v_cache", ctypes.c_void_p), ("rope", ctypes.c_void_p), ("attn_ws", ctypes.c_void_p),
                ("attn_ws_bytes", ctypes.c_int64), ("qkv_bias", ctypes.c_void_p)]


class DecoderDesc(ctypes.Structure):
    """``pyre_decoder_desc`` of include/pyre_b200.h."""
    _fields_ = [(n, ctypes.c_int) for n in ("n_layers", "H", "nq", "nkv", "hd", "ffn_width", "V", "max_t",
                                             "scale_dtype")] + \
               [("eps", ctypes.c_double), ("rope_fraction", ctypes.c_double),
                ("layers", ctypes.POINTER(DecoderLayerDesc)), ("embedding", ctypes.c_void_p),
                ("lm_head", ctypes.c_void_p), ("final_norm", ctypes.c_void_p), ("lm_ws", ctypes.c_void_p),
                ("lm_ws_bytes", ctypes.c_int64)] + \
               [(n, ctypes.c_void_p) for n in ("x", "xn", "hn", "qkv", "attn", "ao", "f", "status", "key",
                                                "pos_dev", "history", "comm")] + \
               [("lm_v0", ctypes.c_int64), ("lm_V", ctypes.c_int), ("batch", ctypes.c_int)]


def check_struct_layout() -> None:
    """The ctypes structs above against the library's sizeof (raises on a mismatch)."""
    lb, db = ctypes.c_int64(0), ctypes.c_int64(0)
    N.call("pyre_decoder_struct_sizes", ctypes.byref(lb), ctypes.byref(db))
    if (lb.value, db.value) != (ctypes.sizeof(DecoderLayerDesc), ctypes.sizeof(DecoderDesc)):
        raise RuntimeError(f"decoder struct layout differs from the library's: {(lb.value, db.value)} vs "
                           f"{(ctypes.sizeof(DecoderLayerDesc), ctypes.sizeof(DecoderDesc))}")


def _q80(w, device) -> Q80Weight:
    if isinstance(w, Q80Weight):
        return Q80Weight(w.q.to(device), w.scale.to(device, torch.float16))
    t = torch.as_tensor(np.asarray(w, dtype=np.float32)) if not isinstance(w, torch.Tensor) else w.float()
    return Q80Weight.from_float(t.to(device), scale_dtype=torch.float16)


def _concat_n(ws: list[Q80Weight]) -> Q80Weight:
    """[K, N1] | [K, N2] | ... -> [K, N1 + N2 + ...]: Q8_0 blocks run along N in 32s, so with
    every N a multiple of 32 the blocks (and scales) of the parts are the blocks of the whole."""
    return Q80Weight(torch.cat([w.q for w in ws], dim=1).contiguous(), torch.cat([w.scale for w in ws], dim=1).contiguous())


def _f32(v) -> torch.Tensor:
    return v.detach().float() if isinstance(v, torch.Tensor) else torch.as_tensor(np.asarray(v, dtype=np.float32))


def _ffn_dim(lw: dict) -> int:
    up = lw["ffn"]["up"]
    return int(up.shape[1])


def _vec(v, H, device) -> torch.Tensor:
    t = _f32(v).reshape(-1)
    if t.numel() != H:
        raise ValueError(f"norm weight must have {H} elements")
    return t.to(device).contiguous()


def head_split(n_heads: int, n_kv: int, world: int) -> list[tuple]:
    """Per rank ((q0, q1), (k0, k1)): the reference's head partition of a decode layer
    (``RootNode._solve_partitions``, src/orchestrator/root_node.py:182-210): n_kv // world kv
    heads per rank, one more for the first n_kv % world, and the query heads that share them
    (n_heads // n_kv per kv head), contiguous in rank order."""
    if n_heads % n_kv:
        raise ValueError("n_heads must be a multiple of n_kv_heads")
    if world > n_kv:
        raise ValueError(f"head-parallel decode needs world <= n_kv_heads ({world} > {n_kv})")
    per, extra = divmod(n_kv, world)
    rep = n_heads // n_kv
    out, k0 = [], 0
    for r in range(world):
        k1 = k0 + per + (1 if r < extra else 0)
        out.append(((k0 * rep, k1 * rep), (k0, k1)))
        k0 = k1
    return out


def vocab_split(V: int, world: int) -> list[tuple]:
    """Contiguous lm_head row ranges per rank (V // world, the remainder to the first ranks)."""
    per, extra = divmod(V, world)
    out, v0 = [], 0
    for r in range(world):
        v1 = v0 + per + (1 if r < extra else 0)
        out.append((v0, v1))
        v0 = v1
    return out


def _bias_part(attn: dict, name: str, lo: int, hi: int):
    b = attn.get(name)
    if b is None:
        return None
    return _f32(b).reshape(-1)[lo:hi]


class _Layer:
    """One decoder layer on this rank: the QKV columns and O rows of its heads (all heads on one
    GPU), its FFN shard, norms, KV cache and the kernels' scratch."""

    def __init__(self, lw: dict, H: int, nq: int, nkv: int, hd: int, max_seq: int, max_prompt: int, theta: float,
                 frac: float, device, heads=None, ffn_range=None, comm=None, batch: int = 1):
        attn, ffn = lw["attn"], lw["ffn"]
        q, k, v, o = (_q80(attn[n], device) for n in ("q", "k", "v", "o"))
        if q.shape != (H, nq * hd) or k.shape != (H, nkv * hd) or v.shape != (H, nkv * hd) or o.shape != (nq * hd, H):
            raise ValueError("attention weights do not match the head counts")
        (q0, q1), (k0, k1) = heads if heads is not None else ((0, nq), (0, nkv))
        self.nq, self.nkv = q1 - q0, k1 - k0
        if (q0, q1, k0, k1) != (0, nq, 0, nkv):
            q, k, v = q.cols(q0 * hd, q1 * hd), k.cols(k0 * hd, k1 * hd), v.cols(k0 * hd, k1 * hd)
            o = o.rows(q0 * hd, q1 * hd)
        parts = [_bias_part(attn, "q_bias", q0 * hd, q1 * hd), _bias_part(attn, "k_bias", k0 * hd, k1 * hd),
                 _bias_part(attn, "v_bias", k0 * hd, k1 * hd)]
        bias = None
        if any(b is not None for b in parts):
            widths = ((q1 - q0) * hd, (k1 - k0) * hd, (k1 - k0) * hd)
            bias = torch.cat([b if b is not None else torch.zeros(w) for b, w in zip(parts, widths)])
        self.qkv = Q80Linear(_concat_n([q, k, v]), max_prompt, device, bias=bias)
        self.o = Q80Linear(o, max_prompt, device)
        gate = _q80(ffn["gate"], device) if ffn.get("gate") is not None else None
        up, down = _q80(ffn["up"], device), _q80(ffn["down"], device)
        if ffn_range is not None:
            s0, s1 = ffn_range
            gate = gate.cols(s0, s1) if gate is not None else None
            up, down = up.cols(s0, s1), down.rows(s0, s1)
        self.ffn_w = FfnWeights.prepare(gate, up, down)
        self.ffn = FfnShardOp(H, self.ffn_w.width, max_prompt, gated=gate is not None, comm=comm, device=device)
        self.comm = comm
        self.ln1 = _vec(lw["input_layernorm"], H, device)
        self.ln2 = _vec(lw["post_attention_layernorm"], H, device)
        self.attn = AttentionOp(self.nq, self.nkv, hd, max_seq, rope_theta=theta, rope_fraction=frac, device=device)
        self.attns = [self.attn]
        self.batch_ws = None
        if batch > 1:
            # a static batch: the sequences' caches stacked [B, nkv, max_t, hd] (the batched decode
            # step reads them as B * nkv kv heads), one attention op per sequence over its slice
            self.kv_k = torch.zeros((batch, self.nkv, max_seq, hd), dtype=torch.float16, device=device)
            self.kv_v = torch.zeros_like(self.kv_k)
            self.attns = [AttentionOp(self.nq, self.nkv, hd, max_seq, rope_theta=theta, rope_fraction=frac,
                                      device=device, cache=KVCache(self.nkv, max_seq, hd, device, self.kv_k[b],
                                                                   self.kv_v[b]), rope=self.attn.rope)
                          for b in range(batch)]
            self.attn = self.attns[0]
            nb = ctypes.c_int64(0)
            N.call("pyre_attn_decode_workspace_bytes", batch * self.nq, batch * self.nkv, hd, max_seq, ctypes.byref(nb))
            self.batch_ws = torch.zeros(int(nb.value), dtype=torch.uint8, device=device)

    def o_proj(self, a: torch.Tensor, stream=None) -> torch.Tensor:
        """a @ Wo for this rank's heads; with tensor parallelism summed over the ranks (the
        root's concatenation of every node's head outputs before Wo, root_node.py:851-858)."""
        if self.comm is None:
            return self.o(a, stream=stream)
        T, H = a.shape[0], self.o.n
        out = torch.empty((T, H), dtype=torch.float32, device=a.device)
        ws = self.o.workspace
        N.call("pyre_ffn_down_q80", D.ptr(a), D.dtype_code(a), T, self.o.k, D.ptr(self.o.w.data),
               self.o.w.scale_code, H, D.ptr(out), D.ptr(ws), ws.numel(), ctypes.c_void_p(self.comm.handle),
               D.stream_ptr(stream))
        return out


class Generator:
    """Greedy generation over token ids (the tokenizer stays with the caller)."""

    def __init__(self, layers: list[dict], embedding, final_norm=None, *, n_heads: int, n_kv_heads: int,
                 head_dim: int, rope_theta: float = 10000.0, rope_fraction: float = 1.0, eps: float = 1e-6,
                 lm_head=None, max_seq: int = 4096, max_prompt: int = 64, device=None, comm=None, ffn_plan=None,
                 batch: int = 1, persistent: bool = False):
        """``comm`` (a :class:`~pyre_b200.tp.TPComm` of hidden size H and at least ``max_prompt``
        tokens) makes this object one rank of a tensor-parallel decoder: it keeps the heads
        :func:`head_split` gives its rank (QKV columns, O rows, KV cache), the FFN columns
        ``ffn_plan`` (a :class:`~pyre_b200.tp.ShardPlan`, default equal 32-blocks) gives it and
        the lm_head rows of :func:`vocab_split`; every rank is given the same full weights and
        runs the same calls. Without it the whole model runs on this GPU.

        ``batch`` > 1 keeps that many KV caches per layer for a static batch of equally long
        prompts decoded in lockstep (:meth:`generate_batch`).

        ``persistent``: decode steps (:meth:`step_into`, :meth:`decode_graphed`) run every layer
        of a token in one persistent launch (``pyre_decoder_step_persistent``: one sequence on one
        GPU) instead of six launches per layer. Off by default: on the Mistral-7B shape it is
        measured slower than the launch-per-op step (3.77 against 2.70 ms per token on a B200)."""
        D.require_cuda()
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        # the reference keeps embedding, lm_head and final norm as f16 (generator.py:31-34)
        emb = torch.as_tensor(np.asarray(embedding)) if not isinstance(embedding, torch.Tensor) else embedding
        self.embedding = emb.to(dev, torch.float16).contiguous()
        self.V, self.H = self.embedding.shape
        table = self.embedding if lm_head is None else (
            lm_head if isinstance(lm_head, torch.Tensor) else torch.as_tensor(np.asarray(lm_head))).to(dev, torch.float16)
        fn = None
        if final_norm is not None:
            fn = _f32(final_norm).half().float()
        self.comm = comm
        rank, world = (comm.rank, comm.world) if comm is not None else (0, 1)
        self.rank, self.world = rank, world
        if comm is not None and (comm.hidden != self.H or comm.max_tokens < max_prompt):
            raise ValueError("the communicator needs hidden = H and max_tokens >= max_prompt")
        heads = head_split(n_heads, n_kv_heads, world)[rank]
        ffn_dim = _ffn_dim(layers[0])
        if ffn_plan is None:
            from .tp import ShardPlan
            ffn_plan = ShardPlan.equal(ffn_dim, world)
        if ffn_plan.ffn_dim != ffn_dim or len(ffn_plan.widths) != world:
            raise ValueError("ffn_plan does not match the FFN width or the world size")
        ffn_range = ffn_plan.bounds[rank] if world > 1 else None
        self.lm_v0, v1 = vocab_split(self.V, world)[rank]
        if not 1 <= batch <= 64:
            raise ValueError("batch must be in [1, 64]")
        self.batch = int(batch)
        self.lm_head = LmHeadOp(table[self.lm_v0:v1].contiguous(), fn, eps, vocab_start=self.lm_v0, comm=comm,
                                max_tokens=min(4, self.batch))
        self.eps = float(eps)
        self.n_heads, self.n_kv_heads = n_heads, n_kv_heads
        self.nq, self.nkv, self.hd = heads[0][1] - heads[0][0], heads[1][1] - heads[1][0], head_dim
        self.max_seq, self.max_prompt = int(max_seq), int(max_prompt)
        self.layers = [_Layer(lw, self.H, n_heads, n_kv_heads, head_dim, self.max_seq, self.max_prompt, rope_theta,
                              rope_fraction, dev, heads=heads, ffn_range=ffn_range, comm=comm, batch=self.batch)
                       for lw in layers]
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.length = 0
        self._desc = self._native_desc()
        self.tokens = torch.zeros(self.max_seq + 1, dtype=torch.int32, device=dev)
        self._pws = None
        if persistent:
            nb = ctypes.c_int64(0)
            N.call("pyre_decoder_persistent_workspace_bytes", ctypes.byref(self._desc), ctypes.byref(nb))
            self._pws = torch.zeros(int(nb.value), dtype=torch.uint8, device=dev)

    @property
    def persistent(self) -> bool:
        """Whether decode steps run as one persistent launch per token."""
        return self._pws is not None

    def _decode_call(self, desc, token_in_ptr, pos: int, token_out_ptr, logits_ptr, stream_ptr) -> None:
        if self._pws is not None:
            N.call("pyre_decoder_step_persistent", ctypes.byref(desc), D.ptr(self._pws), self._pws.numel(),
                   token_in_ptr, pos, token_out_ptr, logits_ptr, stream_ptr)
        else:
            N.call("pyre_decoder_step", ctypes.byref(desc), token_in_ptr, pos, 0, 0, token_out_ptr, logits_ptr,
                   stream_ptr)

    def _native_desc(self) -> DecoderDesc:
        """The descriptor of pyre_decoder_step: pointers into this object's buffers (which it
        keeps alive), built once."""
        check_struct_layout()
        dev, H = self.device, self.H
        codes = {c for L in self.layers for c in (L.qkv.w.scale_code, L.o.w.scale_code, L.ffn_w.gateup.scale_code)}
        if len(codes) != 1:
            raise ValueError("every matrix needs the same scale dtype")
        widths = {L.ffn_w.width for L in self.layers}
        if len(widths) != 1:
            raise ValueError("every layer needs the same FFN width")
        nqkv = (self.nq + 2 * self.nkv) * self.hd
        B = self.batch
        self._buf = {n: torch.zeros(B * k, dtype=torch.float32, device=dev)
                     for n, k in (("x", H), ("xn", H), ("hn", H), ("qkv", nqkv), ("attn", self.nq * self.hd),
                                  ("ao", H), ("f", H))}
        self._key = torch.zeros(B, dtype=torch.int64, device=dev)
        arr = (DecoderLayerDesc * len(self.layers))()
        for i, L in enumerate(self.layers):
            kc, vc = (L.kv_k, L.kv_v) if B > 1 else (L.attn.cache.k, L.attn.cache.v)
            aws = L.batch_ws if B > 1 else L.attn.dec_ws
            arr[i] = DecoderLayerDesc(
                L.qkv.w.data.data_ptr(), L.qkv.workspace.data_ptr(), L.qkv.workspace.numel(),
                L.o.w.data.data_ptr(), L.o.workspace.data_ptr(), L.o.workspace.numel(),
                L.ffn_w.gateup.data.data_ptr(), L.ffn_w.down.data.data_ptr(), int(L.ffn_w.gated),
                L.ffn.workspace.data_ptr(), L.ffn.workspace.numel(), L.ln1.data_ptr(), L.ln2.data_ptr(),
                kc.data_ptr(), vc.data_ptr(), L.attn.rope.data_ptr(), aws.data_ptr(), aws.numel(),
                L.qkv.bias.data_ptr() if L.qkv.bias is not None else None)
        self._layer_arr = arr
        lm = self.lm_head
        d = DecoderDesc(len(self.layers), H, self.nq, self.nkv, self.hd, widths.pop(), self.V, self.max_seq,
                        codes.pop(), self.eps, float(self.layers[0].attn.frac),
                        ctypes.cast(arr, ctypes.POINTER(DecoderLayerDesc)), self.embedding.data_ptr(),
                        lm.table.data_ptr(), lm.norm.data_ptr() if lm.norm is not None else None,
                        lm.workspace.data_ptr(), lm.workspace.numel(),
                        *(self._buf[n].data_ptr() for n in ("x", "xn", "hn", "qkv", "attn", "ao", "f")),
                        self.status.data_ptr(), self._key.data_ptr(), None, None,
                        self.comm.handle if self.comm is not None else None, self.lm_v0, lm.V, B)
        return d

    # ---- one pass of the decoder over T new tokens ------------------------------------------
    def _forward(self, ids: torch.Tensor, prefill: bool, stream=None, seq: int = 0) -> torch.Tensor:
        """ids: int32 [T] on the device (the prompt, or one decode token) of batch sequence
        ``seq``. Returns the last hidden state, f32 [1, H]."""
        T, H = ids.numel(), self.H
        s = D.stream_ptr(stream)
        x = torch.empty((T, H), dtype=torch.float32, device=self.device)
        xn = torch.empty_like(x)
        hn = torch.empty_like(x)
        first = self.layers[0]
        N.call("pyre_embed_rms_norm", D.ptr(ids), T, D.ptr(self.embedding), self.V, H, D.ptr(first.ln1), self.eps,
               D.ptr(x), D.ptr(xn), D.ptr(self.status), s)
        nq_w, nkv_w = self.nq * self.hd, self.nkv * self.hd
        for i, L in enumerate(self.layers):
            qkv = L.qkv(xn, stream=stream)
            q, k, v = qkv[:, :nq_w], qkv[:, nq_w:nq_w + nkv_w], qkv[:, nq_w + nkv_w:]
            att = L.attns[seq]
            a = att.prefill(q, k, v, stream=stream) if prefill else att.decode(q, k, v, stream=stream)
            ao = L.o_proj(a, stream=stream)
            N.call("pyre_add_rms_norm", D.ptr(x), D.ptr(ao), T, H, D.ptr(L.ln2), self.eps, D.ptr(x), D.ptr(hn), s)
            f = L.ffn.run(hn, L.ffn_w, stream=stream)
            nxt = self.layers[i + 1] if i + 1 < len(self.layers) else None
            N.call("pyre_add_rms_norm", D.ptr(x), D.ptr(f), T, H, D.ptr(nxt.ln1) if nxt else None, self.eps, D.ptr(x),
                   D.ptr(xn) if nxt else None, s)
        return x[T - 1:T]

    def reset(self) -> None:
        for L in self.layers:
            for a in L.attns:
                a.reset()
        self.length = 0

    # captured prefill graphs kept at once (least recently used dropped first)
    PREFILL_GRAPHS = 8

    def _prefill_graphed(self, ids: np.ndarray) -> torch.Tensor:
        """The one-pass prefill plus lm_head replayed from a CUDA graph captured once per prompt
        length (the ids are copied into a fixed device buffer first; the graph writes the
        caches in place and leaves the first greedy token in its own output buffer).

        Memory: every captured graph draws its activations ([T, H] rows, the QKV / attention /
        FFN intermediates of one prompt length) from one memory pool shared by all of this
        object's prefill graphs (they only ever replay one at a time, on one stream), and at
        most PREFILL_GRAPHS lengths are kept, so serving many prompt lengths holds about the
        activations of the longest prompt, not one set per length."""
        T = int(ids.size)
        dev = self.device
        if not hasattr(self, "_pf_graphs"):
            self._pf_graphs = {}                 # insertion order = least recently used first
            self._pf_pool = torch.cuda.graph_pool_handle()
            self._pf_ids = torch.zeros(self.max_prompt, dtype=torch.int32, device=dev)
            self._pf_stream = torch.cuda.Stream(dev)
        self._pf_ids[:T].copy_(torch.from_numpy(ids.astype(np.int32)))
        cur = torch.cuda.current_stream(dev)
        entry = self._pf_graphs.pop(T, None)
        if entry is None:
            while len(self._pf_graphs) >= self.PREFILL_GRAPHS:
                self._pf_graphs.pop(next(iter(self._pf_graphs)))
            # one eager pass first: the ops' host-side set-up (tensor maps, limits) happens there
            self.reset()
            self.lm_head(self._forward(self._pf_ids[:T], True))
            self.reset()
            self._pf_stream.wait_stream(cur)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self._pf_pool, stream=self._pf_stream, capture_error_mode="thread_local"):
                tok = self.lm_head(self._forward(self._pf_ids[:T], True))
            entry = (g, tok)
        self._pf_graphs[T] = entry
        g, tok = entry
        self._pf_stream.wait_stream(cur)
        with torch.cuda.stream(self._pf_stream):
            g.replay()
        cur.wait_stream(self._pf_stream)
        self._set_length(T)
        return tok

    def _one_sequence(self, what: str) -> None:
        if self.batch > 1:
            raise ValueError(f"{what} runs one sequence; a Generator with batch > 1 uses prefill_batch / "
                             "generate_batch")

    def prefill_batch(self, prompts, want_logits: bool = False):
        """The prompts of a static batch (``batch`` prompts of equal length, ids [B, T]), each run
        as one pass into its own caches (the same kernels as :meth:`prefill`). Returns the B first
        greedy tokens, int32 [B] on the device (and their logits f32 [B, V] of this rank's
        vocabulary rows with want_logits)."""
        B = self.batch
        if B < 2:
            raise ValueError("prefill_batch needs a Generator with batch > 1")
        ids = np.asarray(prompts)
        if ids.ndim != 2 or ids.shape[0] != B or not 1 <= ids.shape[1] <= self.max_prompt:
            raise ValueError(f"prompts must be [{B}, T] ids with 1 <= T <= {self.max_prompt}")
        if ids.min() < 0 or ids.max() >= self.V:
            raise ValueError(f"token ids must be in [0, {self.V})")
        self.reset()
        dev_ids = torch.as_tensor(ids.astype(np.int32)).to(self.device)
        h = torch.empty((B, self.H), dtype=torch.float32, device=self.device)
        for b in range(B):
            h[b].copy_(self._forward(dev_ids[b], True, seq=b)[0])
        toks = torch.empty(B, dtype=torch.int32, device=self.device)
        logits = torch.empty((B, self.lm_head.V), dtype=torch.float32, device=self.device) if want_logits else None
        for r0 in range(0, B, 4):
            n = min(4, B - r0)
            out = self.lm_head(h[r0:r0 + n], want_logits=want_logits)
            t, lg = (out if want_logits else (out, None))
            toks[r0:r0 + n].copy_(t.reshape(-1))
            if want_logits:
                logits[r0:r0 + n].copy_(lg)
        self._set_length(int(ids.shape[1]))
        return (toks, logits) if want_logits else toks

    def generate_batch(self, prompts, max_tokens: int, want_logits: bool = False, graphed: bool = True):
        """Greedy ids of a static batch (``Generator.generate`` at temperature 0 for each of B
        equally long prompts, decoded in lockstep): a list of B lists of ``max_tokens`` ids. Each
        decode step runs the projections and the FFN on the B tokens together (row groups of at
        most 4, one weight pass per group) and the attention of all B sequences in one launch;
        every sequence's arithmetic is that of a one-sequence run. graphed: steps replayed from
        CUDA graphs (no logits); else one pyre_decoder_step call per step, with want_logits the
        logits [max_tokens, B, V] on the device."""
        B = self.batch
        if max_tokens < 1 or max_tokens > self.max_seq + 1:
            raise ValueError("max_tokens out of range")
        if graphed and want_logits:
            raise ValueError("graphed decoding returns no logits")
        out = self.prefill_batch(prompts, want_logits=want_logits)
        first, lg0 = (out if want_logits else (out, None))
        if graphed:
            start = self.length
            hist = self.decode_graphed(first, max_tokens - 1)
            self.check_status()
            return hist[:, start:start + max_tokens].cpu().tolist()
        toks = torch.zeros((max_tokens, B), dtype=torch.int32, device=self.device)
        toks[0].copy_(first)
        logits = None
        if want_logits:
            logits = torch.empty((max_tokens, B, self.lm_head.V), dtype=torch.float32, device=self.device)
            logits[0].copy_(lg0)
        for i in range(1, max_tokens):
            self.step_into(toks[i - 1], toks[i], logits[i] if want_logits else None)
        self.check_status()
        ids = toks.t().cpu().tolist()
        return (ids, logits) if want_logits else ids

    def prefill(self, ids, want_logits: bool = False, stream=None, stepwise: bool = False, graphed: bool = False):
        """Run the prompt (a fresh sequence) and return the first greedy token, int64 [1, 1] on
        the device (and the logits f32 [1, V] of the last prompt position with want_logits).

        By default the prompt is one pass with T = prompt length: for T > 4 the projections and
        the FFN run on the tensor-core GEMM (f16 operands: activations rounded to f16, weights
        dequantized to f16). ``stepwise`` instead feeds the prompt one token at a time through
        the decode step, whose projections and FFN multiply f32 activations with the exact
        dequantized weights (slower; the reference computes every prompt position in f32).
        ``graphed`` replays the one-pass prefill from a CUDA graph captured per prompt length
        (no logits; the returned token tensor is reused by the next graphed prefill)."""
        self._one_sequence("prefill")
        ids = np.asarray(ids).reshape(-1)
        if ids.size < 1 or ids.size > self.max_prompt:
            raise ValueError(f"prompt length {ids.size} outside [1, {self.max_prompt}]")
        if ids.min() < 0 or ids.max() >= self.V:
            raise ValueError(f"token ids must be in [0, {self.V})")
        if graphed:
            if want_logits or stepwise or stream is not None:
                raise ValueError("graphed prefill takes no logits, stepwise or stream")
            return self._prefill_graphed(ids)
        self.reset()
        dev_ids = torch.as_tensor(ids.astype(np.int32)).to(self.device)
        n = 1 if stepwise else int(ids.size)
        h = self._forward(dev_ids[:n], True, stream)
        self.length = n
        if n == ids.size:
            return self.lm_head(h, want_logits=want_logits, stream=stream)
        scratch = torch.empty(1, dtype=torch.int32, device=self.device)
        for i in range(1, int(ids.size) - 1):
            self.step_into(dev_ids[i:i + 1], scratch, stream=stream)
        logits = torch.empty((1, self.lm_head.V), dtype=torch.float32, device=self.device) if want_logits else None
        self.step_into(dev_ids[-1:], scratch, logits[0] if want_logits else None, stream=stream)
        tok = scratch.to(torch.int64).view(1, 1)
        return (tok, logits) if want_logits else tok

    def step(self, token: torch.Tensor, want_logits: bool = False, stream=None):
        """One decode step on the previous greedy token (int [1, 1] on the device), op by op
        from Python (:meth:`step_into` is the same step in one native call)."""
        self._one_sequence("step")
        if self.length == 0:
            raise ValueError("step() needs a prefill() first")
        if self.length + 1 > self.max_seq:
            raise ValueError("sequence longer than max_seq")
        ids = token.reshape(-1)[:1].to(torch.int32)
        h = self._forward(ids, False, stream)
        self.length += 1
        return self.lm_head(h, want_logits=want_logits, stream=stream)

    def step_into(self, token_in: torch.Tensor, token_out: torch.Tensor, logits: torch.Tensor | None = None,
                  stream=None) -> None:
        """One decode step through ``pyre_decoder_step``: reads int32 ``token_in`` [1] and writes
        the greedy token to int32 ``token_out`` [1] (both on the device; may be views of one
        buffer), and the logits f32 [V] when given. Nothing is synchronised."""
        if self.length == 0:
            raise ValueError("step_into() needs a prefill() first")
        if self.length + 1 > self.max_seq:
            raise ValueError("sequence longer than max_seq")
        for t in (token_in, token_out):
            if t.dtype != torch.int32 or not t.is_cuda:
                raise ValueError("tokens must be int32 on the device")
        B = self.batch
        if token_in.numel() < B or token_out.numel() < B:
            raise ValueError(f"token_in and token_out need {B} entries (one per sequence)")
        if logits is not None and (logits.dtype != torch.float32 or logits.numel() != B * self.lm_head.V):
            raise ValueError(f"logits must be f32 with {B} x {self.lm_head.V} elements (this rank's vocabulary rows)")
        self._decode_call(self._desc, D.ptr(token_in), self.length, D.ptr(token_out), D.ptr(logits),
                          D.stream_ptr(stream))
        self._set_length(self.length + 1)

    def _set_length(self, n: int) -> None:
        self.length = n
        for L in self.layers:
            for a in L.attns:
                a.cache.length = n

    def decode_graphed(self, first_token: torch.Tensor, n_steps: int, steps_per_graph: int = 16,
                       bucket: int = 512) -> torch.Tensor:
        """``n_steps`` greedy steps after a prefill as replays of captured CUDA graphs: each
        graph holds ``steps_per_graph`` decode steps whose position is read and advanced on
        the device (``pyre_decoder_step`` with ``pos_dev``), so a replay issues that many
        tokens with one host call. The attention grids of a graph are planned for the first
        position of its ``bucket``-wide position range and the graph is replayed for every
        position in that range (captured graphs are cached on this object). first_token: the
        prefill's greedy token (one per sequence for a batch). Returns the int32 device tensor of
        all tokens by position (entries prompt length .. prompt length + n_steps), [max_seq + 1],
        or [batch, max_seq + 1] for a batch."""
        if self.length == 0:
            raise ValueError("decode_graphed() needs a prefill() first")
        if self.length + n_steps > self.max_seq:
            raise ValueError("sequence longer than max_seq")
        dev = self.device
        B = self.batch
        if not hasattr(self, "_gdesc"):
            self._gpos = torch.zeros(1, dtype=torch.int32, device=dev)
            self._gslot = torch.zeros(B, dtype=torch.int32, device=dev)
            self._ghist = torch.zeros(B * (self.max_seq + 1), dtype=torch.int32, device=dev)
            self._gdesc = DecoderDesc.from_buffer_copy(self._desc)
            self._gdesc.pos_dev = self._gpos.data_ptr()
            self._gdesc.history = self._ghist.data_ptr()
            self._gstream = torch.cuda.Stream(dev)
            self._graphs = {}
        start = self.length
        self._gpos.fill_(start)
        self._gslot.copy_(first_token.reshape(-1)[:B].to(torch.int32))
        hist = self._ghist.view(B, self.max_seq + 1)
        hist[:, start].copy_(self._gslot)
        cur = torch.cuda.current_stream(dev)
        self._gstream.wait_stream(cur)
        pos, left = start, n_steps
        while left > 0:
            plan = pos // bucket * bucket          # every step of the graph has plan <= position
            k = min(left, steps_per_graph, plan + bucket - pos)
            g = self._graphs.get((plan, k))
            if g is None:
                # capture-time host work (grid plans, tensor maps) happens here; nothing runs
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self._gstream, capture_error_mode="thread_local"):
                    for _ in range(k):
                        self._decode_call(self._gdesc, D.ptr(self._gslot), plan, D.ptr(self._gslot), None,
                                          D.stream_ptr(self._gstream))
                self._graphs[(plan, k)] = g
            with torch.cuda.stream(self._gstream):
                g.replay()
            pos += k
            left -= k
        cur.wait_stream(self._gstream)
        self._set_length(pos)
        return self._ghist if B == 1 else hist

    def check_status(self) -> None:
        """Raise if a kernel reported a problem: the embedding gather's status word and the
        status words of every layer's Q8_0 kernels (QKV, O, FFN workspaces), read in one copy,
        and the attention kernels' status (a position outside the cache in a graphed decode
        step, a timed-out wait), which pyre_attn_status reads and clears."""
        torch.cuda.synchronize(self.device)
        att = ctypes.c_int(0)
        with torch.cuda.device(self.device):     # pyre_attn_status reads the current device
            N.call("pyre_attn_status", ctypes.byref(att))
        if att.value != 0:
            raise RuntimeError(f"attention kernel status {att.value}")
        words = [self.status[0]]
        for L in self.layers:
            for ws in (L.qkv.workspace, L.o.workspace, L.ffn.workspace):
                words.append(ws[8:12].view(torch.int32)[0])
        if self._pws is not None:
            words.append(self._pws[8:12].view(torch.int32)[0])
        if self.comm is not None:
            self.comm.check()          # raises PyreTimeout if a wait on a peer ran out
        vals = torch.stack(words).cpu().tolist()
        if self._pws is not None:
            pv = vals.pop()
            if pv != 0:
                raise RuntimeError(f"persistent decode kernel status {pv}")
        if vals[0] != 0:
            raise RuntimeError(f"embedding gather saw a token id outside [0, {self.V})")
        for i, v in enumerate(vals[1:]):
            if v != 0:
                raise RuntimeError(f"layer {i // 3} {('QKV', 'O', 'FFN')[i % 3]} kernel status {v}")

    def generate_ids(self, prompt_ids, max_tokens: int, want_logits: bool = False, native: bool = True,
                     stepwise_prefill: bool = False, graphed: bool = False):
        """Greedy ids after the prompt (``Generator.generate`` at temperature 0 without the
        tokenizer and EOS stop), as a list of ints; with want_logits also the f32 logits of
        every step, [max_tokens, V] on the device. native: decode steps through
        pyre_decoder_step (else op by op from Python); stepwise_prefill: see :meth:`prefill`;
        graphed: decode steps as CUDA-graph replays (:meth:`decode_graphed`, no logits). With
        tensor parallelism the logits are this rank's vocabulary rows (lm_v0 onwards)."""
        self._one_sequence("generate_ids")
        if max_tokens < 1 or max_tokens > self.max_seq + 1:
            raise ValueError("max_tokens out of range")
        if graphed and want_logits:
            raise ValueError("graphed decoding returns no logits")
        out = self.prefill(prompt_ids, want_logits=want_logits, stepwise=stepwise_prefill,
                           graphed=graphed and not stepwise_prefill)
        tok, lg0 = (out if want_logits else (out, None))
        if graphed:
            start = self.length
            hist = self.decode_graphed(tok, max_tokens - 1)
            self.check_status()
            return hist[start:start + max_tokens].cpu().tolist()
        logits = torch.empty((max_tokens, self.lm_head.V), dtype=torch.float32, device=self.device) \
            if want_logits else None
        if want_logits:
            logits[0].copy_(lg0[0])
        toks = self.tokens
        toks[0].copy_(tok.reshape(-1)[0])
        for i in range(1, max_tokens):
            if native:
                self.step_into(toks[i - 1:i], toks[i:i + 1], logits[i] if want_logits else None)
            else:
                out = self.step(toks[i - 1:i], want_logits=want_logits)
                t, lg = (out if want_logits else (out, None))
                toks[i].copy_(t.reshape(-1)[0])
                if want_logits:
                    logits[i].copy_(lg[0])
        self.check_status()
        ids = toks[:max_tokens].cpu().tolist()
        return (ids, logits) if want_logits else ids
