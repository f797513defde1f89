"""Cross-box wire format: the reference's message framing and Q8_0 activation transfer.

Inside one box the tensor-parallel exchanges go over NVLink (pyre_b200.tp); between boxes the
reference's TCP protocol stays, so a box running this library talks to a reference root or
worker unchanged:

* framing (src/orchestrator/net.py:18-48): a 12-byte big-endian header ``(msg_type,
  payload_len, n_chunks)`` followed by the pickled payload cut into 8 MB chunks;
* message types (src/orchestrator/protocol.py:1-10);
* activations as Q8_0 tuples ``(q int8 [n_blocks, 32], scales f32 [n_blocks], shape)``
  (quantize_activation / dequantize_activation, src/orchestrator/quantizer.py:54-67), here
  quantized and dequantized on the GPU by the library's bit-exact kernels
  (pyre_q80_quantize / pyre_q80_dequantize), so only the 34-36 bytes per 32 values cross
  PCIe and the network.
"""
from __future__ import annotations

import math
import pickle
import socket
import struct
from typing import Any

import numpy as np
import torch

from . import _device as D
from . import _native as N

CHUNK_SIZE = 8 * 1024 * 1024
HEADER = struct.Struct("!III")

MSG_SHARD_SPEC = 0
MSG_READY = 1
MSG_FORWARD_DATA = 2
MSG_FORWARD_RESULT = 3
MSG_SHUTDOWN = 4
MSG_ATTN_OUTPUT = 5
MSG_FFN_RESULT = 6
MSG_ALL_LAYERS_DONE = 8
MSG_DECODE_STEP = 9     # (layer_idx, h_norm): a worker's FFN for one decode token
MSG_DECODE_QKV = 10     # (layer_idx, x_norm, cache_len): a worker's QKV, cache and attention


def encode_msg(msg_type: int, obj: Any = None) -> bytes:
    """Header + payload exactly as the reference's send_msg puts them on the socket."""
    payload = pickle.dumps(obj, protocol=pickle.HIGHEST_PROTOCOL) if obj is not None else b""
    n_chunks = (len(payload) + CHUNK_SIZE - 1) // CHUNK_SIZE
    return HEADER.pack(int(msg_type), len(payload), n_chunks) + payload


def send_msg(conn: socket.socket, msg_type: int, obj: Any = None) -> None:
    data = encode_msg(msg_type, obj)
    view = memoryview(data)
    conn.sendall(view[:HEADER.size])
    for off in range(HEADER.size, len(data), CHUNK_SIZE):
        conn.sendall(view[off:off + CHUNK_SIZE])


def recv_exact(conn: socket.socket, n: int) -> bytes:
    buf = bytearray(n)
    view = memoryview(buf)
    got = 0
    while got < n:
        k = conn.recv_into(view[got:], n - got)
        if k == 0:
            raise ConnectionError("Connection closed")
        got += k
    return bytes(buf)


def recv_msg(conn: socket.socket):
    """(msg_type, obj) of one message framed by send_msg (or the reference's)."""
    msg_type, total, n_chunks = HEADER.unpack(recv_exact(conn, HEADER.size))
    if n_chunks != (total + CHUNK_SIZE - 1) // CHUNK_SIZE:
        raise ValueError(f"bad frame: {total} payload bytes in {n_chunks} chunks")
    payload = recv_exact(conn, total) if total else b""
    return msg_type, (pickle.loads(payload) if payload else None)


def quantize_activation(x) -> tuple:
    """``(q int8 [n_blocks, 32], scales f32 [n_blocks], shape)`` of an activation (any shape,
    f32 or bf16; a CUDA tensor, or host data copied to the current GPU), bit-exact with the
    reference's quantize_activation."""
    t = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x, dtype=np.float32))
    shape = tuple(int(d) for d in t.shape)
    t = D.to_device(t)
    if t.dtype not in (torch.float32, torch.bfloat16):
        t = t.float()
    t = t.contiguous()
    n = t.numel()
    nb = max(1, math.ceil(n / 32))
    q = torch.empty(nb * 32, dtype=torch.int8, device=t.device)
    s = torch.empty(nb, dtype=torch.float32, device=t.device)
    N.call("pyre_q80_quantize", D.ptr(t), D.dtype_code(t), n, D.ptr(q), D.ptr(s), None, D.stream_ptr())
    return q.view(nb, 32).cpu().numpy(), s.cpu().numpy(), shape


def dequantize_activation(data: tuple, device=None) -> torch.Tensor:
    """f32 tensor of the given shape on the GPU from a Q8_0 activation tuple (the reference's
    dequantize_activation, on the device)."""
    q, s, shape = data
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    qt = torch.as_tensor(np.ascontiguousarray(q, dtype=np.int8)).reshape(-1).to(dev)
    st = torch.as_tensor(np.ascontiguousarray(s, dtype=np.float32)).reshape(-1).to(dev)
    n = int(np.prod(shape)) if len(shape) else 1
    if qt.numel() < n or st.numel() * 32 != qt.numel():
        raise ValueError("Q8_0 tuple does not cover the shape")
    out = torch.empty(n, dtype=torch.float32, device=dev)
    N.call("pyre_q80_dequantize", D.ptr(qt), D.ptr(st), N.PYRE_F32, n, D.ptr(out), D.stream_ptr())
    return out.reshape(shape)
