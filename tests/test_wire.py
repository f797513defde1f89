"""Cross-box wire format against the reference's own bytes (tests/golden/wire_golden.npz, written
by src/orchestrator/net.py send_msg through a socketpair): the same frames byte for byte, frames
read back through a socket, and (GPU) Q8_0 activation tuples bit-exact with the reference's
quantize_activation."""
import socket
import threading

import numpy as np
import pytest

from conftest import GOLDEN

G = np.load(GOLDEN / "wire_golden.npz")


def _ref_tuple(i):
    return (G[f"q{i}"], G[f"s{i}"], tuple(int(d) for d in G[f"shape{i}"]))


def _messages():
    return [(2, (3, _ref_tuple(0))), (10, (5, _ref_tuple(1), 2175)), (6, G["ffn"])]


def test_frames_equal_reference_bytes():
    from pyre_b200 import wire
    for i, (mtype, obj) in enumerate(_messages()):
        assert wire.encode_msg(mtype, obj) == G[f"msg{i}"].tobytes(), i


def test_empty_message_header():
    from pyre_b200 import wire
    assert wire.encode_msg(wire.MSG_READY) == wire.HEADER.pack(1, 0, 0)


def test_recv_reads_reference_frames_and_chunks():
    """Frames of the reference and a payload larger than one 8 MB chunk, through a socket."""
    from pyre_b200 import wire
    big = np.arange(3 * 1024 * 1024, dtype=np.float32)          # 12 MB payload: 2 chunks
    stream = b"".join(G[f"msg{i}"].tobytes() for i in range(3))
    a, b = socket.socketpair()

    def send():
        a.sendall(stream)
        wire.send_msg(a, wire.MSG_FFN_RESULT, big)
    t = threading.Thread(target=send)
    t.start()
    got = [wire.recv_msg(b) for _ in range(4)]
    t.join()
    a.close()
    b.close()
    (t0, (l0, (q0, s0, sh0))), (t1, (l1, (q1, s1, sh1), c1)), (t2, f), (t3, bg) = got
    assert (t0, l0, t1, l1, c1, t2, t3) == (2, 3, 10, 5, 2175, 6, 6)
    assert np.array_equal(q0, G["q0"]) and np.array_equal(s0, G["s0"]) and sh0 == tuple(G["shape0"])
    assert np.array_equal(q1, G["q1"]) and sh1 == tuple(G["shape1"])
    assert np.array_equal(f, G["ffn"]) and np.array_equal(bg, big)


@pytest.mark.gpu
def test_activation_tuples_bit_exact_on_device():
    import torch
    from pyre_b200 import wire
    for i, key in ((0, "x"), (1, "x1")):
        q, s, shape = wire.quantize_activation(torch.from_numpy(G[key]).cuda())
        assert np.array_equal(q, G[f"q{i}"]) and q.dtype == np.int8 and q.shape == G[f"q{i}"].shape
        assert np.array_equal(s.view(np.uint32), G[f"s{i}"].view(np.uint32)) and s.dtype == np.float32
        assert shape == tuple(int(d) for d in G[f"shape{i}"])
        back = wire.dequantize_activation((q, s, shape)).cpu().numpy()
        flat = (q.reshape(-1).astype(np.float32) * np.repeat(s, 32))[:int(np.prod(shape))].reshape(shape)
        assert np.array_equal(back, flat)
    # the whole frame of a root's forward message, built from a device activation
    frame = wire.encode_msg(wire.MSG_FORWARD_DATA, (3, wire.quantize_activation(torch.from_numpy(G["x"]).cuda())))
    assert frame == G["msg0"].tobytes()
