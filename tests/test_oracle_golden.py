"""The oracle is pinned to the reference: its Q8_0 bits, FFN partials and partitioner
outputs must equal the fixtures the reference's own code wrote (tests/golden/)."""
import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import cref, ffn as offn, q80 as oq80


def _q80_cases():
    z = np.load(GOLDEN / "q80_golden.npz")
    names = sorted({k.split("__")[0] for k in z.files})
    return [(n, z[f"{n}__x"], z[f"{n}__q"], z[f"{n}__s"], tuple(z[f"{n}__shape"])) for n in names]


@pytest.mark.parametrize("case", _q80_cases(), ids=lambda c: c[0])
def test_oracle_q80_bit_exact_vs_reference(case):
    name, x, q_ref, s_ref, shape = case
    with np.errstate(all="ignore"):
        q, s, sh = oq80.quantize_q80(x)
    assert sh == shape
    np.testing.assert_array_equal(q, q_ref)
    np.testing.assert_array_equal(s.view(np.uint32), s_ref.view(np.uint32))


@pytest.mark.parametrize("case", _q80_cases(), ids=lambda c: c[0])
def test_oracle_c_q80_bit_exact_vs_reference(case, oracle_lib):
    name, x, q_ref, s_ref, shape = case
    q, s = cref.q80_quantize(x)
    np.testing.assert_array_equal(q, q_ref)
    np.testing.assert_array_equal(s.view(np.uint32), s_ref.view(np.uint32))


def test_oracle_dequantize_roundtrip_matches_reference_formula():
    for name, x, q_ref, s_ref, shape in _q80_cases():
        d = oq80.dequantize_q80(q_ref, s_ref, shape)
        manual = (q_ref.astype(np.float32) * s_ref[:, None]).ravel()[: int(np.prod(shape))].reshape(shape)
        np.testing.assert_array_equal(d, manual)


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_oracle_ffn_ungated_vs_reference_builder():
    """tests/test_ffn_builder.py:16-51 of the reference, run through its own builder."""
    z = np.load(GOLDEN / "ffn_golden.npz")
    rng = np.random.default_rng(42)
    x = rng.standard_normal((1, 4, 768)).astype(np.float32)
    up = rng.standard_normal((768, 3072)).astype(np.float32)
    down = rng.standard_normal((3072, 768)).astype(np.float32)
    assert _sha(x) == str(z["ungated__x_sha"]) and _sha(up) == str(z["ungated__up_sha"])
    assert _sha(down) == str(z["ungated__down_sha"])
    for i, (s, e) in enumerate([(0, 1024), (1024, 2048), (2048, 3072)]):
        with np.errstate(over="ignore"):
            p = offn.ffn_shard(x, None, up[:, s:e], down[s:e])
        np.testing.assert_allclose(p, z["ungated__partials"][i], rtol=1e-5, atol=1e-2)


def test_oracle_ffn_gated_q80_vs_reference_builder():
    z = np.load(GOLDEN / "ffn_golden.npz")
    H, I = 256, 384
    w = {}
    for name, shp in (("gate", (H, I)), ("up", (H, I)), ("down", (I, H))):
        w[name] = oq80.dequantize_q80(z[f"gated__{name}_q"], z[f"gated__{name}_s"], shp)
    x = z["gated__x"]
    for i, (s, e) in enumerate(z["gated__bounds"]):
        p = offn.ffn_shard(x, w["gate"][:, s:e], w["up"][:, s:e], w["down"][s:e])
        np.testing.assert_allclose(p, z["gated__partials"][i], rtol=1e-5, atol=1e-6)


def test_oracle_c_matmul_matches_numpy():
    rng = np.random.default_rng(3)
    a = rng.standard_normal((3, 70)).astype(np.float32)
    b = rng.standard_normal((70, 45)).astype(np.float32)
    np.testing.assert_allclose(cref.matmul_f32(a, b), a @ b, rtol=1e-5, atol=1e-4)


def test_oracle_c_root_decode_ffn_matches_graph():
    rng = np.random.default_rng(4)
    H, W = 64, 96
    x = rng.standard_normal(H).astype(np.float32)
    g, u = (rng.standard_normal((H, W)).astype(np.float32) * 0.1 for _ in range(2))
    d = rng.standard_normal((W, H)).astype(np.float32) * 0.1
    full = cref.root_decode_ffn(x, g, u, d, 0, W)
    np.testing.assert_allclose(full, offn.ffn_shard(x[None], g, u, d)[0], rtol=1e-4, atol=1e-5)
    halves = cref.root_decode_ffn(x, g, u, d, 0, 40) + cref.root_decode_ffn(x, g, u, d, 40, W)
    np.testing.assert_allclose(halves, full, rtol=1e-5, atol=1e-5)
