"""Q8_0 quantization on the GPU is bit-exact with the reference (goldens written by the
reference's quantizer.py, plus seeded full-size weights checked against the pinned oracle)."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
import sys, os
sys.path.insert(0, os.path.dirname(__file__))
from oracle import q80 as oq80

pytestmark = pytest.mark.gpu


def _cases():
    z = np.load(GOLDEN / "q80_golden.npz")
    names = sorted({k.split("__")[0] for k in z.files})
    return [(n, z[f"{n}__x"], z[f"{n}__q"], z[f"{n}__s"], tuple(z[f"{n}__shape"])) for n in names]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
def test_quantize_bit_exact_vs_reference_golden(case):
    from pyre_b200.quantizer import quantize_q80
    name, x, q_ref, s_ref, shape = case
    q, s, sh = quantize_q80(torch.from_numpy(x).cuda())
    assert sh == shape
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(_bits(s), s_ref.view(np.uint32))


def test_quantize_bf16_input_path():
    from pyre_b200.quantizer import quantize_q80
    z = np.load(GOLDEN / "q80_golden.npz")
    x = z["weights_bf16_128x64__x"]
    q, s, _ = quantize_q80(torch.from_numpy(x).cuda().to(torch.bfloat16))
    np.testing.assert_array_equal(q.cpu().numpy(), z["weights_bf16_128x64__q"])
    np.testing.assert_array_equal(_bits(s), z["weights_bf16_128x64__s"].view(np.uint32))


@pytest.mark.parametrize("offset", [1, 2, 3])
def test_quantize_unaligned_source(offset):
    from pyre_b200.quantizer import quantize_q80
    rng = np.random.default_rng(offset)
    x = rng.standard_normal(4096 + 77).astype(np.float32)
    dev = torch.from_numpy(x).cuda()
    q, s, _ = quantize_q80(dev[offset:])
    qr, sr, _ = oq80.quantize_q80(x[offset:])
    np.testing.assert_array_equal(q.cpu().numpy(), qr)
    np.testing.assert_array_equal(_bits(s), sr.view(np.uint32))


def test_quantize_full_size_mistral_gate_bit_exact():
    """One Mistral-7B-shape FFN matrix (4096 x 14336, bf16-rounded N(0, 0.02))."""
    from pyre_b200.quantizer import quantize_q80
    g = torch.Generator(device="cuda").manual_seed(1)
    w = (torch.randn((14336, 4096), generator=g, device="cuda") * 0.02).to(torch.bfloat16).t().contiguous()
    q, s, _ = quantize_q80(w)
    qr, sr, _ = oq80.quantize_q80(w.float().cpu().numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), qr)
    np.testing.assert_array_equal(_bits(s), sr.view(np.uint32))


def test_f16_scales_and_dequantize():
    from pyre_b200.quantizer import Q80Weight, dequantize_q80, quantize_q80
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((96, 256)) * 0.02).astype(np.float32)
    w16 = Q80Weight.from_float(torch.from_numpy(x).cuda(), torch.float16)
    w32 = Q80Weight.from_float(torch.from_numpy(x).cuda(), torch.float32)
    assert torch.equal(w16.q, w32.q)
    assert torch.equal(w16.scale, w32.scale.to(torch.float16))
    qr, sr, _ = oq80.quantize_q80(x)
    np.testing.assert_array_equal(w32.dequantize().cpu().numpy(), oq80.dequantize_q80(qr, sr, x.shape))
    q, s, sh = quantize_q80(torch.from_numpy(x).cuda())
    np.testing.assert_array_equal(dequantize_q80(q, s, sh).cpu().numpy(), oq80.dequantize_q80(qr, sr, x.shape))


def test_shard_slices_equal_slice_quantization():
    """Quantizing the full [H, I] matrix then slicing equals quantizing the slice (block
    edges are multiples of 32), which is what lets every rank hold the reference's bits."""
    from pyre_b200.quantizer import Q80Weight
    rng = np.random.default_rng(6)
    x = (rng.standard_normal((64, 384)) * 0.02).astype(np.float32)
    full = Q80Weight.from_float(torch.from_numpy(x).cuda(), torch.float32)
    for s, e in [(0, 96), (96, 256), (256, 384)]:
        part = Q80Weight.from_float(torch.from_numpy(np.ascontiguousarray(x[:, s:e])).cuda(), torch.float32)
        c = full.cols(s, e)
        assert torch.equal(c.q, part.q) and torch.equal(c.scale, part.scale)
    xt = np.ascontiguousarray(x.T)
    fullr = Q80Weight.from_float(torch.from_numpy(xt).cuda(), torch.float32)
    r = fullr.rows(96, 256)
    pr = Q80Weight.from_float(torch.from_numpy(np.ascontiguousarray(xt[96:256])).cuda(), torch.float32)
    assert torch.equal(r.q, pr.q) and torch.equal(r.scale, pr.scale)


def test_weights_dict_roundtrip_tags():
    from pyre_b200.quantizer import MIN_QUANTIZE_ELEMS, dequantize_weights_dict, quantize_weights_dict
    rng = np.random.default_rng(8)
    d = {"ffn": {"gate": rng.standard_normal((64, 128)).astype(np.float32)},
         "norm": rng.standard_normal(64).astype(np.float32)}
    qd = quantize_weights_dict(d)
    assert qd["ffn"]["gate"][0] == "q8" and qd["norm"] is d["norm"]
    assert d["norm"].size < MIN_QUANTIZE_ELEMS
    rd = dequantize_weights_dict(qd)
    q, s, sh = oq80.quantize_q80(d["ffn"]["gate"])
    np.testing.assert_array_equal(rd["ffn"]["gate"].cpu().numpy(), oq80.dequantize_q80(q, s, sh))


def test_q80weight_tuple_roundtrip_is_reference_bits():
    from pyre_b200.quantizer import Q80Weight
    z = np.load(GOLDEN / "q80_golden.npz")
    x, q, s = z["normal_64x96__x"], z["normal_64x96__q"], z["normal_64x96__s"]
    w = Q80Weight.from_tuple(("q8", q, s, x.shape), scale_dtype=torch.float32)
    _, q2, s2, sh = w.to_tuple()
    assert sh == x.shape
    np.testing.assert_array_equal(q2.cpu().numpy(), q)
    np.testing.assert_array_equal(s2.cpu().numpy().view(np.uint32), s.view(np.uint32))


@pytest.mark.parametrize("M,K,N", [(1, 64, 256), (1, 100, 800), (2, 96, 512), (2, 40, 352), (1, 4096, 1344)])
@pytest.mark.parametrize("scale_dtype", [torch.float16, torch.float32])
def test_pack_kernel_matches_layout(M, K, N, scale_dtype):
    from test_layout import pack_reference
    from pyre_b200.quantizer import Q80Packed, Q80Weight
    g = torch.Generator().manual_seed(K + N + M)
    ws = [Q80Weight(torch.randint(-128, 128, (K, N), generator=g, dtype=torch.int8).cuda(),
                    torch.rand((K, N // 32), generator=g).to(scale_dtype).cuda()) for _ in range(M)]
    packed = Q80Packed.pack(ws)
    es = np.float16 if scale_dtype == torch.float16 else np.float32
    ref = pack_reference([w.q.cpu().numpy() for w in ws], [w.scale.cpu().numpy() for w in ws], es)
    np.testing.assert_array_equal(packed.data.cpu().numpy(), ref)
