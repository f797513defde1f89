"""The lm_head oracle (oracle/lmhead.py) against the reference's own Generator methods
(tests/golden/lmhead_golden.npz, written by tests/golden/make_golden.py)."""
import numpy as np

from conftest import GOLDEN
from oracle import lmhead as OL


def test_oracle_equals_reference_generator():
    z = np.load(GOLDEN / "lmhead_golden.npz")
    for name in ("small", "rows"):
        h, w, E = z[f"{name}__h"], z[f"{name}__w"], z[f"{name}__E"]
        logits = OL.compute_logits(h, E, w.astype(np.float32))
        assert np.array_equal(logits, z[f"{name}__logits"]), name
        assert np.array_equal(OL.greedy_token(logits), z[f"{name}__token"]), name


def test_tied_maxima_take_the_first_index():
    z = np.load(GOLDEN / "lmhead_golden.npz")
    logits = z["rows__logits"]
    assert logits[1, 7] == logits[1, 200] == logits[1, 301] == logits[1].max()
    assert int(z["rows__token"][1, 0]) == 7
