"""The oracle restatement against the committed golden fixtures made by the
reference engine's own C attention (tests/golden/make_golden.py): int8 KV
caches and saved-prefix image byte-identical, outputs within 1e-5. Runs
without the reference sources."""
import hashlib
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as G  # noqa: E402
import ndoracle as O  # noqa: E402


@pytest.mark.parametrize("name", sorted(G.CASES))
def test_oracle_reproduces_golden(name):
    gold = np.load(os.path.join(HERE, "golden", name + ".npz"))
    s, out, img = G.run(O.OracleSeq, G.CASES[name])
    assert hashlib.sha256(s.k.tobytes()).hexdigest() == str(gold["k_sha"])
    assert hashlib.sha256(s.v.tobytes()).hexdigest() == str(gold["v_sha"])
    assert np.array_equal(s.ks, gold["ks"]) and np.array_equal(s.vs, gold["vs"])
    assert hashlib.sha256(img).hexdigest() == str(gold["prefix_sha"])
    ref = gold["out"].astype(np.float64)
    assert out.shape == ref.shape
    assert np.max(np.abs(out - ref) / np.maximum(1.0, np.abs(ref))) <= 1e-5
