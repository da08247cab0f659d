"""The committed golden fixtures (tests/golden/, made by tests/golden/make_golden.py from the oracle) still hold:
the CPU oracle reproduces every fixture bit for bit. The GPU side is checked in test_gpu_golden.py."""
import os
import sys

import numpy as np
import pytest

from oracle import oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)
import make_golden  # noqa: E402


def load(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.mark.parametrize("name", ["linear_g64_h2048.npz", "linear_g128_h512.npz"])
def test_oracle_linear_fixture(name):
    f = load(name)
    B = f["B"] if "B" in f else None
    signs = f["signs"] if "signs" in f else None
    Y, xr = orc.rotate_ternary_linear(f["W"], f["S"], B, int(f["group"]), f["xb"], int(f["HB"]), signs)
    assert np.array_equal(Y.astype(np.float32), f["Y"])
    assert np.array_equal(xr.astype(np.float32), f["xr"])


def test_oracle_gdn_fixture():
    f = load("gdn_verify.npz")
    q, k, v, a, b, al, dt, S = make_golden.gdn_inputs()
    for n in (0, 5, 9):
        y, st = orc.gdn_verify(q, k, v, a, b, al, dt, S.copy(), n)
        assert np.array_equal(y, f[f"y{n}"])
        assert np.array_equal(st[:, :8, :], f[f"state_rows{n}"])
        assert (st.astype(np.float64) ** 2).sum() == float(f[f"state_ss{n}"])


def test_oracle_tiny_model_fixture():
    from bonsai_b200 import synth
    from bonsai_b200.config import tiny

    f = load("tiny_model.npz")
    cfg = tiny()
    o = orc.OracleModel(cfg, synth.model_tensors(cfg, 7))
    assert np.array_equal(synth.zipf_tokens(21, 40, cfg.vocab).astype(np.uint32), f["prompt"])
    first = o.prefill(f["prompt"])
    assert first == int(f["first"])
    snap = o.snapshot()
    assert np.array_equal(o.greedy(first, 24), f["greedy"])
    o.restore(snap)
    pred, logits = o.forward(f["verify_ids"], logits=True)
    assert np.array_equal(pred, f["verify_pred"])
    assert np.array_equal(logits[f["logit_rows"]], f["logits"])
    o.free_snapshot(snap)
