"""The CUDA path through the C ABI against the committed golden fixtures (tests/golden/), at the tolerances of the
other GPU parity tests: ternary linear |dy| <= 2e-5 * sum_k |w_k x_k| + 1e-5; gated delta rule 2e-4 relative /
2e-6 absolute; whole-model logits within 2e-3 absolute, predictions, accept length and the greedy continuation
exact."""
import ctypes
import os
import sys

import numpy as np
import pytest

import refimpl
from bonsai_b200 import _lib

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)
import make_golden  # noqa: E402


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def vp(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


@pytest.mark.parametrize("name", ["linear_g64_h2048.npz", "linear_g128_h512.npz"])
def test_linear_matches_fixture(gpu, name):
    torch = pytest.importorskip("torch")
    f = load(name)
    W, S, group, HB = f["W"], f["S"], int(f["group"]), int(f["HB"])
    B = f["B"] if "B" in f else None
    signs = f["signs"] if "signs" in f else None
    O, K = W.shape[0], W.shape[1] * 16
    L = _lib.lib()
    h = ctypes.c_void_p()
    assert L.bcu_linear_prepare(W.ctypes.data, S.ctypes.data, B.ctypes.data if B is not None else None, O, K, group,
                                0, ctypes.byref(h)) == _lib.OK
    try:
        x = torch.from_numpy(f["xb"].view(np.int16)).cuda()
        sg = torch.from_numpy(signs).cuda() if signs is not None else None
        y = torch.empty((x.shape[0], O), dtype=torch.float32, device="cuda")
        assert L.bcu_linear_rotate_forward(h, vp(x), x.shape[0], HB, vp(sg), vp(y), None) == _lib.OK
        torch.cuda.synchronize()
        Wd = refimpl.dense_weights(W, S, B, group)
        bound = 2e-5 * (np.abs(f["xr"]).astype(np.float64) @ np.abs(Wd).T) + 1e-5
        err = np.abs(y.cpu().numpy().astype(np.float64) - f["Y"])
        assert np.all(err <= bound), f"max err {err.max()}"
    finally:
        L.bcu_linear_free(h)


def test_gdn_verify_matches_fixture(gpu):
    torch = pytest.importorskip("torch")
    f = load("gdn_verify.npz")
    q, k, v, a, b, al, dt, S = make_golden.gdn_inputs()
    T, NK, NV = q.shape[0], q.shape[1], v.shape[1]
    L = _lib.lib()
    dev = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (q, k, v, a, b, al, dt)]
    for n in (0, 5, 9):
        st = torch.from_numpy(S.copy()).cuda()
        y = torch.empty((T, NV, 128), dtype=torch.float32, device="cuda")
        assert L.bcu_gdn_verify(*[vp(x) for x in dev], vp(st), vp(y), T, NK, NV, n, None) == _lib.OK
        torch.cuda.synchronize()
        np.testing.assert_allclose(y.cpu().numpy(), f[f"y{n}"], rtol=2e-4, atol=2e-6)
        np.testing.assert_allclose(st.cpu().numpy()[:, :8, :], f[f"state_rows{n}"], rtol=2e-4, atol=2e-6)


def test_tiny_model_matches_fixture(gpu):
    from bonsai_b200 import synth
    from bonsai_b200.config import tiny
    from bonsai_b200.runtime import Model

    f = load("tiny_model.npz")
    cfg = tiny()
    m = Model(cfg).load(synth.model_tensors(cfg, 7))
    try:
        first = m.prefill(f["prompt"])
        assert first == int(f["first"])
        snap = m.snapshot()
        out, _ = m.decode(first, speculate=False, max_tokens=24)
        assert np.array_equal(np.asarray(out, np.uint32), f["greedy"])
        m.restore(snap)
        m.keep_logits(True)
        pred, acc = m.verify(f["verify_ids"])
        assert np.array_equal(np.asarray(pred, np.uint32), f["verify_pred"])
        assert acc == int(f["accept"])
        for i, r in enumerate(f["logit_rows"]):
            err = np.abs(m.logits(int(r)) - f["logits"][i]).max()
            assert err <= 2e-3, f"row {r}: max logit error {err}"
        snap.free()
    finally:
        m.close()
