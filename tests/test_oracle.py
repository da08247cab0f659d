"""The CPU oracle against independent known answers (CPU only). The reference itself cannot run here (Rust + Metal /
Vulkan), so these checks are what pins the oracle: IEEE conversions against numpy/torch, the transform against the
Sylvester matrix, the ternary linear and the gated delta rule against float64 restatements, and the oracle model's
own consistency (a verify of T rows then accept(n) equals n single steps)."""
import numpy as np
import pytest

import refimpl
from oracle import oracle as orc


def test_f16_roundtrip_all_patterns():
    L = orc.lib()
    bits = np.arange(65536, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([L.orc_f16_to_f32(int(b)) for b in bits[::7]], np.float32)
    w = want[::7]
    nan = np.isnan(w)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), w[~nan].view(np.uint32))


def test_f32_to_f16_rne_matches_numpy():
    L = orc.lib()
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(3000).astype(np.float32) * s for s in (1e-7, 1e-4, 1, 300, 7e4)])
    want = xs.astype(np.float16).view(np.uint16)
    got = np.array([L.orc_f32_to_f16(float(x)) for x in xs], np.uint16)
    assert np.array_equal(got, want)


def test_bf16_rne_matches_torch():
    torch = pytest.importorskip("torch")
    L = orc.lib()
    xs = np.random.default_rng(1).standard_normal(5000).astype(np.float32) * 3
    want = torch.from_numpy(xs).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = np.array([L.orc_f32_to_bf16(float(x)) for x in xs], np.uint16)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("n", [512, 2048])
def test_fwht_is_sylvester_hadamard(n):
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
    y = x.copy()
    orc.lib().orc_fwht(orc.ptr(y), n)
    want = refimpl.hadamard_rotate(x, n) * np.sqrt(n)
    np.testing.assert_allclose(y, want, rtol=1e-4, atol=1e-4 * np.abs(x).sum() / np.sqrt(n))
    # exact on integers: add/sub only
    xi = np.random.default_rng(2).integers(-100, 100, n).astype(np.float32)
    yi = xi.copy()
    orc.lib().orc_fwht(orc.ptr(yi), n)
    assert np.array_equal(yi, (refimpl.hadamard_rotate(xi, n) * np.sqrt(n)).round().astype(np.float32))


@pytest.mark.parametrize("HB,signed", [(512, True), (2048, False)])
def test_rotate_is_orthonormal(HB, signed):
    x = np.random.default_rng(3).standard_normal(4096).astype(np.float32)
    s = np.where(np.random.default_rng(4).random(4096) < 0.5, -1, 1).astype(np.float32) if signed else None
    y = orc.rotate(x, HB, s)
    np.testing.assert_allclose(y, refimpl.hadamard_rotate(x, HB, s), rtol=1e-5, atol=1e-5)
    assert abs(np.linalg.norm(y) / np.linalg.norm(x) - 1) < 1e-5


def ternary_case(O, K, group, T, bias, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 3, (O, K)).astype(np.uint32)
    W = np.zeros((O, K // 16), np.uint32)
    for e in range(16):
        W |= codes[:, e::16] << (2 * e)
    S = rng.uniform(0.01, 0.05, (O, K // group)).astype(np.float16).view(np.uint16)
    B = (S ^ 0x8000).astype(np.uint16) if bias == "neg" else (
        rng.uniform(-0.05, 0.05, (O, K // group)).astype(np.float16).view(np.uint16) if bias == "free" else None)
    X = rng.standard_normal((T, K)).astype(np.float32)
    return W, S, B, X


@pytest.mark.parametrize("group,bias", [(64, "neg"), (64, "free"), (128, None)])
def test_ternary_linear_vs_float64(group, bias):
    W, S, B, X = ternary_case(256, 2048, group, 9, bias, group)
    Y = orc.ternary_linear(W, S, B, group, X)
    Wd = refimpl.dense_weights(W, S, B, group)
    want = X.astype(np.float64) @ Wd.T
    scale = np.abs(X).astype(np.float64) @ np.abs(Wd).T
    assert np.all(np.abs(Y - want) <= 1e-5 * scale + 1e-6)


def test_ternary_decode_bit_exact():
    # codes the oracle reads back are exactly the ones packed
    W, S, B, X = ternary_case(16, 512, 64, 1, None, 7)
    c = refimpl.decode_codes(W)
    onehot = np.eye(512, dtype=np.float32)[:16]
    # x = e_k picks weight (row, k): (c - 1) * s with the implicit bias
    Y = orc.ternary_linear(W, S, None, 64, onehot)
    want = (c[:, :16] - 1) * np.repeat(refimpl.f16(S), 64, axis=1)[:, :16]
    assert np.array_equal(Y.T.astype(np.float64), want)


def gdn_case(T, NK, NV, seed):
    rng = np.random.default_rng(seed)

    def l2(x):
        return x / np.linalg.norm(x, axis=-1, keepdims=True)

    q = l2(rng.standard_normal((T, NK, 128))).astype(np.float32)
    k = l2(rng.standard_normal((T, NK, 128))).astype(np.float32)
    v = rng.standard_normal((T, NV, 128)).astype(np.float32)
    a = rng.standard_normal((T, NV)).astype(np.float32)
    b = rng.standard_normal((T, NV)).astype(np.float32)
    S = (rng.standard_normal((NV, 128, 128)) * 0.02).astype(np.float32)
    return q, k, v, a, b, np.zeros(NV, np.float32), np.zeros(NV, np.float32), S


@pytest.mark.parametrize("n", [0, 1, 4, 9])
def test_gdn_verify_vs_float64(n):
    case = gdn_case(9, 2, 4, 11)
    y, st = orc.gdn_verify(*case, n)
    y64, st64 = refimpl.gdn_verify(*case, n)
    np.testing.assert_allclose(y, y64, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(st, st64, rtol=1e-4, atol=1e-6)


def test_accept_len_and_argmax_ties():
    L = orc.lib()
    ids = np.array([5, 1, 2, 3, 4], np.uint32)
    for pred, m in (([1, 2, 3, 4, 9], 4), ([1, 2, 7, 4, 9], 2), ([9, 2, 3, 4, 9], 0)):
        p = np.array(pred, np.uint32)
        assert L.orc_accept_len(orc.u32p(ids), orc.u32p(p), 5) == m
    x = np.array([1, 3, 3, -np.inf, np.nan, 3], np.float32)
    assert L.orc_argmax(x.ctypes.data_as(orc.PF), 6) == 1
    x = np.full(5, -np.inf, np.float32)
    assert L.orc_argmax(x.ctypes.data_as(orc.PF), 5) == 0


def test_token_key_rules():
    k = orc.token_key
    assert k(b" Sam") == k(b"sam") == k(b"SAM")
    assert k(b" Sam") & 1 == 1
    assert k(b",") == 0 and k(b" .") == 0
    assert k(b"\n") == 2 and k(b"\n\n") == 2
    assert k(b"hi\n") & 3 == 3
    assert k(b"a") != k(b"b")


def test_lookup_follows_source():
    keys = np.array([orc.token_key(b" w%d" % i) for i in range(100)], np.uint64)
    src = np.array([1, 2, 3, 4, 5, 6, 7, 8, 9, 10], np.uint32)
    d, pos = orc.lookup(src, [50, 2, 3], keys, 3, 1, 4, 100, 0)
    assert list(d) == [4, 5, 6, 7] and pos == 3
    d, pos = orc.lookup(src, [3, 4, 99], keys, 3, 1, 4, 100, 0)  # unknown last word: no draft
    assert len(d) == 0
    d, pos = orc.lookup(src, [8], keys, 3, 1, 8, 3, 0)  # limit caps the draft
    assert list(d) == [9, 10]


def test_policy_prefers_long_drafts_when_cheap():
    L = orc.lib()
    flat = (np.ones(9)).astype(np.float64)
    cost_p = flat.ctypes.data_as(__import__("ctypes").POINTER(__import__("ctypes").c_double))
    assert L.orc_policy_choose(0.0, 0.0, cost_p, 7, 7, 1.05, None) == 7
    steep = np.arange(1, 10).astype(np.float64) * 2
    assert L.orc_policy_choose(0.0, 10.0, steep.ctypes.data_as(cost_p.__class__), 7, 7, 1.05, None) == 0
