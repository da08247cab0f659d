"""The tcgen05 prefill GEMM (bcu_linear_gemm: tensor-memory accumulators, bulk-copy staging, weights decoded to fp16
in shared memory) against the oracle's ternary linear and a float64 restatement.

Tolerance (as the verify GEMV, whose arithmetic it shares): |y - y_ref| <= 2e-5 * sum_k |w_k x_k| + 1e-5 per output
(fp16 hi + lo activations with a per-token power-of-two scale, exact products for ternary codes, fp32 sums)."""
import ctypes

import numpy as np
import pytest

import refimpl
from bonsai_b200 import _lib
from oracle import oracle as orc
from test_oracle import ternary_case

pytestmark = pytest.mark.gpu


class Gemm:
    def __init__(self, W, S, B, group):
        self.L = _lib.lib()
        self.h = ctypes.c_void_p()
        O, K = W.shape[0], W.shape[1] * 16
        s = self.L.bcu_linear_prepare(orc.ptr(W), orc.ptr(S), orc.ptr(B) if B is not None else None, O, K, group, 0,
                                      ctypes.byref(self.h))
        assert s == _lib.OK
        self.O = O

    def __call__(self, torch, X):
        x = torch.from_numpy(np.ascontiguousarray(X, np.float32)).cuda()
        y = torch.full((X.shape[0], self.O), float("nan"), dtype=torch.float32, device="cuda")
        assert self.L.bcu_linear_gemm(self.h, ctypes.c_void_p(x.data_ptr()), X.shape[0],
                                      ctypes.c_void_p(y.data_ptr()), None) == _lib.OK
        assert self.L.bcu_linear_sync(self.h, None) == _lib.OK
        return y.cpu().numpy()

    def __del__(self):
        self.L.bcu_linear_free(self.h)


def check(y, X, W, S, B, group, want=None):
    Wd = refimpl.dense_weights(W, S, B, group).astype(np.float64)
    Xd = X.astype(np.float64)
    if want is None:
        want = Xd @ Wd.T
    bound = 2e-5 * (np.abs(Xd) @ np.abs(Wd).T) + 1e-5
    err = np.abs(y.astype(np.float64) - want)
    assert np.all(np.isfinite(y)), "non-finite outputs"
    assert np.all(err <= bound), f"max err {err.max()} (worst ratio {(err / bound).max():.3f})"


@pytest.mark.parametrize("O,K,M,group,bias", [
    (256, 512, 1, 64, "neg"),          # one token, one bias chunk
    (384, 1024, 300, 64, "free"),      # free fp16 bias, 3 token tiles (the last partial)
    (128, 2048, 129, 128, None),       # reference pack: group 128, implicit bias -s
    (256, 6144, 257, 64, "free"),      # 96 groups: two bias chunks
])
def test_gemm_matches_oracle(gpu, O, K, M, group, bias):
    torch = pytest.importorskip("torch")
    W, S, B, X = ternary_case(O, K, group, M, bias, 7 + M)
    y = Gemm(W, S, B, group)(torch, X)
    check(y, X, W, S, B, group, want=orc.ternary_linear(W, S, B, group, X).astype(np.float64))
    check(y, X, W, S, B, group)


def test_gemm_many_tiles_per_cta(gpu):
    """More tiles than SMs (each CTA loops over several, reusing its tensor memory), and inputs with a wide dynamic
    range per token (the per-token exponent)."""
    torch = pytest.importorskip("torch")
    O, K, M = 2048, 2048, 2100
    W, S, B, X = ternary_case(O, K, 64, M, "neg", 3)
    X *= np.exp2(np.random.default_rng(4).integers(-20, 20, (M, 1))).astype(np.float32)
    X[5] = 0.0
    y = Gemm(W, S, B, 64)(torch, X)
    check(y, X, W, S, B, 64)
    assert np.all(y[5] == 0.0)


def test_gemm_rows_do_not_depend_on_batch(gpu):
    """A token's outputs are the same bits whatever the other tokens of the call and its column in the tile."""
    torch = pytest.importorskip("torch")
    O, K, M = 512, 2048, 400
    W, S, B, X = ternary_case(O, K, 64, M, "free", 11)
    g = Gemm(W, S, B, 64)
    full = g(torch, X)
    part = g(torch, X[37:250])
    assert np.array_equal(full[37:250].view(np.uint32), part.view(np.uint32))


def test_activation_tiles_layout(gpu):
    """gemm_prep_kernel's output byte for byte against a restatement of the layout: per token tile and chunk of 64
    inputs, 256 rows of 8 pieces of 8 fp16 (piece j of row r at position j ^ (r % 8)), rows 0..127 the hi parts and
    128..255 the lo parts of
    x 2^E, E = clamp(14 - frexp exponent of max |x|), inputs in the weight decode's order, then the bias chunks of
    group sums x 2^(E - 6)."""
    torch = pytest.importorskip("torch")
    O, K, M, G = 128, 512, 130, 64
    W, S, B, X = ternary_case(O, K, G, M, "neg", 5)
    X[3] *= 1e-3
    g = Gemm(W, S, B, G)
    nmain, nbias, nt = K // 64, 1, (M + 127) // 128
    nch = nmain + nbias
    bop = torch.zeros(nt * nch * 32768, dtype=torch.uint8, device="cuda")
    ex = torch.zeros(M, dtype=torch.int32, device="cuda")
    x = torch.from_numpy(X).cuda()
    assert g.L.bcu_gemm_prep_debug(g.h, ctypes.c_void_p(x.data_ptr()), M, ctypes.c_void_p(bop.data_ptr()),
                                   ctypes.c_void_p(ex.data_ptr())) == _lib.OK
    # tiles of 256 rows x 8 pieces of 8 fp16, piece j of row r stored at position j ^ (r % 8) (128-byte swizzle)
    raw = bop.cpu().numpy().view(np.uint16).reshape(nt, nch, 256, 8, 8)
    sw = np.array([[j ^ (r % 8) for j in range(8)] for r in range(256)])
    got = np.take_along_axis(raw, sw[None, None, :, :, None].repeat(8, -1).astype(np.int64), axis=3)
    got = got.transpose(0, 1, 3, 2, 4).reshape(nt, nch, 8, 32, 8, 8)  # [tt][chunk][piece][row group][row][half]
    E = np.array([min(max(14 - np.frexp(np.abs(r).max())[1], -60), 100) for r in X])
    assert np.array_equal(ex.cpu().numpy(), E)
    want = np.zeros_like(got)
    # half p of k-row kk of a chunk holds input 16 (kk / 2) + 4 (kk % 2) + p / 2 + 8 (p % 2) (the decode's order)
    order = np.array([16 * (kk // 2) + 4 * (kk % 2) + p // 2 + 8 * (p % 2) for kk in range(8) for p in range(8)])
    for t in range(M):
        tt, tl = divmod(t, 128)
        v = X[t].astype(np.float32) * np.float32(2.0 ** E[t])
        hi = v.astype(np.float16)
        lo = (v - hi.astype(np.float32)).astype(np.float16)
        # each lane sums its 16 inputs in order, then the group's 4 lanes are summed as a butterfly tree
        ls = np.cumsum(X[t].reshape(-1, 16), axis=1, dtype=np.float32)[:, -1].reshape(-1, 4)
        gs = ((ls[:, 0] + ls[:, 1]) + (ls[:, 2] + ls[:, 3])) * np.float32(2.0 ** (E[t] - 6))
        ghi = gs.astype(np.float16)
        glo = (gs - ghi.astype(np.float32)).astype(np.float16)
        for c in range(nmain):
            ks = 64 * c + order
            want[tt, c, :, tl // 8, tl % 8, :] = hi[ks].reshape(8, 8).view(np.uint16)
            want[tt, c, :, (128 + tl) // 8, tl % 8, :] = lo[ks].reshape(8, 8).view(np.uint16)
        ng = K // G
        for gi in range(ng):
            want[tt, nmain, gi // 8, tl // 8, tl % 8, gi % 8] = ghi[gi].view(np.uint16)
            want[tt, nmain, gi // 8, (128 + tl) // 8, tl % 8, gi % 8] = glo[gi].view(np.uint16)
    rows = [t % 128 for t in range(M)]
    for tt in range(nt):
        valid = [r for t, r in enumerate(rows) if t // 128 == tt]
        for r in valid:
            for half in (r // 8, (128 + r) // 8):
                np.testing.assert_array_equal(got[tt, :, :, half, r % 8, :], want[tt, :, :, half, r % 8, :])
