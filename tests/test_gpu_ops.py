"""GPU parity of the standalone hot ops through the C ABI against the oracle.

Tolerances (stated per north star): the ternary linear is fp32-accurate — |y_gpu - y_oracle| <= 2e-5 * sum_k |w_k x_k|
+ 1e-5 (the fp16 hi/lo activation split keeps ~22 bits, products are exact, sums are fp32); rows are bit-identical
whatever T is (batch invariance). The gated delta rule: 2e-4 relative / 2e-6 absolute on outputs and state."""
import ctypes

import numpy as np
import pytest

import refimpl
from bonsai_b200 import _lib
from oracle import oracle as orc
from test_oracle import gdn_case, ternary_case

pytestmark = pytest.mark.gpu


def dev(torch, arr, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def vp(t):
    return ctypes.c_void_p(t.data_ptr())


class Linear:
    def __init__(self, W, S, B, group):
        self.L = _lib.lib()
        self.h = ctypes.c_void_p()
        O, K = W.shape[0], W.shape[1] * 16
        s = self.L.bcu_linear_prepare(orc.ptr(W), orc.ptr(S), orc.ptr(B) if B is not None else None, O, K, group, 0,
                                      ctypes.byref(self.h))
        assert s == _lib.OK
        self.O = O

    def rotate_forward(self, torch, xb_bits, HB, signs):
        T = xb_bits.shape[0]
        x = dev(torch, xb_bits)
        y = torch.empty((T, self.O), dtype=torch.float32, device="cuda")
        sg = dev(torch, signs) if signs is not None else None
        s = self.L.bcu_linear_rotate_forward(self.h, vp(x), T, HB, vp(sg) if sg is not None else None, vp(y), None)
        assert s == _lib.OK
        torch.cuda.synchronize()
        return y.cpu().numpy()

    def __del__(self):
        self.L.bcu_linear_free(self.h)


def bf16_bits(torch, x):
    return torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("group,bias,HB,signed", [(64, "neg", 2048, False), (128, None, 512, True),
                                                  (64, "free", 512, False)])
def test_config1_rotate_linear_parity(gpu, group, bias, HB, signed):
    torch = pytest.importorskip("torch")
    O, K, T = 1024, 2048, 9
    W, S, B, X = ternary_case(O, K, group, T, bias, 100 + group)
    xb = bf16_bits(torch, X)
    signs = np.where(np.random.default_rng(5).random(K) < 0.5, -1, 1).astype(np.float32) if signed else None
    lin = Linear(W, S, B, group)
    y = lin.rotate_forward(torch, xb, HB, signs)
    want, xr = orc.rotate_ternary_linear(W, S, B, group, xb, HB, signs)
    Wd = refimpl.dense_weights(W, S, B, group)
    bound = 2e-5 * (np.abs(xr).astype(np.float64) @ np.abs(Wd).T) + 1e-5
    err = np.abs(y.astype(np.float64) - want)
    assert np.all(err <= bound), f"max err {err.max()} vs bound {bound[err > bound].min()}"


def test_config1_full_shape_and_batch_invariance(gpu):
    """Graded config 1 shape (9 x 2048 -> 6144, g64 + bias, 2048-point rotation); every row is bit-identical to the
    same row computed alone, for every T in 1..16."""
    torch = pytest.importorskip("torch")
    O, K = 6144, 2048
    W, S, B, X = ternary_case(O, K, 64, 16, "neg", 42)
    xb = bf16_bits(torch, X)
    lin = Linear(W, S, B, 64)
    y16 = lin.rotate_forward(torch, xb, 2048, None)
    want, xr = orc.rotate_ternary_linear(W, S, B, 64, xb, 2048)
    Wd = refimpl.dense_weights(W, S, B, 64)
    bound = 2e-5 * (np.abs(xr).astype(np.float64) @ np.abs(Wd).T) + 1e-5
    assert np.all(np.abs(y16.astype(np.float64) - want) <= bound)
    alone = [lin.rotate_forward(torch, xb[t:t + 1], 2048, None)[0] for t in range(16)]
    for T in range(1, 17):
        yT = lin.rotate_forward(torch, xb[:T], 2048, None)
        for t in range(T):
            assert np.array_equal(yT[t].view(np.uint32), alone[t].view(np.uint32)), (T, t)


@pytest.mark.parametrize("O,K,group,HB,T", [(6144, 2048, 64, 2048, 9), (1024, 2048, 128, 512, 16),
                                            (2048, 4096, 64, 1024, 5), (1024, 2048, 64, 2048, 1),
                                            (6144, 2048, 64, 2048, 16), (1024, 4096, 128, 2048, 13)])
def test_rotate_linear_grid_and_local_build_agree(gpu, O, K, group, HB, T):
    """The operand built by all CTAs together (the default when they fit at once) and by each CTA for its own slice:
    the same plan and the same operand values, so the outputs are the same bits."""
    torch = pytest.importorskip("torch")
    W, S, B, X = ternary_case(O, K, group, T, "neg", 300 + HB)
    xb = bf16_bits(torch, X)
    signs = np.where(np.random.default_rng(HB).random(K) < 0.5, -1, 1).astype(np.float32)
    lin = Linear(W, S, B, group)
    grid = lin.rotate_forward(torch, xb, HB, signs)
    assert lin.L.bcu_linear_set_local_build(lin.h, 1) == _lib.OK
    local = lin.rotate_forward(torch, xb, HB, signs)
    assert lin.L.bcu_linear_set_local_build(lin.h, 0) == _lib.OK
    assert np.array_equal(grid.view(np.uint32), local.view(np.uint32))
    want, xr = orc.rotate_ternary_linear(W, S, B, group, xb, HB, signs)
    Wd = refimpl.dense_weights(W, S, B, group)
    bound = 2e-5 * (np.abs(xr).astype(np.float64) @ np.abs(Wd).T) + 1e-5
    assert np.all(np.abs(grid.astype(np.float64) - want) <= bound)


@pytest.mark.parametrize("O,K,group,HB,T", [(2048, 4096, 64, 512, 9), (2048, 6144, 64, 512, 9),
                                            (2048, 4096, 64, 512, 16), (1024, 2560, 64, 512, 1),
                                            (1024, 8192, 128, 512, 4)])
def test_split_sums_cluster_and_partial_buffer_agree(gpu, O, K, group, HB, T):
    """A row block's K-split sums through the shared memory of a thread-block cluster (the default when the clusters
    fit; 8 and 6 splits here, 5 for the 4B shape's 2560 inputs) and through the global partial buffer (the path for
    more than 8 splits, the last case): the same sums in the same order, so the outputs are the same bits."""
    torch = pytest.importorskip("torch")
    W, S, B, X = ternary_case(O, K, group, T, "neg", 500 + K + T)
    xb = bf16_bits(torch, X)
    signs = np.where(np.random.default_rng(K).random(K) < 0.5, -1, 1).astype(np.float32)
    lin = Linear(W, S, B, group)
    try:
        cl = lin.rotate_forward(torch, xb, HB, signs)
        assert lin.L.bcu_gemv_set_clusters(0) == 0
        buf = lin.rotate_forward(torch, xb, HB, signs)
    finally:
        lin.L.bcu_gemv_set_clusters(1)
    assert np.array_equal(cl.view(np.uint32), buf.view(np.uint32))
    want, xr = orc.rotate_ternary_linear(W, S, B, group, xb, HB, signs)
    Wd = refimpl.dense_weights(W, S, B, group)
    bound = 2e-5 * (np.abs(xr).astype(np.float64) @ np.abs(Wd).T) + 1e-5
    assert np.all(np.abs(cl.astype(np.float64) - want) <= bound)


@pytest.mark.parametrize("n", list(range(10)))
def test_config2_gdn_verify_rollback(gpu, n):
    torch = pytest.importorskip("torch")
    NK, NV, T = 16, 32, 9
    q, k, v, a, b, alog, dtb, S = gdn_case(T, NK, NV, 77)
    want_y, want_s = orc.gdn_verify(q, k, v, a, b, alog, dtb, S, n)
    t = [dev(torch, x) for x in (q, k, v, a, b, alog, dtb)]
    st = dev(torch, S)
    y = torch.empty((T, NV, 128), dtype=torch.float32, device="cuda")
    s = _lib.lib().bcu_gdn_verify(*[vp(x) for x in t], vp(st), vp(y), T, NK, NV, n, None)
    assert s == _lib.OK
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), want_y, rtol=2e-4, atol=2e-6)
    np.testing.assert_allclose(st.cpu().numpy(), want_s, rtol=2e-4, atol=2e-6)


@pytest.mark.parametrize("T,n", [(1, 0), (1, 1), (16, 16), (20, 0), (20, 17), (20, 20), (37, 33)])
def test_gdn_verify_rows_past_one_chunk(gpu, T, n):
    """Rows are staged 16 at a time: passes longer than one chunk, and checkpoints in the second or third chunk."""
    torch = pytest.importorskip("torch")
    NK, NV = 2, 4
    q, k, v, a, b, alog, dtb, S = gdn_case(T, NK, NV, 100 + T)
    want_y, want_s = orc.gdn_verify(q, k, v, a, b, alog, dtb, S, n)
    t = [dev(torch, x) for x in (q, k, v, a, b, alog, dtb)]
    st = dev(torch, S)
    y = torch.empty((T, NV, 128), dtype=torch.float32, device="cuda")
    assert _lib.lib().bcu_gdn_verify(*[vp(x) for x in t], vp(st), vp(y), T, NK, NV, n, None) == _lib.OK
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), want_y, rtol=2e-4, atol=2e-6)
    np.testing.assert_allclose(st.cpu().numpy(), want_s, rtol=2e-4, atol=2e-6)


def run_gdn_prefill(torch, case, T, NK, NV):
    q, k, v, a, b, alog, dtb, S = case
    t = [dev(torch, x) for x in (q, k, v, a, b, alog, dtb)]
    st = dev(torch, S)
    y = torch.empty((T, NV, 128), dtype=torch.float32, device="cuda")
    nb = ctypes.c_uint64()
    assert _lib.lib().bcu_gdn_prefill_workspace(T, NV, ctypes.byref(nb)) == _lib.OK
    ws = torch.empty(nb.value // 4, dtype=torch.float32, device="cuda")
    assert _lib.lib().bcu_gdn_prefill(*[vp(x) for x in t], vp(st), vp(y), T, NK, NV, vp(ws), None) == _lib.OK
    torch.cuda.synchronize()
    return y.cpu().numpy(), st.cpu().numpy()


@pytest.mark.parametrize("T", [1, 5, 63, 64, 65, 130, 300])
def test_gdn_prefill_chunks_match_oracle(gpu, T):
    """The prefill chunk's gated delta rule in 64-row chunks against the oracle's row-by-row recurrence (n = T):
    one partial chunk, exactly one chunk, chunk boundaries, several chunks."""
    torch = pytest.importorskip("torch")
    NK, NV = 2, 4
    case = gdn_case(T, NK, NV, 300 + T)
    want_y, want_s = orc.gdn_verify(*case, T)
    y, st = run_gdn_prefill(torch, case, T, NK, NV)
    np.testing.assert_allclose(y, want_y, rtol=2e-4, atol=2e-6)
    np.testing.assert_allclose(st, want_s, rtol=2e-4, atol=2e-6)


def test_gdn_prefill_graded_heads_long_chunk(gpu):
    """The benchmark's GDN widths (16 key / 32 value heads) over a 2047-row prefill chunk, with a starting state."""
    torch = pytest.importorskip("torch")
    T, NK, NV = 2047, 16, 32
    case = gdn_case(T, NK, NV, 4242)
    want_y, want_s = orc.gdn_verify(*case, T)
    y, st = run_gdn_prefill(torch, case, T, NK, NV)
    np.testing.assert_allclose(y, want_y, rtol=2e-4, atol=2e-6)
    np.testing.assert_allclose(st, want_s, rtol=2e-4, atol=2e-6)
