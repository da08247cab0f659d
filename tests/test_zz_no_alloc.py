"""The no-allocation entry point bcu_linear_rotate_forward_static, through the C ABI.

It serves callers that may not allocate device memory while they run the layer (a host whose device memory
belongs to its own pool, or a decode loop that must not stall on the device synchronisation a cudaMalloc/cudaFree
can cause): its scratch is a static device array in the library instead of the handle's buffers. Each case checks
two calls in a row, with different inputs, against the existing entry point bcu_linear_rotate_forward on the same
inputs, within the config-1 tolerance |dy| <= 2e-5 * sum_k |w_k x_k| + 1e-5 (the two share the kernel and its
reduction order, so in practice they agree bit for bit). Sizes beyond the static capacity must be refused with
BCU_ERR_TOO_LARGE. This file is collected last so it runs after the other GPU tests; it also passes alone."""
import ctypes

import numpy as np
import pytest

import refimpl
from bonsai_b200 import _lib
from oracle import oracle as orc
from test_oracle import ternary_case

pytestmark = pytest.mark.gpu


def _vp(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _bf16_bits(torch, x):
    return torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("O,K,group,HB,signed", [(2048, 6144, 64, 512, True), (6144, 2048, 64, 2048, False),
                                                  (2048, 2048, 128, 0, False)])
def test_static_scratch_matches_allocating_entry(gpu, O, K, group, HB, signed):
    torch = pytest.importorskip("torch")
    L = _lib.lib()
    T = 9
    W, S, B, X1 = ternary_case(O, K, group, T, "neg", 7 + O)
    X2 = np.random.default_rng(11 + K).standard_normal((T, K)).astype(np.float32)
    signs = np.where(np.random.default_rng(3).random(K) < 0.5, -1, 1).astype(np.float32) if signed else None
    h = ctypes.c_void_p()
    assert L.bcu_linear_prepare(orc.ptr(W), orc.ptr(S), orc.ptr(B), O, K, group, 0, ctypes.byref(h)) == _lib.OK
    try:
        sg = torch.from_numpy(signs).cuda() if signs is not None else None
        Wd = refimpl.dense_weights(W, S, B, group)
        for X in (X1, X2):
            xb = _bf16_bits(torch, X)
            x = torch.from_numpy(xb.view(np.int16)).cuda()
            y_ref = torch.full((T, O), float("nan"), dtype=torch.float32, device="cuda")
            y_new = torch.full((T, O), float("nan"), dtype=torch.float32, device="cuda")
            assert L.bcu_linear_rotate_forward(h, _vp(x), T, HB, _vp(sg), _vp(y_ref), None) == _lib.OK
            assert L.bcu_linear_rotate_forward_static(h, _vp(x), T, HB, _vp(sg), _vp(y_new), None) == _lib.OK
            torch.cuda.synchronize()
            a, b = y_ref.cpu().numpy().astype(np.float64), y_new.cpu().numpy().astype(np.float64)
            assert np.isfinite(b).all()
            if HB:
                want, xr = orc.rotate_ternary_linear(W, S, B, group, xb, HB, signs)
            else:
                xr = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).float().numpy()
                want = orc.ternary_linear(W, S, B, group, xr)
            bound = 2e-5 * (np.abs(xr).astype(np.float64) @ np.abs(Wd).T) + 1e-5
            err = np.abs(a - b)
            assert np.all(err <= bound), f"static vs allocating entry: max err {err.max()}"
            err = np.abs(want.astype(np.float64) - b)
            assert np.all(err <= bound), f"static entry vs oracle: max err {err.max()}"
        # the error word of the static array: clean after these calls, and a recorded timeout is reported once
        assert L.bcu_linear_sync(h, None) == _lib.OK
        assert L.bcu_static_scratch_debug(0, 1) == _lib.OK
        assert L.bcu_linear_sync(h, None) == _lib.ERR_TIMEOUT
        assert L.bcu_linear_sync(h, None) == _lib.OK
    finally:
        L.bcu_linear_free(h)


def test_static_scratch_rejects_oversize(gpu):
    """16384 x 4096 runs as 2 K-splits: 2 x 9 x 16384 partial sums exceed the 262144-float static array."""
    torch = pytest.importorskip("torch")
    L = _lib.lib()
    O, K, group = 16384, 4096, 64
    rng = np.random.default_rng(1)
    W = rng.integers(0, 2**32, size=(O, K // 16), dtype=np.uint64).astype(np.uint32)
    S = np.full((O, K // group), 0.01, dtype=np.float16).view(np.uint16)
    B = np.full((O, K // group), -0.01, dtype=np.float16).view(np.uint16)
    h = ctypes.c_void_p()
    assert L.bcu_linear_prepare(orc.ptr(W), orc.ptr(S), orc.ptr(B), O, K, group, 0, ctypes.byref(h)) == _lib.OK
    try:
        x = torch.zeros((9, K), dtype=torch.int16, device="cuda")  # valid buffers all the same
        y = torch.zeros((9, O), dtype=torch.float32, device="cuda")
        st = L.bcu_linear_rotate_forward_static(h, _vp(x), 9, 512, None, _vp(y), None)
        torch.cuda.synchronize()
        assert st == _lib.ERR_TOO_LARGE
    finally:
        L.bcu_linear_free(h)


def test_static_scratch_rejects_too_many_row_blocks(gpu):
    """131200 rows are 1025 row blocks: one more than the static array's 1024 counters."""
    torch = pytest.importorskip("torch")
    L = _lib.lib()
    O, K, group = 131200, 512, 128
    W = np.zeros((O, K // 16), np.uint32)
    S = np.full((O, K // group), 0.01, dtype=np.float16).view(np.uint16)
    h = ctypes.c_void_p()
    assert L.bcu_linear_prepare(orc.ptr(W), orc.ptr(S), None, O, K, group, 0, ctypes.byref(h)) == _lib.OK
    try:
        x = torch.zeros((1, K), dtype=torch.int16, device="cuda")
        y = torch.zeros((1, O), dtype=torch.float32, device="cuda")
        assert L.bcu_linear_rotate_forward_static(h, _vp(x), 1, 0, None, _vp(y), None) == _lib.ERR_TOO_LARGE
    finally:
        L.bcu_linear_free(h)
