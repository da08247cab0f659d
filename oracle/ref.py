"""ctypes wrapper of oracle/_ref/libbonsai_ref.so: the reference's own Metal text kernels (kernels.metal) compiled for
the host through oracle/ref_metal/metal_stdlib, and the reference's layer sequence (model.rs) over them. TEST
INFRASTRUCTURE ONLY: it pins the oracle to the reference; the product never loads it.

The library is built by oracle/Makefile from the reference tree where it lies; where the tree is absent (the GPU
box), available() is False and the tests that need it skip.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libbonsai_ref.so")
_L = None

P = ctypes.c_void_p
U = ctypes.c_uint32
I = ctypes.c_int32


def available():
    return os.path.exists(LIB)


def lib():
    global _L
    if _L is None:
        L = ctypes.CDLL(LIB)
        sig = {
            "rk_norm_rotate": (None, [P, P, P, P, P, U, U, U]),
            "rk_swiglu_rotate": (None, [P, P, P, P, U, U]),
            "rk_gate_rotate": (None, [P, P, P, P, U, U]),
            "rk_gated_norm_rotate": (None, [P, P, P, P, P, U, U]),
            "rk_embed": (None, [P, P, P, P, P, U, U]),
            "rk_ternary_matmul": (None, [P, P, U, U, P, U, P, I]),
            "rk_gdn_recurrent": (None, [P, P, P, P, P, P, P, U, U, U]),
            "rk_argmax": (None, [P, U, U, P]),
            "rk_model_create": (P, [P]),
            "rk_model_load_tensor": (I, [P, ctypes.c_char_p, P, ctypes.c_uint64]),
            "rk_model_finalize": (I, [P]),
            "rk_model_pass": (I, [P, P, U, I, P, P]),
            "rk_model_accept": (None, [P, U, U]),
            "rk_model_len": (U, [P]),
            "rk_model_destroy": (None, [P]),
        }
        for k, (r, a) in sig.items():
            f = getattr(L, k)
            f.restype = r
            f.argtypes = a
        _L = L
    return _L


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _c(a, dt):
    return np.ascontiguousarray(a, dt)


def norm_rotate(h, w, signs, write_xn=0):
    h = _c(h, np.float32)
    T, D = h.shape
    xn = np.zeros_like(h)
    xr = np.zeros_like(h)
    lib().rk_norm_rotate(_p(h), _p(_c(w, np.float32)), _p(_c(signs, np.float32)), _p(xn), _p(xr), D, write_xn, T)
    return xn, xr


def swiglu_rotate(g, u, signs):
    g, u = _c(g, np.float32), _c(u, np.float32)
    T, D = g.shape
    xr = np.zeros_like(g)
    lib().rk_swiglu_rotate(_p(g), _p(u), _p(_c(signs, np.float32)), _p(xr), D, T)
    return xr


def gate_rotate(attn, qp, signs):
    attn, qp = _c(attn, np.float32), _c(qp, np.float32)
    T, W = attn.shape
    xr = np.zeros_like(attn)
    lib().rk_gate_rotate(_p(attn), _p(qp), _p(_c(signs, np.float32)), _p(xr), W, T)
    return xr


def gated_norm_rotate(y, zg, w, signs):
    y, zg = _c(y, np.float32), _c(zg, np.float32)
    T, W = y.shape
    xr = np.zeros_like(y)
    lib().rk_gated_norm_rotate(_p(y), _p(zg), _p(_c(w, np.float32)), _p(_c(signs, np.float32)), _p(xr), W, T)
    return xr


def embed(W, S, signs, ids, D):
    ids = _c(ids, np.int32)
    out = np.zeros((len(ids), D), np.float32)
    lib().rk_embed(_p(_c(W, np.uint32)), _p(_c(S, np.uint16)), _p(_c(signs, np.float32)), _p(ids), _p(out), D, len(ids))
    return out


def ternary_matmul(W, S, x, y=None):
    """y (+)= x W^T with the kernel the reference picks for x's row count (qmv4, qmvr, qmvxm or qmm)."""
    W, S, x = _c(W, np.uint32), _c(S, np.uint16), _c(x, np.float32)
    O, K = W.shape[0], W.shape[1] * 16
    t = x.shape[0]
    add = y is not None
    out = _c(y, np.float32).copy() if add else np.zeros((t, O), np.float32)
    lib().rk_ternary_matmul(_p(W), _p(S), O, K, _p(x), t, _p(out), 1 if add else 0)
    return out


def gdn_recurrent(qkvc, ab, alog, dtb, state, NK, NV):
    qkvc, ab = _c(qkvc, np.float32), _c(ab, np.float32)
    T = qkvc.shape[0]
    st = _c(state, np.float32).copy()
    y = np.zeros((T, NV * 128), np.float32)
    lib().rk_gdn_recurrent(_p(qkvc), _p(ab), _p(_c(alog, np.float32)), _p(_c(dtb, np.float32)), _p(st), _p(st), _p(y),
                           T, NK, NV)
    return y, st


def argmax(x):
    x = _c(x, np.float32)
    n, V = x.shape
    out = np.zeros(n, np.int32)
    lib().rk_argmax(_p(x), V, n, _p(out))
    return out


class RefModel:
    """The reference's Text on its own kernels (reference pack only: g128, implicit bias, 512-point blocks with
    signs, ternary tied head, 4 query heads per KV head)."""

    def __init__(self, cfg, tensors):
        L = lib()
        self.cfg = cfg
        self.h = L.rk_model_create(ctypes.byref(cfg))
        self._keep = []
        for name, _code, arr in tensors:
            arr = np.ascontiguousarray(arr)
            L.rk_model_load_tensor(self.h, name.encode(), _p(arr), arr.nbytes)
        r = L.rk_model_finalize(self.h)
        if r != 0:
            raise ValueError(f"reference model: finalize failed ({r})")

    def pass_(self, ids, verify):
        ids = _c(ids, np.uint32)
        t = len(ids)
        lg = np.zeros((t, self.cfg.vocab), np.float32)
        pred = np.zeros(t, np.int32)
        if lib().rk_model_pass(self.h, _p(ids), t, 1 if verify else 0, _p(lg), _p(pred)) != 0:
            raise ValueError("reference model: bad pass")
        return pred, lg

    def prefill_chunk(self, ids):
        return self.pass_(ids, False)

    def verify(self, ids):
        return self.pass_(ids, True)

    def accept(self, t, n):
        lib().rk_model_accept(self.h, t, n)

    @property
    def length(self):
        return lib().rk_model_len(self.h)

    def __del__(self):
        try:
            lib().rk_model_destroy(self.h)
        except Exception:
            pass
