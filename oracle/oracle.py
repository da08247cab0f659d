"""ctypes wrapper of the CPU oracle (oracle/bonsai_oracle.cpp). TEST INFRASTRUCTURE ONLY: imported by tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker; never part of the product path.

Pinned to the reference's own Metal kernels compiled for the host (oracle/ref.py, tests/test_ref_pin.py); the host
logic restated from Rust (drafting, policy) is pinned by known-answer tests only.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libbonsai_oracle.so")
_L = None

P = ctypes.c_void_p
I = ctypes.c_int
PU32 = ctypes.POINTER(ctypes.c_uint32)
PF = ctypes.POINTER(ctypes.c_float)


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _L
    if _L is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        sig = {
            "orc_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "orc_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
            "orc_bf16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "orc_f32_to_bf16": (ctypes.c_uint16, [ctypes.c_float]),
            "orc_fwht": (None, [P, I]),
            "orc_rotate": (None, [P, P, I, I, P]),
            "orc_norm_rotate": (None, [P, P, P, I, I, I, P, P]),
            "orc_swiglu_rotate": (None, [P, P, P, I, I, I, P]),
            "orc_gate_rotate": (None, [P, P, P, I, I, I, P]),
            "orc_gated_norm_rotate": (None, [P, P, P, P, I, I, I, P]),
            "orc_embed_ternary": (None, [P, P, P, P, I, I, I, PU32, I, P]),
            "orc_ternary_linear": (None, [P, P, P, I, I, I, P, I, P]),
            "orc_rotate_ternary_linear": (None, [P, P, P, I, I, I, P, I, I, P, P, P]),
            "orc_gdn_verify": (None, [P, P, P, P, P, P, P, P, P, I, I, I, I]),
            "orc_accept_len": (I, [PU32, PU32, I]),
            "orc_argmax": (I, [PF, I]),
            "orc_model_create": (P, [P]),
            "orc_model_load_tensor": (I, [P, ctypes.c_char_p, I, ctypes.POINTER(ctypes.c_int64), I, P]),
            "orc_model_finalize": (I, [P]),
            "orc_model_reset": (None, [P]),
            "orc_model_forward": (I, [P, PU32, I, PF, PU32]),
            "orc_model_accept": (None, [P, I]),
            "orc_model_len": (I, [P]),
            "orc_model_prefill": (I, [P, PU32, I, I, PU32]),
            "orc_model_snapshot": (P, [P]),
            "orc_model_restore": (None, [P, P]),
            "orc_state_free": (None, [P]),
            "orc_model_set_state": (I, [P, P, P, P, P, I]),
            "orc_model_destroy": (None, [P]),
            "orc_greedy": (I, [P, ctypes.c_uint32, I, PU32, I, PU32]),
            "orc_model_set_lora": (I, [P, I, ctypes.c_char_p, P, P, I, ctypes.c_float]),
            "orc_model_clear_lora": (None, [P]),
            "orc_lora_add": (None, [P, P, I, I, I, P, I, P]),
            "orc_token_key": (ctypes.c_uint64, [P, I]),
            "orc_lookup": (I, [PU32, I, PU32, I, ctypes.POINTER(ctypes.c_uint64), I, I, I, I, I, I, PU32, ctypes.POINTER(I)]),
            "orc_draft_source": (I, [PU32, I, P, ctypes.POINTER(ctypes.c_uint64), I, PU32, I, PU32]),
            "orc_normalize_draft": (I, [PU32, I, ctypes.c_uint32, P, ctypes.POINTER(ctypes.c_uint64), I, P, P]),
            "orc_policy_choose": (I, [ctypes.c_double, ctypes.c_double, ctypes.POINTER(ctypes.c_double), I, I,
                                      ctypes.c_double, ctypes.POINTER(ctypes.c_double)]),
        }
        for k, (r, a) in sig.items():
            f = getattr(L, k)
            f.restype = r
            f.argtypes = a
        _L = L
    return _L


def ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def u32p(a):
    return a.ctypes.data_as(PU32)


def ternary_linear(W, S, B, group, X):
    """W u32 [O, K/16], S/B fp16 bits [O, K/group] (B may be None), X fp32 [T, K] -> fp32 [T, O]."""
    O, K = W.shape[0], W.shape[1] * 16
    X = np.ascontiguousarray(X, np.float32)
    T = X.shape[0]
    Y = np.zeros((T, O), np.float32)
    lib().orc_ternary_linear(ptr(W), ptr(S), ptr(B) if B is not None else None, O, K, group, ptr(X), T, ptr(Y))
    return Y


def rotate_ternary_linear(W, S, B, group, Xbf16, HB, signs=None):
    O, K = W.shape[0], W.shape[1] * 16
    T = Xbf16.shape[0]
    Y = np.zeros((T, O), np.float32)
    Xr = np.zeros((T, K), np.float32)
    lib().orc_rotate_ternary_linear(ptr(W), ptr(S), ptr(B) if B is not None else None, O, K, group, ptr(Xbf16), T, HB,
                                    ptr(signs) if signs is not None else None, ptr(Y), ptr(Xr))
    return Y, Xr


def rotate(x, HB, signs=None):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().orc_rotate(ptr(x), ptr(signs) if signs is not None else None, x.size, HB, ptr(out))
    return out


def _f(a):
    return np.ascontiguousarray(a, np.float32)


def norm_rotate(h, w, signs, HB=512):
    h = _f(h)
    T, D = h.shape
    xn, xr = np.zeros_like(h), np.zeros_like(h)
    lib().orc_norm_rotate(ptr(h), ptr(_f(w)), ptr(_f(signs)) if signs is not None else None, D, HB, T, ptr(xn), ptr(xr))
    return xn, xr


def swiglu_rotate(g, u, signs, HB=512):
    g, u = _f(g), _f(u)
    T, D = g.shape
    xr = np.zeros_like(g)
    lib().orc_swiglu_rotate(ptr(g), ptr(u), ptr(_f(signs)) if signs is not None else None, D, HB, T, ptr(xr))
    return xr


def gate_rotate(attn, qp, signs, HB=512):
    attn, qp = _f(attn), _f(qp)
    T, W = attn.shape
    xr = np.zeros_like(attn)
    lib().orc_gate_rotate(ptr(attn), ptr(qp), ptr(_f(signs)) if signs is not None else None, W, HB, T, ptr(xr))
    return xr


def gated_norm_rotate(y, z, w, signs, HB=512):
    y, z = _f(y), _f(z)
    T, W = y.shape
    xr = np.zeros_like(y)
    lib().orc_gated_norm_rotate(ptr(y), ptr(z), ptr(_f(w)), ptr(_f(signs)) if signs is not None else None, W, HB, T,
                                ptr(xr))
    return xr


def embed_ternary(W, S, B, signs, group, HB, d, ids):
    ids = np.ascontiguousarray(ids, np.uint32)
    out = np.zeros((len(ids), d), np.float32)
    lib().orc_embed_ternary(ptr(W), ptr(S), ptr(B) if B is not None else None,
                            ptr(_f(signs)) if signs is not None else None, group, HB, d, u32p(ids), len(ids), ptr(out))
    return out


def gdn_verify(q, k, v, a, b, a_log, dt_bias, state, n):
    """Returns (y, new_state); inputs are not modified."""
    T, NK = q.shape[0], q.shape[1]
    NV = v.shape[1]
    st = np.ascontiguousarray(state, np.float32).copy()
    y = np.zeros((T, NV, 128), np.float32)
    arrs = [np.ascontiguousarray(x, np.float32) for x in (q, k, v, a, b, a_log, dt_bias)]
    lib().orc_gdn_verify(*[ptr(x) for x in arrs], ptr(st), ptr(y), T, NK, NV, n)
    return y, st


def lora_add(a, b, xu, y):
    """y [T, O] + B (A xu) per row (the oracle's LoRA arithmetic); returns a new array."""
    a, b, xu = (np.ascontiguousarray(x, np.float32) for x in (a, b, xu))
    out = np.ascontiguousarray(y, np.float32).copy()
    lib().orc_lora_add(ptr(a), ptr(b), a.shape[0], b.shape[0], a.shape[1], ptr(xu), xu.shape[0], ptr(out))
    return out


class OracleModel:
    """The oracle's Model: same tensor names and pass semantics as the product's bcu_model."""

    def __init__(self, cfg, tensors):
        L = lib()
        self.cfg = cfg
        self.h = L.orc_model_create(ctypes.byref(cfg))
        for name, code, arr in tensors:
            arr = np.ascontiguousarray(arr)
            shape = (ctypes.c_int64 * arr.ndim)(*arr.shape)
            L.orc_model_load_tensor(self.h, name.encode(), code, shape, arr.ndim, ptr(arr))
        if L.orc_model_finalize(self.h) != 0:
            raise RuntimeError("oracle: missing or mis-shaped tensor")

    def set_lora(self, linears, fold):
        """linears: (layer, module, A [r, in], B [out, r]) as lora.rs reads them; fold = alpha / r x scale."""
        lib().orc_model_clear_lora(self.h)
        for layer, module, a, b in linears:
            a = np.ascontiguousarray(a, np.float32)
            b = np.ascontiguousarray(b, np.float32)
            if lib().orc_model_set_lora(self.h, layer, module.encode(), ptr(a), ptr(b), a.shape[0], fold) != 0:
                raise ValueError(f"oracle: no linear layers.{layer}.{module}")

    def clear_lora(self):
        lib().orc_model_clear_lora(self.h)

    def forward(self, ids, logits=False):
        ids = np.ascontiguousarray(ids, np.uint32)
        T = len(ids)
        pred = np.zeros(T, np.uint32)
        lg = np.zeros((T, self.cfg.vocab), np.float32) if logits else None
        r = lib().orc_model_forward(self.h, u32p(ids), T, lg.ctypes.data_as(PF) if logits else None, u32p(pred))
        if r != 0:
            raise RuntimeError("oracle: context full")
        return (pred, lg) if logits else pred

    def accept(self, n):
        lib().orc_model_accept(self.h, n)

    def verify(self, ids):
        """Forward + accept of m+1 rows, like bcu_verify: (pred, m)."""
        pred = self.forward(ids)
        m = lib().orc_accept_len(u32p(np.ascontiguousarray(ids, np.uint32)), u32p(pred), len(ids))
        self.accept(m + 1)
        return pred, m

    def prefill(self, ids, chunk=16):
        ids = np.ascontiguousarray(ids, np.uint32)
        nxt = ctypes.c_uint32()
        if lib().orc_model_prefill(self.h, u32p(ids), len(ids), chunk, ctypes.byref(nxt)) != 0:
            raise RuntimeError("oracle: context full")
        return nxt.value

    def greedy(self, first, max_tokens, eos=()):
        out = np.zeros(max_tokens, np.uint32)
        e = np.ascontiguousarray(eos if len(eos) else [0], np.uint32)
        n = lib().orc_greedy(self.h, first, max_tokens, u32p(e), len(eos), u32p(out))
        return out[:n]

    @property
    def length(self):
        return lib().orc_model_len(self.h)

    def snapshot(self):
        return lib().orc_model_snapshot(self.h)

    def restore(self, s):
        lib().orc_model_restore(self.h, s)

    def set_state(self, gdn, conv, kc, vc, length):
        """The committed state from the four state parts (fp32 arrays in the bcu_state_read layout)."""
        arrs = [np.ascontiguousarray(x, np.float32) for x in (gdn, conv, kc, vc)]
        if lib().orc_model_set_state(self.h, *[ptr(x) for x in arrs], length) != 0:
            raise ValueError("oracle: state longer than the context")

    def free_snapshot(self, s):
        lib().orc_state_free(s)

    def reset(self):
        lib().orc_model_reset(self.h)

    def __del__(self):
        try:
            lib().orc_model_destroy(self.h)
        except Exception:
            pass


def token_key(b):
    buf = np.frombuffer(b, np.uint8) if b else np.zeros(1, np.uint8)
    return lib().orc_token_key(ptr(buf), len(b))


def lookup(src, seq, keys, ngram_max, ngram_min, draft_max, limit, cursor):
    src = np.ascontiguousarray(src, np.uint32)
    seq = np.ascontiguousarray(seq, np.uint32)
    keys = np.ascontiguousarray(keys, np.uint64)
    out = np.zeros(16, np.uint32)
    dpos = ctypes.c_int()
    n = lib().orc_lookup(u32p(src), len(src), u32p(seq), len(seq), keys.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
                         len(keys), ngram_max, ngram_min, draft_max, limit, cursor, u32p(out), ctypes.byref(dpos))
    return out[:n].copy(), dpos.value
