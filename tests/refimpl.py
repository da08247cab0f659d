"""Independent float64 numpy statements of the hot-path math, used to pin the C++ oracle (and, through the golden
fixtures, the GPU path). Written from the mathematics, not from the oracle's code."""
import numpy as np
import scipy.linalg


def f16(bits):
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float64)


def decode_codes(W):
    """u32 [O, K/16] -> codes [O, K] (code e of a word at bits 2e)."""
    O, kw = W.shape
    sh = np.arange(16, dtype=np.uint32) * 2
    return ((W[:, :, None] >> sh[None, None, :]) & 3).reshape(O, kw * 16).astype(np.float64)


def dense_weights(W, S, B, group):
    c = decode_codes(W)
    s = np.repeat(f16(S), group, axis=1)
    b = np.repeat(f16(B), group, axis=1) if B is not None else -s
    return s * c + b


def hadamard_rotate(x, HB, signs=None):
    """Block Walsh-Hadamard rotation, normalised, Sylvester order."""
    x = np.asarray(x, np.float64)
    if signs is not None:
        x = x * signs
    H = scipy.linalg.hadamard(HB).astype(np.float64) / np.sqrt(HB)
    sh = x.shape
    return (x.reshape(-1, HB) @ H.T).reshape(sh)


def gdn_verify(q, k, v, a_in, b_in, a_log, dt_bias, state, n):
    q, k, v = (np.asarray(x, np.float64) for x in (q, k, v))
    T, NK, _ = q.shape
    NV = v.shape[1]
    S = np.asarray(state, np.float64).copy()
    keep = S.copy()
    y = np.zeros((T, NV, 128))
    for t in range(T):
        for h in range(NV):
            hk = h // (NV // NK)
            a = a_in[t, h] + dt_bias[h]
            g = np.exp(-np.exp(a_log[h]) * np.logaddexp(0.0, a))
            beta = 1.0 / (1.0 + np.exp(-b_in[t, h]))
            S[h] *= g
            kv = S[h] @ k[t, hk]
            delta = (v[t, h] - kv) * beta
            S[h] += np.outer(delta, k[t, hk])
            y[t, h] = S[h] @ q[t, hk]
        if t + 1 == n:
            keep = S.copy()
    return y, keep
