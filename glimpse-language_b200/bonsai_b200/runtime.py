"""Model: the Python face of one bcu_model (runtime/mod.rs `Model` + model.rs `Text`), method for method."""
import ctypes

import numpy as np

from . import _lib


class BackendError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"{_lib.STATUS_NAMES[status] if 0 <= status < len(_lib.STATUS_NAMES) else status}: {message}")
        self.status = status
        self.message = message


def _u32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


class Model:
    def __init__(self, cfg, device=0):
        self.L = _lib.lib()
        self.cfg = cfg
        self.h = ctypes.c_void_p()
        s = self.L.bcu_create(ctypes.byref(cfg), device, ctypes.byref(self.h))
        if s != _lib.OK:
            msg = self.L.bcu_last_error(self.h).decode() if self.h else "bad config"
            raise BackendError(s, msg)

    def _ck(self, s):
        if s != _lib.OK:
            raise BackendError(s, self.L.bcu_last_error(self.h).decode())

    def close(self):
        if self.h:
            self.L.bcu_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- loading
    def load_tensor(self, name, code, arr):
        arr = np.ascontiguousarray(arr)
        shape = (ctypes.c_int64 * arr.ndim)(*arr.shape)
        self._ck(self.L.bcu_load_tensor(self.h, name.encode(), code, shape, arr.ndim,
                                        arr.ctypes.data_as(ctypes.c_void_p)))

    def load(self, tensors):
        for name, code, arr in tensors:
            self.load_tensor(name, code, arr)
        self._ck(self.L.bcu_finalize(self.h))
        return self

    # ---------------------------------------------------------------- passes
    def reset(self):
        self._ck(self.L.bcu_reset(self.h))

    def prefill(self, ids):
        ids = _u32(ids)
        nxt = ctypes.c_uint32()
        self._ck(self.L.bcu_prefill(self.h, ids.ctypes.data_as(_lib.PU32), len(ids), ctypes.byref(nxt)))
        return nxt.value

    def step(self, tok):
        nxt = ctypes.c_uint32()
        self._ck(self.L.bcu_step(self.h, int(tok), ctypes.byref(nxt)))
        return nxt.value

    def verify(self, ids):
        """Model::verify + the device accept length: (pred per row, m)."""
        ids = _u32(ids)
        pred = np.zeros(len(ids), np.uint32)
        m = ctypes.c_int32()
        self._ck(self.L.bcu_verify(self.h, ids.ctypes.data_as(_lib.PU32), len(ids), pred.ctypes.data_as(_lib.PU32),
                                   ctypes.byref(m)))
        return pred, m.value

    def verify_accept(self, ids):
        ids = _u32(ids)
        m = ctypes.c_int32()
        b = ctypes.c_uint32()
        self._ck(self.L.bcu_verify_accept(self.h, ids.ctypes.data_as(_lib.PU32), len(ids), ctypes.byref(m),
                                          ctypes.byref(b)))
        return m.value, b.value

    def accept(self, t, n):
        self._ck(self.L.bcu_accept(self.h, t, n))

    def flush(self):
        self._ck(self.L.bcu_flush(self.h))

    @property
    def length(self):
        v = ctypes.c_int32()
        self._ck(self.L.bcu_length(self.h, ctypes.byref(v)))
        return v.value

    def keep_logits(self, on=True):
        self._ck(self.L.bcu_set_keep_logits(self.h, 1 if on else 0))

    def logits(self, row):
        out = np.empty(self.cfg.vocab, np.float32)
        self._ck(self.L.bcu_read_logits(self.h, row, out.ctypes.data_as(ctypes.c_void_p)))
        return out

    # ---------------------------------------------------------------- prefix cache
    def snapshot(self):
        s = ctypes.c_void_p()
        self._ck(self.L.bcu_snapshot(self.h, ctypes.byref(s)))
        return Snapshot(self, s)

    def restore(self, snap):
        self._ck(self.L.bcu_restore(self.h, snap.h))

    def new_snapshot(self, length):
        s = ctypes.c_void_p()
        self._ck(self.L.bcu_state_new(self.h, length, ctypes.byref(s)))
        return Snapshot(self, s)

    # ---------------------------------------------------------------- decoding
    def decode(self, first, user=(), *, speculate=True, mode=_lib.DRAFT_LOOKUP, planted=None, seed=0, eos=(),
               max_tokens=300, ngram_max=3, ngram_min=1, draft_max=7):
        user = _u32(user) if len(user) else np.zeros(1, np.uint32)
        n_user = len(user) if len(user) and user.size else 0
        planted_a = _u32(planted) if planted is not None else np.zeros(1, np.uint32)
        eos_a = _u32(eos) if len(eos) else np.zeros(1, np.uint32)
        out = np.zeros(max(max_tokens, 1), np.uint32)
        n = ctypes.c_int32()
        st = _lib.BcuStats()
        spec = _lib.BcuSpec(ngram_max, ngram_min, draft_max)
        self._ck(self.L.bcu_decode(self.h, int(first), user.ctypes.data_as(_lib.PU32), n_user,
                                   ctypes.byref(spec) if speculate else None, mode,
                                   planted_a.ctypes.data_as(_lib.PU32), len(planted) if planted is not None else 0,
                                   seed, eos_a.ctypes.data_as(_lib.PU32), len(eos), max_tokens,
                                   out.ctypes.data_as(_lib.PU32), ctypes.byref(n), ctypes.byref(st)))
        return out[: n.value].copy(), st

    def set_vocab_bytes(self, tokens):
        """Per-token bytes for prompt-lookup keys (token_key, runtime/mod.rs:73-81)."""
        data = b"".join(tokens)
        offs = np.zeros(len(tokens) + 1, np.uint64)
        offs[1:] = np.cumsum([len(t) for t in tokens])
        buf = np.frombuffer(data, np.uint8) if data else np.zeros(1, np.uint8)
        self._ck(self.L.bcu_set_vocab_bytes(self.h, buf.ctypes.data_as(ctypes.c_void_p),
                                            offs.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), len(tokens)))

    def cancel(self, flag=True):
        self._ck(self.L.bcu_cancel(self.h, 1 if flag else 0))

    # ---------------------------------------------------------------- introspection
    def device_name(self):
        buf = ctypes.create_string_buffer(256)
        self._ck(self.L.bcu_device_name(self.h, buf, 256))
        return buf.value.decode()

    def pass_launches(self, t):
        v = ctypes.c_int32()
        self._ck(self.L.bcu_pass_launches(self.h, t, ctypes.byref(v)))
        return v.value

    def pass_bytes(self, t):
        v = ctypes.c_double()
        self._ck(self.L.bcu_pass_bytes(self.h, t, ctypes.byref(v)))
        return v.value

    def time_pass(self, t, iters=10):
        v = ctypes.c_float()
        self._ck(self.L.bcu_time_pass(self.h, t, iters, ctypes.byref(v)))
        return v.value

    def set_planted(self, ids, base):
        ids = _u32(ids)
        self._ck(self.L.bcu_set_planted(self.h, ids.ctypes.data_as(_lib.PU32), len(ids), base))

    def enqueue_passes(self, t, passes, feed):
        self._ck(self.L.bcu_enqueue_passes(self.h, t, passes, feed))

    def sync(self):
        self._ck(self.L.bcu_sync(self.h))

    def stream(self):
        s = ctypes.c_void_p()
        self._ck(self.L.bcu_stream(self.h, ctypes.byref(s)))
        return s.value


class Snapshot:
    """A bcu_state: the model state after a prefix (Prefix::snap, runtime/mod.rs:219-223)."""

    def __init__(self, model, h):
        self.model = model
        self.h = h

    def parts(self):
        sizes = (ctypes.c_uint64 * 4)()
        n = ctypes.c_int32()
        self.model._ck(self.model.L.bcu_state_parts(self.model.h, self.h, sizes, ctypes.byref(n)))
        return list(sizes), n.value

    def read(self, part):
        sizes, _ = self.parts()
        out = np.empty(sizes[part], np.uint8)
        self.model._ck(self.model.L.bcu_state_read(self.model.h, self.h, part, out.ctypes.data_as(ctypes.c_void_p),
                                                   sizes[part]))
        return out

    def write(self, part, data):
        sizes, n = self.parts()
        data = np.ascontiguousarray(np.frombuffer(bytes(data), np.uint8))
        self.model._ck(self.model.L.bcu_state_write(self.model.h, self.h, part, data.ctypes.data_as(ctypes.c_void_p),
                                                    data.size, n))

    def free(self):
        if self.h:
            self.model.L.bcu_state_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
