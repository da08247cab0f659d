"""Model: the Python face of one bcu_model (runtime/mod.rs `Model` + model.rs `Text`), method for method."""
import ctypes

import numpy as np

from . import _lib


class BackendError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"{_lib.STATUS_NAMES[status] if 0 <= status < len(_lib.STATUS_NAMES) else status}: {message}")
        self.status = status
        self.message = message


PREFIX_SLOTS = 3  # runtime/mod.rs:213


def _u32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


class Model:
    def __init__(self, cfg, device=0):
        self.L = _lib.lib()
        self.cfg = cfg
        # prefix cache (runtime/mod.rs:213-223, 455-485): newest first, (ids, adapter, Snapshot)
        self.prefixes = []
        self.adapter = 0
        self.prefix_dir = None
        self.identity = None
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

    # ---------------------------------------------------------------- LoRA
    def set_lora_linears(self, linears, fold):
        """Text::set_lora with lora::load's tensors: linears = [(layer, module, A [r, in], B [out, r])] (empty
        removes the adapter); fold = alpha / r x scale."""
        arrs, items = [], (_lib.BcuLoraLinear * max(len(linears), 1))()
        for i, (layer, module, a, b) in enumerate(linears):
            a = np.ascontiguousarray(a, np.float32)
            b = np.ascontiguousarray(b, np.float32)
            mod = module.encode()
            arrs += [a, b, mod]
            it = items[i]
            it.layer = layer
            it.module = mod
            it.a = a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
            it.b = b.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
            it.a_shape[:] = list(a.shape) if a.ndim == 2 else [a.size, 1]
            it.b_shape[:] = list(b.shape) if b.ndim == 2 else [b.size, 1]
        self._ck(self.L.bcu_set_lora(self.h, items, len(linears), ctypes.c_float(fold)))

    def set_lora(self, path=None, scale=1.0):
        """Model::set_lora (runtime/mod.rs:328-337): loads the adapter file (or removes it: no path or scale 0),
        records its id and drops the cached prefixes of other adapters."""
        from . import lora

        if path is not None and scale != 0.0:
            linears, fold = lora.parse(path)
            self.set_lora_linears(linears, float(np.float32(fold) * np.float32(scale)))
            ident = lora.adapter_id(path, scale)
        else:
            self.set_lora_linears([], 1.0)
            ident = 0
        self.adapter = ident
        self.prefixes = [p for p in self.prefixes if p[1] == ident]

    def set_batched_prefill(self, on=True):
        """Test hook: bcu_prefill runs long prompts as tcgen05 GEMM chunks (on, the default) or as verify passes."""
        self._ck(self.L.bcu_set_batched_prefill(self.h, 1 if on else 0))

    def set_local_build(self, local=True):
        """Test hook: every GEMV builds its operand per CTA instead of once across its grid."""
        self._ck(self.L.bcu_set_local_build(self.h, 1 if local else 0))

    def debug_wait_timeout(self):
        """Test hook: a device wait that runs out; returns (status, message)."""
        st = self.L.bcu_debug_wait_timeout(self.h)
        return st, (self.L.bcu_last_error(self.h).decode() if st != _lib.OK else "")

    def lora_info(self):
        """Text::lora_info (model.rs:399-402): (adapted linears, rank), or None."""
        n, r = ctypes.c_int32(), ctypes.c_int32()
        self._ck(self.L.bcu_lora_info(self.h, ctypes.byref(n), ctypes.byref(r)))
        return (n.value, r.value) if n.value else None

    # ---------------------------------------------------------------- saved prefix files (BNSPFX01)
    def prefix_identity(self, adapter, weights, config, exe=None):
        """Model::prefix_identity (runtime/mod.rs:494-510); None when a file cannot be read."""
        n = ctypes.c_uint64()
        args = (self.h, adapter, exe.encode() if exe else None, weights.encode(), config.encode())
        s = self.L.bcu_prefix_identity(*args, None, 0, ctypes.byref(n))
        if s == _lib.ERR_NOT_FOUND:
            return None
        self._ck(s)
        buf = ctypes.create_string_buffer(n.value)
        self._ck(self.L.bcu_prefix_identity(*args, buf, n.value, ctypes.byref(n)))
        return buf.raw[: n.value]

    def save_prefix(self, snap, directory, identity, ids, background=False):
        """Model::save_prefix (runtime/mod.rs:549-578)."""
        ids = _u32(ids)
        self._ck(self.L.bcu_prefix_save(self.h, snap.h, directory.encode(), identity, len(identity),
                                        ids.ctypes.data_as(_lib.PU32), len(ids), 1 if background else 0))

    def load_prefix(self, directory, identity, ids):
        """Model::load_prefix (runtime/mod.rs:517-546): a Snapshot, or None when there is no usable file."""
        ids = _u32(ids)
        s = ctypes.c_void_p()
        self._ck(self.L.bcu_prefix_load(self.h, directory.encode(), identity, len(identity),
                                        ids.ctypes.data_as(_lib.PU32), len(ids), ctypes.byref(s)))
        return Snapshot(self, s) if s.value else None

    def set_prefix_files(self, directory, identity):
        """Model::prefix_dir plus the identity its files are saved under (None: memory slots only)."""
        self.prefix_dir, self.identity = directory, identity

    def start_prefix(self, prefix):
        """Model::start_prefix (runtime/mod.rs:455-485): restores the state after `prefix` from a memory slot or a
        saved file, or prefills it, keeps it in a slot and saves it. Returns the number of tokens served from a
        cache."""
        prefix = [int(t) for t in prefix]
        if not prefix:
            self.reset()
            return 0
        hit = next((i for i, (ids, ad, _) in enumerate(self.prefixes) if ids == prefix and ad == self.adapter), None)
        snap = self.prefixes.pop(hit)[2] if hit is not None else None
        files = self.prefix_dir is not None and self.identity is not None
        if snap is None and files:
            snap = self.load_prefix(self.prefix_dir, self.identity, prefix)
        if snap is not None:
            self.restore(snap)
            self.prefixes.insert(0, (prefix, self.adapter, snap))
            return len(prefix)
        self.reset()
        self.prefill(prefix)
        snap = self.snapshot()
        if files:
            self.save_prefix(snap, self.prefix_dir, self.identity, prefix, background=True)
        self.prefixes.insert(0, (prefix, self.adapter, snap))
        del self.prefixes[PREFIX_SLOTS:]
        return 0

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

    def set_fillers(self, ids):
        """draft_source's filler ids (the FILLERS that encode to one token); empty: derived from the vocab bytes."""
        n = len(ids)
        arr = _u32(ids) if n else np.zeros(1, np.uint32)
        self._ck(self.L.bcu_set_fillers(self.h, arr.ctypes.data_as(_lib.PU32), n))

    def set_encoder(self, encode):
        """normalize_draft's tokenizer: encode(bytes) -> list of ids (None: drafts are not normalized)."""
        if encode is None:
            self._enc = None
            self._ck(self.L.bcu_set_encoder(self.h, None, None))
            return

        def cb(user, text, n, out, cap):
            try:
                ids = encode(bytes(text[:n]))
            except Exception:
                return -1
            if ids is None or len(ids) > cap:
                return -1
            for i, v in enumerate(ids):
                out[i] = int(v)
            return len(ids)

        self._enc = _lib.ENCODE_FN(cb)  # kept alive as long as the model uses it
        self._ck(self.L.bcu_set_encoder(self.h, ctypes.cast(self._enc, ctypes.c_void_p), None))

    def set_emit(self, emit):
        """Streaming emission: emit(id) for every token decode outputs, as it lands (None: off)."""
        if emit is None:
            self._emit = None
            self._ck(self.L.bcu_set_emit(self.h, None, None))
            return
        self._emit = _lib.EMIT_FN(lambda user, tok: emit(int(tok)))
        self._ck(self.L.bcu_set_emit(self.h, ctypes.cast(self._emit, ctypes.c_void_p), None))

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


# -------------------------------------------------------------------- prefix files, host only
def hash_bytes(h, data):
    """hash_bytes (runtime/mod.rs:225-235)."""
    data = bytes(data)
    return _lib.lib().bcu_hash_bytes(h, data, len(data))


def kernel_hash():
    return _lib.lib().bcu_kernel_hash()


def prefix_path(directory, identity, ids):
    """Model::prefix_path (runtime/mod.rs:512-515)."""
    ids = _u32(ids)
    buf = ctypes.create_string_buffer(len(directory) + 64)
    s = _lib.lib().bcu_prefix_path(directory.encode(), identity, len(identity), ids.ctypes.data_as(_lib.PU32),
                                   len(ids), buf, len(buf))
    if s != _lib.OK:
        raise BackendError(s, "prefix path")
    return buf.value.decode()


def wait_saves():
    """Joins the background prefix writers."""
    _lib.lib().bcu_prefix_wait_saves()


def file_write(directory, identity, ids, parts):
    """The prefix file writer on host buffers (uint8 arrays), as bcu_prefix_save writes it."""
    ids = _u32(ids)
    parts = [np.ascontiguousarray(np.frombuffer(bytes(p), np.uint8)) for p in parts]
    ptrs = (ctypes.c_void_p * 4)(*[p.ctypes.data if p.size else None for p in parts])
    sizes = (ctypes.c_uint64 * 4)(*[p.size for p in parts])
    return _lib.lib().bcu_prefix_file_write(directory.encode(), identity, len(identity),
                                            ids.ctypes.data_as(_lib.PU32), len(ids), ptrs, sizes)


def file_read(directory, identity, ids, sizes):
    """The prefix file reader on host buffers: the parts as bytes, or None when there is no usable file."""
    ids = _u32(ids)
    bufs = [np.zeros(max(int(n), 1), np.uint8) for n in sizes]
    ptrs = (ctypes.c_void_p * 4)(*[b.ctypes.data for b in bufs])
    sz = (ctypes.c_uint64 * 4)(*[int(n) for n in sizes])
    found = ctypes.c_int32()
    s = _lib.lib().bcu_prefix_file_read(directory.encode(), identity, len(identity), ids.ctypes.data_as(_lib.PU32),
                                        len(ids), ptrs, sz, ctypes.byref(found))
    if s != _lib.OK:
        raise BackendError(s, "prefix file read")
    return [b[: int(n)].tobytes() for b, n in zip(bufs, sizes)] if found.value else None
